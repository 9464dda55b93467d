// IQ3_S x MXFP8 weight-streaming linear on the 5th-generation tensor cores
// (tcgen05, sm_100a), with the decoded weight operand kept in tensor memory.
//
// Same arithmetic as the reference (src/python/mambo/kernels/iq3_s_fp8.py:279-333):
// per 32-weight group g, P_g = sum_k E4M3(w) * E4M3(x) * 2^e(x, g) is summed by
// the tensor core in FP32 (block-scaled MMA: the activation's UE8M0 scale is
// applied in the MMA, an exact power of two), then out += P_g * d * (1 + 2*nibble_g)
// in FP32.
//
// One persistent CTA per SM walks a range of work units (128 weight rows x one
// 256-wide K block): a stream-K range, one row tile, or one K part of a row
// tile within a thread-block cluster. Roles:
//  * warp 0, weight producer: one bulk copy of the unit's tile-major record
//    (or five, one per IQ3_S field; evict-first) into a ring of weight stages,
//    and an L2 prefetch of the records `prefetch` units further on. A stage is
//    refilled as soon as the decoders have read it.
//  * activation producer warp: once the previous kernel has finished
//    (programmatic dependent launch), one 3D TMA copy of the unit's activation
//    block straight into the UMMA B-operand layout (16-byte K chunks x tokens;
//    rows past M read as zero) and one of its scale bytes, into a separate ring
//    that runs up to 8 units ahead of the MMAs.
//  * decoder warps (8 or 16): a thread owns one weight row (its TMEM lane) and
//    a quarter or half of the block; it reads its raw bytes with 128-bit loads,
//    expands each 4-weight code through a lane-private codebook in shared
//    memory, adds the sign bits and writes the E4M3 bytes to its TMEM lane with
//    tcgen05.st (a ring of 3 A operands). Weight rows' d and scale nibbles go
//    to a small shared buffer for the epilogue.
//  * warp 1, MMA: the converged warp elects one lane that issues 8 block-scaled
//    tcgen05.mma (A from TMEM, B from shared memory, M=128, N=16/32, K=32: one
//    per group) with descriptors formed once per unit, and commits them.
//  * 4 epilogue warps (one per TMEM lane quadrant): each thread owns one weight
//    row, reads the 8 group partials of its lane with tcgen05.ld, applies
//    d*(1+2*nibble) and accumulates in FP32 registers; finished rows go to the
//    output or to the deterministic split-K reduction (acq_rel counter,
//    CTA-ordered sum, or the cluster's rank 0). Before releasing a D buffer
//    they write the activation scales of the unit whose MMAs wait for that
//    buffer into TMEM (tcgen05.st, all four quadrants), so the MMA warp only
//    issues MMAs.
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

#include "kernels.cuh"
#include "tcgen05.cuh"
#include "iq3s_tm.cuh"
#include "mxfp8.cuh"

namespace mambo {

namespace {

constexpr int kRows = 128;                 // weight rows per unit = MMA M = TMEM lanes
using tm::kTableBytes;
constexpr int kEpiWarps = 4;
constexpr int kMaxStagesTm = 12;
constexpr int kRing = 3;  // decoded units in flight: A operands in TMEM, epilogue data in shared memory
constexpr uint32_t kBarBytes = 512;
using tm::kTableStageBytes;
using tm::kRecordBytes;

// Warps: weight producer, MMA, decoders, 4 epilogue, activation producer.
// Warps: weight producer, MMA, decoders, epilogue, two activation producers.
__host__ __device__ constexpr int tm_threads(int dec_warps) { return (4 + dec_warps + kEpiWarps) * 32; }
__host__ __device__ constexpr int tm_box_tokens(int nt) { return 8 * nt; }    // activation rows per B tile
// Activation tiles in flight (their own ring, filled ahead of the weights).
constexpr int kMaxXStages = 8;
__host__ __device__ constexpr int tm_xstages(int nt) { return nt == 1 ? 8 : nt == 2 ? 6 : 4; }
// Fused quantization: a ring of bf16 activation boxes (one K block of the
// token tile, [tokens][256 bf16]) that the activation warp quantizes into the
// slots above. Its barriers follow the TMEM address slot in the barrier area.
// An even count: a warp refills the slot of each of its own units (every other one).
__host__ __device__ constexpr int tm_bstages(int nt) { return nt == 1 ? 4 : 2; }
constexpr uint32_t kBfRowBytes = 512;
constexpr int kBfBarIndex = 2 * kMaxStagesTm + 2 * kMaxXStages + 2 * kRing + 6;
static_assert(kBfBarIndex + 4 <= (int)(kBarBytes / 8), "barrier area");
__host__ __device__ constexpr int tm_nmma(int nt) { return nt == 4 ? 32 : 16; }  // MMA N
// TMEM columns: the A ring at [0, 64*kRing), then D (8 groups x N columns),
// double-buffered unless that would not fit in 512 columns (N = 32), then the
// scale factors: A's (all 2^0) and a ring of B's (8 columns a unit: K blocks
// 0-3 and 4-7 of the unit in byte 0-3 of columns +0 and +4).
// The MMA reads a scale-factor matrix from 4 columns starting at the address
// it is given (column + row / 32), so every such address is a multiple of 4.
constexpr uint32_t kTmemD = 64u * kRing;
__host__ __device__ constexpr int tm_d_buffers(int nt) { return nt != 4 ? 2 : 1; }
__host__ __device__ constexpr uint32_t tm_sfa_col(int nt) { return kTmemD + tm_d_buffers(nt) * 8u * tm_nmma(nt); }
__host__ __device__ constexpr uint32_t tm_sfb_col(int nt) { return tm_sfa_col(nt) + 16u; }
__host__ __device__ constexpr uint32_t tm_tmem_cols(int nt) { return tm_sfb_col(nt) + 8u * kRing <= 256u ? 256u : 512u; }
static_assert(tm_sfb_col(1) + 8u * kRing <= 512u && tm_sfb_col(2) + 8u * kRing <= 512u &&
                  tm_sfb_col(4) + 8u * kRing <= 512u,
              "TMEM plan exceeds 512 columns");
static_assert(tm_sfa_col(1) % 16u == 0 && tm_sfa_col(2) % 16u == 0 && tm_sfa_col(4) % 16u == 0,
              "scale-factor columns must stay aligned");
__host__ __device__ constexpr uint32_t align_up_tm(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// A weight stage: the IQ3_S fields of a unit (one tile-major record, or the
// five fields copied separately to the same offsets). An activation slot: the
// B tile, then the scale bytes. Weight stages are 128-byte aligned, the
// activation slots (after the stages) 1024-byte aligned.
struct TmLayout {
  uint32_t qs, signs, qh, d, scales, stage;
  uint32_t b, xs, xslot;
  uint32_t w, aux;  // one of kRing epilogue buffers: rows' (d, scale word)
};

// q4k: Q4_K records (kQ4kRecordBytes; no codebook, 16 bytes of epilogue data per row).
__host__ __device__ inline TmLayout tm_layout(int nt, bool q4k = false) {
  TmLayout L{};
  L.qs = 0;
  L.signs = kRows * 64;         // 8192
  L.qh = L.signs + kRows * 32;  // 12288
  L.d = L.qh + kRows * 8;       // 13312
  L.scales = L.d + kRows * 2;   // 13568
  L.stage = q4k ? kQ4kRecordBytes : L.scales + kRows * 4;  // 14080 = kRecordBytes
  L.b = 0;
  L.xs = 256u * tm_box_tokens(nt);  // activation scale bytes: [tokens][16] (two K blocks' groups)
  L.xslot = align_up_tm(L.xs + 16u * tm_box_tokens(nt), 1024);
  L.w = 0;
  L.aux = kRows * (q4k ? 16 : 8);
  return L;
}

// The region after the epilogue ring: the IQ3_S decoders' codebook staging,
// or for Q4_K the epilogue warps' copies of a unit's activation group sums
// (4 warps x 8*nt tokens x 8 floats).
__host__ __device__ constexpr uint32_t tm_stage_region(int nt, bool q4k) {
  return q4k && 1024u * (uint32_t)nt > kTableStageBytes ? 1024u * (uint32_t)nt : kTableStageBytes;
}

// kparts > 1: rank 0 of each cluster also holds the other ranks' partials.
__host__ __device__ inline uint32_t tm_smem_bytes(int nt, int stages, int kparts, bool fused = false,
                                                  bool q4k = false) {
  const TmLayout L = tm_layout(nt, q4k);
  const uint32_t cpart = kparts > 1 ? (uint32_t)(kparts - 1) * kRows * 8u * nt * 4u : 0u;
  const uint32_t bf = fused ? 128u + (uint32_t)tm_bstages(nt) * tm_box_tokens(nt) * kBfRowBytes : 0u;
  return (q4k ? 0u : kTableBytes) + 1024 + align_up_tm(stages * L.stage, 1024) + tm_xstages(nt) * L.xslot +
         kRing * L.aux + tm_stage_region(nt, q4k) + kBarBytes + cpart + bf;
}

__device__ __forceinline__ int unit_begin_tm(int cta, int grid, int units) {
  return (int)(((int64_t)cta * units) / grid);
}
__device__ __forceinline__ int cta_of_unit_tm(int u, int grid, int units) {
  return (int)((((int64_t)u + 1) * grid - 1) / units);
}

// Where one linear's results go.
struct OutView {
  void* out;
  int64_t ldo;
  int out_bf16;
  int n_rows;
  int m;
};

// Where the MXFP8 quantization of a linear's output goes, for the next linear
// (q: E4M3 bytes, s: UE8M0 codes; null q: none; n_rows % 32 == 0). Only
// kernels instantiated with kQ carry it.
struct QuantView {
  uint8_t* q;
  int64_t ldq;
  uint8_t* s;
  int64_t lds;
};

// The MXFP8 quantization of 32 consecutive outputs (rows row - lane .. row -
// lane + 31, one per lane) of token `tok`: one MXFP8 group of the next
// linear's activation row, quantized as the standalone quantizer quantizes
// the stored values (largest magnitude by one warp reduction over the bit
// patterns, where a NaN orders above every number and gives the scale code
// 0xFF; values times 2^-e rounded to nearest even with saturation). Called by
// all 32 lanes together. Out of line: only launches asked for the quantized
// output reach it, and the store path of the others keeps its size.
__device__ __noinline__ void quantize_out_tm(uint8_t* q, int64_t ldq, uint8_t* sc, int64_t lds, int n_rows,
                                            int out_bf16, int row, int tok, float v) {
  const bool in = row < n_rows;  // the same for the whole warp (n_rows % 32 == 0)
  if (out_bf16) v = __bfloat162float(__float2bfloat16_rn(v));  // what a reader of out sees
  const uint32_t mag = in ? (__float_as_uint(v) & 0x7FFFFFFFu) : 0u;
  const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, mag);
  const uint32_t code = mxfp8_scale_code(__uint_as_float(amax));
  const float inv = e8m0_to_float(code == 0xFFu ? 0u : 254u - code);
  if (in) {
    q[(int64_t)tok * ldq + row] = (uint8_t)(cvt_e4m3x2_rn(v * inv, 0.f) & 0xFFu);
    if ((row & 31) == 0) sc[(int64_t)tok * lds + row / 32] = (uint8_t)code;
  }
}

// Stores the final value v of (row, tok). Called by all 32 lanes of a warp
// together, for 32 consecutive rows (a warp's lanes are consecutive TMEM rows
// of a 128-row tile) and one token; with kQ and qv.q set, also the MXFP8
// quantization of those 32 outputs for the next linear.
template <bool kQ>
__device__ __forceinline__ void store_out_tm(const OutView& o, const QuantView& qv, int row, int tok, float v) {
  if (row < o.n_rows && tok < o.m) {
    if (o.out_bf16) {
      reinterpret_cast<__nv_bfloat16*>(o.out)[(int64_t)tok * o.ldo + row] = __float2bfloat16_rn(v);
    } else {
      reinterpret_cast<float*>(o.out)[(int64_t)tok * o.ldo + row] = v;
    }
  }
  if constexpr (kQ) {
    if (qv.q != nullptr && tok < o.m)  // warp-uniform condition
      quantize_out_tm(qv.q, qv.ldq, qv.s, qv.lds, o.n_rows, o.out_bf16, row, tok, v);
  }
}

// Fused all-reduce of a row-split linear, for one warp's 32 rows (lane = row)
// and TOK tokens, called where the rows' final sums over this rank's K slice
// are formed. Each value travels with the launch's tag (epoch + 1) in one
// 8-byte word, which a single aligned store writes and a single load reads
// whole: a reader that sees the tag sees the value, with no fence or flag
// (the low-latency scheme of NCCL's LL protocol). This rank's partial goes into
// every rank's slot for this rank (plain stores, over NVLink for peers); then
// each lane polls its row of every rank's slot here until the tags carry this
// launch's, and sums the partials in rank order, so every rank forms the
// identical result. The slots alternate between two buffers by epoch parity: a
// rank one launch ahead writes the other buffer, and none gets two launches
// ahead (it needs this rank's next partials). False when a rank's partial did
// not arrive within the wait limit (recorded as a timeout at kSiteArPeer).
template <int TOK>
__device__ bool ar_exchange(const GemvAr& ar, uint32_t epoch, int row, int lane, float (&acc)[TOK]) {
  static_assert(TOK % 2 == 0, "values go in pairs");
  const uint32_t par = epoch & 1u, tag = epoch + 1u;
  const size_t slot = (size_t)ar.max_rows * TOK;  // 8-byte words of one source rank's partial
  const size_t row_off = (size_t)row * TOK;
  for (int j = 0; j < ar.world; ++j) {
    uint2* dst = reinterpret_cast<uint2*>(ar.base[j]) + ((size_t)par * ar.world + ar.rank) * slot + row_off;
#pragma unroll
    for (int t = 0; t < TOK; t += 2)
      asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst + t), "r"(__float_as_uint(acc[t])),
                   "r"(tag), "r"(__float_as_uint(acc[t + 1])), "r"(tag)
                   : "memory");
  }
  const uint2* src = reinterpret_cast<const uint2*>(ar.base[ar.rank]) + (size_t)par * ar.world * slot + row_off;
  float sum[TOK];
#pragma unroll
  for (int t = 0; t < TOK; ++t) sum[t] = 0.f;
  bool ok = true;
  const unsigned long long limit = g_wait_limit_ns;
  unsigned long long t0 = 0;
  for (int j = 0; j < ar.world; ++j) {
#pragma unroll
    for (int t = 0; t < TOK; t += 2) {
      uint32_t a, ta, b, tb;
      for (uint32_t i = 0;; ++i) {
        asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(a), "=r"(ta), "=r"(b), "=r"(tb)
                     : "l"(src + (size_t)j * slot + t)
                     : "memory");
        if ((ta == tag && tb == tag) || !ok) break;
        if (i == 0) t0 = globaltimer_ns();
        __nanosleep(20);
        if ((i & 15u) == 15u && (*(volatile int*)&g_device_status.code != 0 || globaltimer_ns() - t0 > limit)) {
          record_timeout(kSiteArPeer);
          ok = false;
        }
      }
      sum[t] += __uint_as_float(a);
      sum[t + 1] += __uint_as_float(b);
    }
  }
#pragma unroll
  for (int t = 0; t < TOK; ++t) acc[t] = sum[t];
  return __all_sync(0xFFFFFFFFu, ok);
}

// Q4_K: eight stored codes of one 32-bit word (bits 0-15: four values of one
// group, bits 16-31: four of the next; each (v > 0) << 3 | (|v| - 1) / 2 for
// the odd integer v = 2q - 15) -> the E4M3 bytes of v, four per output word.
// The magnitude comes from an 8-byte table (prmt on the low three bits); a
// selector nibble with bit 3 set picks the replicated sign of a 0x01 byte
// (0x00), a clear one the byte itself (0x01), which times 128 is the sign bit.
__device__ __forceinline__ void q4k_e4m3(uint32_t w, uint32_t& lo, uint32_t& hi) {
  constexpr uint32_t kOdd0 = 0x4E4A4438u, kOdd1 = 0x57555351u;  // E4M3 of 1, 3, 5, ..., 15
  const uint32_t sel = w & 0x77777777u, wh = w >> 16;
  const uint32_t a0 = prmt(kOdd0, kOdd1, sel), a1 = prmt(kOdd0, kOdd1, sel >> 16);
  const uint32_t n0 = prmt(0x01010101u, 0x01010101u, w), n1 = prmt(0x01010101u, 0x01010101u, wh);
  lo = n0 * 128u + a0;
  hi = n1 * 128u + a1;
}

// The item of a grouped launch that holds unit u, searching upwards from item l.
__device__ __forceinline__ int group_item(const GemvGroup& g, int u, int l) {
  while (l + 1 < g.count && g.items[l + 1].unit0 <= u) ++l;
  return l;
}

// Sums the partials of one weight row (local row rl of tile rt) over the
// contributing CTAs in CTA order and stores it; the partials of CTA `self`
// come from `acc` (its registers) instead of memory. Loads for several
// contributors are in flight together.
// tile: the row tile's number; tile_of(u): the row tile holding unit u;
// begin_of(c): the first unit of CTA c.
template <int TOK, bool kQ, class TileOf, class BeginOf>
__device__ __forceinline__ void sum_partials(const float* partials, BeginOf begin_of, const OutView& o,
                                             const QuantView& qv, int tile,
                                             int rl, int row, int self, int c_first, int c_last, TileOf tile_of,
                                             const float (&acc)[TOK]) {
#pragma unroll
  for (int t0 = 0; t0 < TOK; t0 += 8) {
    float sum[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) sum[t] = 0.f;
    constexpr int kB = TOK <= 8 ? 4 : 2;  // contributors whose loads are in flight together
#pragma unroll 1
    for (int c0 = c_first; c0 <= c_last; c0 += kB) {
      float4 v[kB][2];
#pragma unroll
      for (int j = 0; j < kB; ++j) {
        const int c = c0 + j;
        if (c <= c_last && c != self) {
          const int cs = (tile == tile_of(begin_of(c))) ? 0 : 1;
          const float4* src = reinterpret_cast<const float4*>(partials + ((size_t)(c * 2 + cs) * 128 + rl) * TOK + t0);
          v[j][0] = __ldcg(src);
          v[j][1] = __ldcg(src + 1);
        } else {
          float x[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) x[t] = 0.f;
          if (c == self) {
#pragma unroll
            for (int t = 0; t < 8; ++t) x[t] = acc[t0 + t];
          }
          v[j][0] = make_float4(x[0], x[1], x[2], x[3]);
          v[j][1] = make_float4(x[4], x[5], x[6], x[7]);
        }
      }
#pragma unroll
      for (int j = 0; j < kB; ++j) {
        if (c0 + j <= c_last) {
          sum[0] += v[j][0].x; sum[1] += v[j][0].y; sum[2] += v[j][0].z; sum[3] += v[j][0].w;
          sum[4] += v[j][1].x; sum[5] += v[j][1].y; sum[6] += v[j][1].z; sum[7] += v[j][1].w;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) store_out_tm<kQ>(o, qv, row, t0 + t, sum[t]);
  }
}

}  // namespace

// G: GemvNoGroup (one linear, described by p and maps) or GemvGroup (a grouped
// launch: units of every item back to back, stream-K; weights packed,
// activations bf16 quantized here).
// kQ: the launch also writes its output's MXFP8 quantization (QuantView);
// launches without it run a kernel that has none of that code.
// kQ4K: Q4_K weights (q4k records; prequantized activations with their group
// sums, p.xsum): the decoders turn the stored codes into E4M3 operands 2q - 15
// and the epilogue applies d*s_g/2 and the group's constant term
// (7.5*d*s_g - dmin*m_g) times the activation group sum.
template <int NT, int kDecWarps, class G, bool kQ, bool kQ4K = false>
__global__ void __launch_bounds__(tm_threads(kDecWarps), 1)
    iq3s_gemv_tm_kernel(const __grid_constant__ GemvTmParams p, const __grid_constant__ GemvTmMaps maps,
                        const __grid_constant__ G grp) {
  constexpr bool kPre = std::is_same<G, GemvGroupPre>::value;  // a group with its activation tiles made beforehand
  constexpr bool kGroup = std::is_same<G, GemvGroup>::value || kPre;
  constexpr bool kAR = std::is_same<G, GemvAr>::value;  // row split with its all-reduce fused
  constexpr int TOK = 8 * NT;             // tokens the epilogue keeps
  constexpr int NM = tm_nmma(NT);         // MMA N
  constexpr int BOX = tm_box_tokens(NT);  // activation rows in a B tile
  constexpr uint32_t kIdesc = tc::idesc_mx_e4m3(kRows, NM, 0, 0);
  constexpr int kDBuf = tm_d_buffers(NT);
  constexpr uint32_t kCols = tm_tmem_cols(NT);
  constexpr int kParts = kDecWarps / 4;  // decoder threads per weight row
  constexpr int kGroups = 8 / kParts;    // 32-weight groups per decoder thread and unit
  // B tile [16-byte K chunk][R tokens][16 bytes]: K-direction core-matrix
  // stride R*16, token-group stride 128. R = BOX when the kernel quantizes the
  // activations itself; with TMA loads R = the box rows (the launch's tokens),
  // so that no box holds out-of-bounds rows (TMA zero-fills them one 16-byte
  // line at a time, which made a one-token launch slower than an eight-token
  // one). A core matrix's rows past R read the next chunk's rows: they feed
  // only D columns of tokens past M, which are never read. With 8 tokens the
  // MMA's rows 8-15 repeat rows 0-7 (stride 0) and their results are never read.
  const uint32_t xrows = (!kGroup && p.x_bf16 == nullptr && p.box_rows > 0) ? (uint32_t)p.box_rows : (uint32_t)BOX;
  const uint32_t kBytesX = xrows * 256u + xrows * 16u;
  const uint32_t kLbo = xrows * 16u;
  constexpr uint32_t kSbo = NT == 1 ? 0u : 128u;
  constexpr int kEpiWarp0 = 2 + kDecWarps, kXWarp0 = kEpiWarp0 + kEpiWarps;
  constexpr int AS = tm_xstages(NT);
  static_assert(kDecWarps == 8 || kDecWarps == 16, "8 or 16 decoder warps");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const TmLayout L = tm_layout(NT, kQ4K);
  constexpr uint32_t kTableRegion = kQ4K ? 0u : (uint32_t)kTableBytes;  // no codebook for Q4_K
  constexpr uint32_t kRecBytes = kQ4K ? kQ4kRecordBytes : (uint32_t)kRecordBytes;
  static_assert(!(kQ4K && (kQ || (kGroup && !kPre))), "Q4_K runs single linears or pre-quantized groups");
  // The codebook sits at the start of dynamic shared memory (a link-time
  // constant address); the stages follow, aligned to 1024 bytes at run time.
  // (Offsets from smem_raw keep the pointers in the shared address space, so
  // every access below compiles to a shared-memory instruction.)
  uint8_t* table = smem_raw;
  uint8_t* st0 = smem_raw + kTableRegion + ((1024u - ((smem_u32(smem_raw) + kTableRegion) & 1023u)) & 1023u);
  uint8_t* x0 = st0 + align_up_tm((uint32_t)p.stages * L.stage, 1024);  // activation slots
  uint8_t* aux0 = x0 + (size_t)AS * L.xslot;
  uint32_t* tstage = reinterpret_cast<uint32_t*>(aux0 + kRing * L.aux);
  constexpr uint32_t kStageRegion = tm_stage_region(NT, kQ4K);
  uint64_t* bars = reinterpret_cast<uint64_t*>(aux0 + kRing * L.aux + kStageRegion);
  float* cpart = reinterpret_cast<float*>(aux0 + kRing * L.aux + kStageRegion + kBarBytes);  // cluster partials
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStagesTm + 2 * kMaxXStages + 2 * kRing + 5);
  const uint32_t bar0 = smem_u32(bars);
  // Barriers: per weight stage wfull (landed) and empty (decoded); per
  // activation slot xfull (landed) and xempty (its MMAs complete); per ring
  // slot afull (A decoded and the epilogue's row data written), efree
  // (epilogue done with the slot); per D buffer mdone (MMAs complete); edone
  // (epilogue finished); cred (cluster K-split: the other CTAs of the cluster
  // have written their partials into this CTA's shared memory; used in the
  // cluster's rank 0); sfinit (scales of the first units written).
  const uint32_t kWfull = bar0, kEmpty = bar0 + 8 * kMaxStagesTm;
  const uint32_t kXfull = bar0 + 16 * kMaxStagesTm, kXempty = kXfull + 8 * kMaxXStages;
  const uint32_t kAfull = kXempty + 8 * kMaxXStages, kEfree = kAfull + 8 * kRing;
  const uint32_t kMdone = kEfree + 8 * kRing, kEdone = kMdone + 16, kCred = kEdone + 8, kSfInit = kCred + 8;
  const uint32_t kBfull = bar0 + 8 * kBfBarIndex;  // bf16 boxes landed (fused quantization)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work range: with kparts > 0 each row tile is split into kparts K ranges,
  // one per CTA of a cluster (rank = K part); otherwise a stream-K range.
  // Stream-K ranges: a grouped launch takes them from the host's table,
  // a single linear splits its units evenly.
  auto unit_begin = [&](int c) -> int {
    if constexpr (kGroup) return grp.cta_start[c];
    else return unit_begin_tm(c, gridDim.x, p.total_units);
  };
  auto cta_of_unit = [&](int u) -> int {
    if constexpr (kGroup) {
      int lo = 0, hi = (int)gridDim.x - 1;  // last CTA whose range starts at or before u
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (grp.cta_start[mid] <= u) lo = mid;
        else hi = mid - 1;
      }
      return lo;
    } else {
      return cta_of_unit_tm(u, gridDim.x, p.total_units);
    }
  };
  int u0, u1;
  if (p.kparts > 0) {
    const int t = blockIdx.x / p.kparts, k = blockIdx.x % p.kparts;
    u0 = t * p.n_blocks + (int)((int64_t)k * p.n_blocks / p.kparts);
    u1 = t * p.n_blocks + (int)((int64_t)(k + 1) * p.n_blocks / p.kparts);
  } else {
    u0 = unit_begin(blockIdx.x);
    u1 = unit_begin(blockIdx.x + 1);
  }
  const int n_units = u1 - u0;
  const int S = p.stages;

  // Decoder threads fetch the 2 KB codebook now, so that its global-memory
  // latency overlaps the barrier and TMEM set-up below.
  uint32_t tw[512 / (kDecWarps * 32)];
  if (!kQ4K && warp >= 2 && warp < kEpiWarp0) {
#pragma unroll
    for (int j = 0; j < 512 / (kDecWarps * 32); ++j) tw[j] = __ldg(p.table + (threadIdx.x - 64) + j * kDecWarps * 32);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(kWfull + 8 * s, 1);
      mbar_init(kEmpty + 8 * s, kDecWarps);
    }
    for (int x = 0; x < AS; ++x) {
      mbar_init(kXfull + 8 * x, 1);
      mbar_init(kXempty + 8 * x, 1);  // MMA commit
    }
    for (int r = 0; r < kRing; ++r) {
      mbar_init(kAfull + 8 * r, kDecWarps);
      mbar_init(kEfree + 8 * r, kEpiWarps);
    }
    for (int b = 0; b < 2; ++b) mbar_init(kMdone + 8 * b, 1);
    mbar_init(kEdone, kEpiWarps);
    mbar_init(kCred, p.kparts > 1 ? (p.kparts - 1) * kEpiWarps : 1);
    mbar_init(kSfInit, kEpiWarps);
    for (int s = 0; s < tm_bstages(NT); ++s) mbar_init(kBfull + 8 * s, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tc::alloc(smem_u32(tmem_slot), kCols);
    tc::relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (p.kparts > 1) cluster_sync_all();  // every CTA's barriers initialized before any remote arrival
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  // ------------------------------------------------------------------ weight producer
  // The whole warp issues: lane f < 5 copies weight field f, so one warp
  // instruction starts all five copies of a unit (a copy instruction costs
  // its thread ~100 cycles or more to issue). Weights do not depend on the
  // previous kernel: no wait for it.
  if (warp == 0) {
    const uint64_t policy = l2_policy_evict_first();
    const uint8_t* fptr = lane == 0 ? p.qs : lane == 1 ? p.signs : lane == 2 ? p.qh : lane == 3 ? p.d : p.scales;
    const uint32_t fbpr = lane == 0 ? 64u : lane == 1 ? 32u : lane == 2 ? 8u : lane == 3 ? 2u : 4u;  // bytes per row
    const uint32_t foff = lane == 0 ? L.qs : lane == 1 ? L.signs : lane == 2 ? L.qh : lane == 3 ? L.d : L.scales;
    // Rows of the unit's tile (a multiple of 8) and their index in each field.
    auto tile = [&](int u, uint32_t& rows, size_t& base) {
      const int n0 = (u / p.n_blocks) * kRows;
      rows = (uint32_t)min(kRows, p.n_rows - n0);
      base = (size_t)(u % p.n_blocks) * p.n_rows + n0;
    };
    // Tile-major record of unit u (units visited in ascending order through `hint`).
    auto record = [&](int u, int& hint) -> const uint8_t* {
      if constexpr (kGroup) {
        hint = group_item(grp, u, hint);
        return grp.items[hint].packed + (size_t)(u - grp.items[hint].unit0) * kRecBytes;
      } else {
        return p.packed + (size_t)u * kRecBytes;
      }
    };
    int issue_hint = 0, prefetch_hint = 0;
    auto issue_weights = [&](int it, int s) {
      const uint32_t full = kWfull + 8 * s;
      const uint32_t st = smem_u32(st0 + (size_t)s * L.stage);
      if (kGroup || p.packed) {
        // Tile-major records have the stage's layout: one copy per unit.
        const uint8_t* rec = record(u0 + it, issue_hint);
        if (lane == 0) {
          mbar_arrive_expect_tx(full, kRecBytes);
          bulk_load_hint(st, rec, kRecBytes, full, policy);
        }
      } else {
        uint32_t rows;
        size_t base;
        tile(u0 + it, rows, base);
        if (lane == 0) mbar_arrive_expect_tx(full, rows * 110u);
        __syncwarp();
        if (lane < 5) bulk_load_hint(st + foff, fptr + base * fbpr, rows * fbpr, full, policy);
      }
      __syncwarp();
    };
    auto prefetch = [&](int it) {
      if (kGroup || p.packed) {
        const uint8_t* rec = record(u0 + it, prefetch_hint);
        if (lane == 0) bulk_prefetch_l2(rec, kRecBytes);
      } else {
        uint32_t rows;
        size_t base;
        tile(u0 + it, rows, base);
        if (lane < 5) bulk_prefetch_l2(fptr + base * fbpr, rows * fbpr);
      }
      __syncwarp();
    };
    const int pre = min(S, n_units);
    for (int it = 0; it < pre; ++it) issue_weights(it, it);
    int pf = pre;
    for (; pf < min(n_units, pre + p.prefetch); ++pf) prefetch(pf);
    int es = pre % S;
    uint32_t eph = (uint32_t)(pre / S) & 1u;  // stage and phase of unit `it`
    for (int it = pre; it < n_units; ++it) {
      const bool ok = mbar_wait_bounded(kEmpty + 8 * es, eph ^ 1, kSiteGemvEmpty);
      const int s = es;
      if (++es == S) {
        es = 0;
        eph ^= 1;
      }
      if (!__all_sync(0xFFFFFFFFu, ok)) return;
      issue_weights(it, s);
      // L2 prefetch of the units after the ones already requested. (The window
      // once began at the unit just issued: with no prefetch distance every
      // unit was requested twice, and the copy engine spent its time on both.)
      pf = max(pf, it + 1);
      for (; pf < min(n_units, it + 1 + p.prefetch); ++pf) prefetch(pf);
    }
    return;
  }

  // ------------------------------------------------------------------ activation producers
  // Activation tiles (B operand and scale bytes of a K block) once the previous
  // kernel has finished (programmatic dependent launch), AS units ahead: slot
  // j % AS is refilled when the MMAs of unit j - AS have completed. TMA
  // copies need one warp; fused quantization takes both, every other unit.
  if (warp >= kXWarp0) {
    const int xw = warp - kXWarp0;
    if constexpr (kPre) {
      // Tiles quantized by the pre-pass: three bulk copies per unit (the B
      // tile and the rows of both scale blocks) complete the slot's barrier;
      // the two warps take alternate units, following their item with a
      // forward cursor.
      pdl_wait();
      int l = group_item(grp, u0 + xw, 0);
      int v = u0 + xw - grp.items[l].unit0, nb = grp.items[l].n_blocks;
      int units = ((grp.items[l].n_rows + kRows - 1) / kRows) * nb;
      int kb = v % nb;
      for (int j = xw; j < n_units; j += 2) {
        const int x = j % AS;
        if (j >= AS && !__all_sync(0xFFFFFFFFu, mbar_wait_bounded(kXempty + 8 * x, ((j / AS) & 1) ^ 1, kSiteGemvEmpty)))
          return;
        if (lane == 0) {
          const uint8_t* src = grp.xtiles + (size_t)(grp.items[l].xt0 + kb) * gemv_xtile_bytes(NT);
          const uint32_t dst = smem_u32(x0 + (size_t)x * L.xslot), full = kXfull + 8 * x;
          mbar_arrive_expect_tx(full, gemv_xtile_bytes(NT));
          bulk_load(dst + L.b, src, 256u * BOX, full);
          bulk_load(dst + L.xs, src + 256u * BOX, 16u * BOX, full);
          bulk_load(dst + L.xs + 512u, src + 272u * BOX, 16u * BOX, full);
        }
        __syncwarp();
        v += 2;
        kb += 2;
        while (kb >= nb) kb -= nb;
        while (v >= units && l + 1 < grp.count) {  // into the next item
          v -= units;
          ++l;
          nb = grp.items[l].n_blocks;
          units = ((grp.items[l].n_rows + kRows - 1) / kRows) * nb;
          kb = v % nb;
        }
      }
      return;
    }
    const bool fused = kGroup || p.x_bf16 != nullptr;
    if (xw != 0 && !fused) return;
    const uint64_t keep = l2_policy_evict_last();  // every CTA reads them
    if constexpr (kGroup) {
      if (xw == 0 && lane < grp.count) tma_prefetch_desc(&grp.xb[lane]);
    } else if (lane == 0 && xw == 0) {
      if (p.x_bf16) {
        tma_prefetch_desc(&maps.xb);
      } else {
        tma_prefetch_desc(&maps.x);
        tma_prefetch_desc(&maps.xs);
      }
    }
    pdl_wait();
    if (fused) {
      // Fused quantization (the standalone quantizer's arithmetic): the bf16
      // box of each K block arrives by TMA, BS units ahead. A lane quantizes
      // one 32-value group of one token (4 tokens x 8 groups a pass; with one
      // token, four lanes a group), reading its four 16-byte chunks in an
      // order rotated by token so that each quarter warp hits all banks, and
      // writes the E4M3 bytes straight into
      // the B tile [16-byte K chunk][token][16 bytes], the scale code into
      // two 512-byte scale blocks ([token][16 bytes], groups 0-3 then 4-7 in
      // bytes 0-3), which the MMA warp copies to TMEM. Rows past M are left
      // as they are: their D columns are never read.
      constexpr int BS = tm_bstages(NT);
      constexpr uint32_t kBoxBytes = BOX * kBfRowBytes;
      const uint32_t cpart_bytes = p.kparts > 1 ? (uint32_t)(p.kparts - 1) * kRows * 8u * NT * 4u : 0u;
      uint8_t* xb0 = reinterpret_cast<uint8_t*>(cpart) + cpart_bytes;
      xb0 += (128u - (smem_u32(xb0) & 127u)) & 127u;
      const int tl = lane & 3, g = lane >> 2;
      // Unit cursor: item, unit within the item, K block. It only moves to
      // units of this CTA's range (which exist), by a few units at a time.
      struct XCursor {
        int j, l, v, kb, nb, units;
      };
      auto cursor_at = [&](int j) {
        XCursor c{j, 0, u0 + j, 0, p.n_blocks, 0x7FFFFFFF};
        if constexpr (kGroup) {
          c.l = group_item(grp, u0 + j, 0);
          const GemvItem& gi = grp.items[c.l];
          c.nb = gi.n_blocks;
          c.units = ((gi.n_rows + kRows - 1) / kRows) * gi.n_blocks;
          c.v = u0 + j - gi.unit0;
        }
        c.kb = c.v % c.nb;
        return c;
      };
      auto move_to = [&](XCursor& c, int j) {
        const int d = j - c.j;
        c.j = j;
        c.v += d;
        c.kb += d;
        while (c.kb >= c.nb) c.kb -= c.nb;
        if constexpr (kGroup) {
          while (c.v >= c.units && c.l + 1 < grp.count) {  // into the next item
            c.v -= c.units;
            const GemvItem& gi = grp.items[++c.l];
            c.nb = gi.n_blocks;
            c.units = ((gi.n_rows + kRows - 1) / kRows) * gi.n_blocks;
            c.kb = c.v % c.nb;
          }
        }
      };
      XCursor ic = cursor_at(xw), qc = ic;  // next box to issue, unit being quantized
      auto issue_box = [&](int j) {  // lane 0: the bf16 box of unit j
        move_to(ic, j);
        const CUtensorMap* map = &maps.xb;
        if constexpr (kGroup) map = &grp.xb[ic.l];
        const uint32_t bar = kBfull + 8 * (j % BS);
        mbar_arrive_expect_tx(bar, kBoxBytes);
        tma_load_2d(smem_u32(xb0 + (size_t)(j % BS) * kBoxBytes), map, ic.kb * 256, 0, bar, keep);
      };
      if (lane == 0)
        for (int j = xw; j < BS && j < n_units; j += 2) issue_box(j);
      for (int j = xw; j < n_units; j += 2) {
        const int x = j % AS;
        bool ok = mbar_wait_bounded(kBfull + 8 * (j % BS), (uint32_t)(j / BS) & 1u, kSiteGemvFull);
        if (j >= AS) ok = ok && mbar_wait_bounded(kXempty + 8 * x, ((j / AS) & 1) ^ 1, kSiteGemvEmpty);
        if (!__all_sync(0xFFFFFFFFu, ok)) return;
        const uint8_t* box = xb0 + (size_t)(j % BS) * kBoxBytes;
        uint8_t* sl = x0 + (size_t)x * L.xslot;
        move_to(qc, j);
        int mq = p.m;
        if constexpr (kGroup) mq = grp.items[qc.l].m;
        if (mq <= 1) {
          // One token: four lanes per group (one 16-byte chunk each). From two tokens
          // one lane per group takes fewer passes (two tokens: one pass, not two).
          for (int t = 0; t < mq; ++t) {
            const uint4 c = *reinterpret_cast<const uint4*>(box + t * kBfRowBytes + lane * 16);
            uint2 q;
            const uint32_t code = mxfp8_quad_bf16_rne(c, q);
            *reinterpret_cast<uint2*>(sl + L.b + ((2 * g + (tl >> 1)) * BOX + t) * 16 + (tl & 1) * 8) = q;
            if (tl == 0) sl[L.xs + (g >> 2) * 512 + t * 16 + (g & 3)] = (uint8_t)code;
          }
        } else {
          for (int t = tl; t < mq; t += 4) {
            uint4 c[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              c[i] = *reinterpret_cast<const uint4*>(box + t * kBfRowBytes + g * 64 + ((i + tl) & 3) * 16);
            uint2 q[4];
            const uint32_t code = mxfp8_group32_bf16_rne(c, q);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int ch = (i + tl) & 3;  // 8-value chunk of the group held in c[i]
              *reinterpret_cast<uint2*>(sl + L.b + ((2 * g + (ch >> 1)) * BOX + t) * 16 + (ch & 1) * 8) = q[i];
            }
            sl[L.xs + (g >> 2) * 512 + t * 16 + (g & 3)] = (uint8_t)code;
          }
        }
        // The MMA reads the tile through the async proxy, and the next TMA
        // load overwrites the bf16 box just read.
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(kXfull + 8 * x);
          if (j + BS < n_units) issue_box(j + BS);
        }
        __syncwarp();
      }
      return;
    }
    int kb = u0 % p.n_blocks;
    for (int j = 0; j < n_units; ++j, kb = (kb + 1 == p.n_blocks) ? 0 : kb + 1) {
      const int x = j % AS;
      if (j >= AS) {
        const bool ok = mbar_wait_bounded(kXempty + 8 * x, ((j / AS) & 1) ^ 1, kSiteGemvEmpty);
        if (!__all_sync(0xFFFFFFFFu, ok)) return;
      }
      const uint32_t full = kXfull + 8 * x, slot = smem_u32(x0 + (size_t)x * L.xslot);
      if (lane == 0) {
        mbar_arrive_expect_tx(full, kBytesX);
        tma_load_3d(slot + L.b, &maps.x, 0, 0, kb * 16, full, keep);
        tma_load_2d(slot + L.xs, &maps.xs, (kb >> 1) * 16, 0, full, keep);
      }
      __syncwarp();
    }
    return;
  }

  // ------------------------------------------------------------------ MMA
  if (warp == 1) {
    for (int it = 0; it < n_units; ++it) {
      const int r = it % kRing, x = it % AS, db = kDBuf == 2 ? (it & 1) : 0;
      // The D buffer is free once the epilogue is done with the unit that used it last.
      const int prev = it - kDBuf;
      bool ok = mbar_try_wait(kAfull + 8 * r, (it / kRing) & 1);
      bool ok2 = mbar_try_wait(kXfull + 8 * x, (it / AS) & 1);
      // The activation scales of units 0 .. kDBuf-1 are written before the
      // epilogue's first unit; later ones before it frees the D buffer.
      bool ok3 = prev < 0 ? (it > 0 || mbar_try_wait(kSfInit, 0))
                          : mbar_try_wait(kEfree + 8 * (prev % kRing), (prev / kRing) & 1);
      if (!__all_sync(0xFFFFFFFFu, ok && ok2 && ok3)) {  // slow path, taken by the whole warp
        ok = mbar_wait_bounded(kAfull + 8 * r, (it / kRing) & 1, kSiteGemvFull);
        ok = ok && mbar_wait_bounded(kXfull + 8 * x, (it / AS) & 1, kSiteGemvFull);
        if (prev >= 0) ok = ok && mbar_wait_bounded(kEfree + 8 * (prev % kRing), (prev / kRing) & 1, kSiteGemvEmpty);
        else if (it == 0) ok = ok && mbar_wait_bounded(kSfInit, 0, kSiteGemvFull);
        if (!__all_sync(0xFFFFFFFFu, ok)) break;
      }
      tc::fence_after_sync();
      const uint64_t db0 = tc::smem_desc(smem_u32(x0 + (size_t)x * L.xslot + L.b), kLbo, kSbo);
      const uint32_t dcol = tmem + kTmemD + (uint32_t)(db * 8 * NM), acol = tmem + (uint32_t)(r * 64);
      // Written by the epilogue (activation tiles by TMA) or copied below (fused quantization).
      const uint32_t sfb = tmem + tm_sfb_col(NT) + 8u * r;
      if (tm::elect_one()) {
        if (kGroup || p.x_bf16) {  // fused quantization: this unit's activation scales from shared memory
          const uint32_t sfs = smem_u32(x0 + (size_t)x * L.xslot + L.xs);
          tc::cp_32x128b_warpx4(sfb, tc::smem_desc(sfs, 128u, 128u));
          tc::cp_32x128b_warpx4(sfb + 4u, tc::smem_desc(sfs + 512u, 128u, 128u));
        }
#pragma unroll
        for (int g = 0; g < 8; ++g)
          tc::mma_mx_e4m3_ts(dcol + (uint32_t)(g * NM), acol + (uint32_t)(g * 8), db0 + (uint64_t)((2u * kLbo * g) >> 4),
                             kIdesc | ((uint32_t)(g & 3) << 4), tmem + tm_sfa_col(NT), sfb + 4u * (uint32_t)(g >> 2), 0);
        tc::commit(kXempty + 8 * x);
        tc::commit(kMdone + 8 * db);
      }
      __syncwarp();
    }
    // Free the TMEM once every epilogue warp has read its last partials.
    mbar_wait_bounded(kEdone, 0, kSiteGemvFull);
    __syncwarp();
    tc::fence_after_sync();
    tc::dealloc(tmem, kCols);
    return;
  }

  // ------------------------------------------------------------------ decoders
  if (warp < kEpiWarp0) {
    const int dw = warp - 2;
    const int q = warp & 3;        // TMEM lane quadrant this warp may access
    const int part = dw >> 2;      // which 1/kParts of the K block
    const int rl = 32 * q + lane;  // weight row within the tile = TMEM lane
    const int nthreads = kDecWarps * 32;
    const int tid = threadIdx.x - 64;
    if constexpr (kQ4K) {
      // Q4_K: this thread's half of the block is code bytes 64*part .. 64*part+63
      // (chunks 4*part .. 4*part+3): byte groups 2*part and 2*part+1, each holding
      // two 32-value groups (low and high nibbles) = local groups 0..3.
      static_assert(kParts == 2, "Q4_K decodes with 8 decoder warps");
      (void)tw;
      const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(part * 32);
      if (part == 0)
        tc::st_x4(tmem + ((uint32_t)(32 * q) << 16) + tm_sfa_col(NT), 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu,
                  0x7F7F7F7Fu);
      int s = 0, r = 0;
      uint32_t sph = 0, rph = 0;
      for (int it = 0; it < n_units; ++it) {
        const bool ok1 = mbar_try_wait(kWfull + 8 * s, sph);
        const bool ok2 = it < kRing || mbar_try_wait(kEfree + 8 * r, rph ^ 1);
        if (!__all_sync(0xFFFFFFFFu, ok1 && ok2)) {
          bool ok = mbar_wait_bounded(kWfull + 8 * s, sph, kSiteGemvFull);
          if (it >= kRing) ok = ok && mbar_wait_bounded(kEfree + 8 * r, rph ^ 1, kSiteGemvEmpty);
          if (!__all_sync(0xFFFFFFFFu, ok)) return;
        }
        const uint8_t* st = st0 + (size_t)s * L.stage;
        uint4 ch[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) ch[i] = *reinterpret_cast<const uint4*>(st + (4 * part + i) * 2048 + rl * 16);
        if (part == 0) {
          // The row's d, dmin and 12 scale bytes for the epilogue.
          const uint8_t* sc = st + kQ4kRecSc + rl * 12;
          reinterpret_cast<uint4*>(aux0 + (size_t)r * L.aux + L.w)[rl] =
              make_uint4(*reinterpret_cast<const uint32_t*>(st + kQ4kRecDm + rl * 4),
                         *reinterpret_cast<const uint32_t*>(sc), *reinterpret_cast<const uint32_t*>(sc + 4),
                         *reinterpret_cast<const uint32_t*>(sc + 8));
        }
        uint32_t v[32];  // local group g: columns 8g..8g+7, weights 4c..4c+3 in column c
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int g = 2 * (i >> 1), h = i & 1;  // byte group i/2: groups g (low) and g+1 (high)
          const uint32_t w4[4] = {ch[i].x, ch[i].y, ch[i].z, ch[i].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) q4k_e4m3(w4[k], v[g * 8 + 4 * h + k], v[(g + 1) * 8 + 4 * h + k]);
        }
        tc::st_cols<32>(tq + (uint32_t)(r * 64), v);
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(kAfull + 8 * r);
          mbar_arrive(kEmpty + 8 * s);
        }
        __syncwarp();
        if (++s == S) {
          s = 0;
          sph ^= 1;
        }
        if (++r == kRing) {
          r = 0;
          rph ^= 1;
        }
      }
      return;
    } else {
    // Codebook: stage the 2 KB read at kernel entry, then expand to the
    // lane-private copy, four lanes' copies (16 contiguous bytes) per store.
    tm::build_table(table, tstage, tw, tid, nthreads);

    const uint32_t l4 = (uint32_t)(lane << 2) * 0x01010101u;
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(part * kGroups * 8);
    // The weights' MMA scale factors are all 2^0 (UE8M0 127); the first afull
    // arrival orders these stores before the first MMA.
    if (part == 0) tc::st_x4(tmem + ((uint32_t)(32 * q) << 16) + tm_sfa_col(NT), 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
    // Offsets of this thread's raw bytes in a stage. Packed records are
    // chunk-major ([16-byte chunk][row][16 bytes] for qs and signs, [4-byte
    // column][row][4 bytes] for qh), so the 8 rows of a load phase read
    // consecutive bytes; bulk-copied SoA fields land row-major.
    const bool cm = kGroup || p.packed != nullptr;
    uint32_t off_q0, off_q1, off_sg, off_qh;
    if constexpr (kParts == 2) {
      off_q0 = L.qs + (cm ? (2 * part) * 2048 + rl * 16 : rl * 64 + 32 * part);
      off_q1 = off_q0 + (cm ? 2048 : 16);
      off_sg = L.signs + (cm ? part * 2048 + rl * 16 : rl * 32 + 16 * part);
      off_qh = L.qh + (cm ? part * 512 + rl * 4 : rl * 8 + 4 * part);
    } else {
      off_q0 = L.qs + (cm ? part * 2048 + rl * 16 : rl * 64 + 16 * part);
      off_q1 = off_q0;
      off_sg = L.signs + (cm ? (part >> 1) * 2048 + rl * 16 + (part & 1) * 8 : rl * 32 + 8 * part);
      // Packed records: the whole 4-group qh word (its bits are permuted per group pair).
      off_qh = L.qh + (cm ? (part >> 1) * 512 + rl * 4 : rl * 8 + 2 * part);
    }
    // First group of this thread within its packed qh word (the word's shift base).
    const uint32_t gl0 = kParts == 4 ? 2u * (uint32_t)(part & 1) : 0u;
    int s = 0, r = 0;
    uint32_t sph = 0, rph = 0;  // phases of stage s and ring slot r
    for (int it = 0; it < n_units; ++it) {
      // A ring slot r is free once the epilogue is done with unit it - kRing.
      const bool ok1 = mbar_try_wait(kWfull + 8 * s, sph);
      const bool ok2 = it < kRing || mbar_try_wait(kEfree + 8 * r, rph ^ 1);
      if (!__all_sync(0xFFFFFFFFu, ok1 && ok2)) {  // slow path, taken by the whole warp
        bool ok = mbar_wait_bounded(kWfull + 8 * s, sph, kSiteGemvFull);
        if (it >= kRing) ok = ok && mbar_wait_bounded(kEfree + 8 * r, rph ^ 1, kSiteGemvEmpty);
        if (!__all_sync(0xFFFFFFFFu, ok)) return;
      }
      const uint8_t* st = st0 + (size_t)s * L.stage;
      uint32_t qw[2 * kGroups], sw[kGroups], hw;
      if constexpr (kParts == 2) {
        const uint4 a = *reinterpret_cast<const uint4*>(st + off_q0);
        const uint4 c = *reinterpret_cast<const uint4*>(st + off_q1);
        const uint4 g = *reinterpret_cast<const uint4*>(st + off_sg);
        qw[0] = a.x; qw[1] = a.y; qw[2] = a.z; qw[3] = a.w;
        qw[4] = c.x; qw[5] = c.y; qw[6] = c.z; qw[7] = c.w;
        sw[0] = g.x; sw[1] = g.y; sw[2] = g.z; sw[3] = g.w;
        hw = *reinterpret_cast<const uint32_t*>(st + off_qh);
      } else {
        const uint4 a = *reinterpret_cast<const uint4*>(st + off_q0);
        const uint2 g = *reinterpret_cast<const uint2*>(st + off_sg);
        qw[0] = a.x; qw[1] = a.y; qw[2] = a.z; qw[3] = a.w;
        sw[0] = g.x; sw[1] = g.y;
        hw = cm ? *reinterpret_cast<const uint32_t*>(st + off_qh) : *reinterpret_cast<const uint16_t*>(st + off_qh);
      }
      if (part == 0) {
        // The row's d and scale nibbles for the epilogue (it forms d * (1 + 2*nibble)).
        reinterpret_cast<uint2*>(aux0 + (size_t)r * L.aux + L.w)[rl] =
            make_uint2(*reinterpret_cast<const uint16_t*>(st + L.d + rl * 2),
                       *reinterpret_cast<const uint32_t*>(st + L.scales + rl * 4));
      }
      // All groups first, then one store: the codebook loads of every group can be in flight together.
      uint32_t v[kGroups * 8];
      if (cm) {
#pragma unroll
        for (int g = 0; g < kGroups; ++g)
          tm::decode_group_packed(table, qw[2 * g], qw[2 * g + 1], hw, 2u * (gl0 + (uint32_t)g), sw[g], l4, v + 8 * g);
      } else {
#pragma unroll
        for (int g = 0; g < kGroups; ++g)
          tm::decode_group(table, qw[2 * g], qw[2 * g + 1], (hw >> (8 * g)) & 0xFFu, sw[g], l4, v + 8 * g);
      }
      tc::st_cols<kGroups * 8>(tq + (uint32_t)(r * 64), v);
      tc::wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(kAfull + 8 * r);
        mbar_arrive(kEmpty + 8 * s);
      }
      __syncwarp();  // reconverge before the next waits
      if (++s == S) {
        s = 0;
        sph ^= 1;
      }
      if (++r == kRing) {
        r = 0;
        rph ^= 1;
      }
    }
    return;
    }  // the IQ3_S decoders
  }

  // ------------------------------------------------------------------ epilogue
  {
    const int q = warp & 3;        // TMEM lane quadrant of this warp
    const int rl = 32 * q + lane;  // local weight row = TMEM lane
    const uint32_t tq0 = tmem + ((uint32_t)(32 * q) << 16) + kTmemD;
    float acc[TOK];
#pragma unroll
    for (int t = 0; t < TOK; ++t) acc[t] = 0.f;
    pdl_wait();  // the workspace and output may still be in use by the previous kernel
    pdl_launch_dependents();
    uint32_t ar_epoch = 0;  // this launch's exchange epoch (the previous launch has completed)
    if constexpr (kAR) ar_epoch = *reinterpret_cast<volatile const uint32_t*>(grp.base[grp.rank] + grp.ctl_offset);
    // Unit j's activation scales (UE8M0, one per token and 32-wide group) go
    // to TMEM scale-factor slot j % kRing of this warp's quadrant, token t in
    // lane t: groups 0-3 in bytes 0-3 of column +0, groups 4-7 in column +4
    // (the MMA's scale addresses must be 4-column aligned). Lanes past the
    // activation tile's rows read other bytes of shared memory; their columns
    // of D are never read.
    const uint32_t tsf = tmem + ((uint32_t)(32 * q) << 16) + tm_sfb_col(NT);
    // kbj: the K block of unit j (for the half of the scale row it uses).
    auto write_sf = [&](int j, int kbj) -> bool {
      if (kGroup || p.x_bf16) return true;  // the MMA warp copies them (fused quantization)
      const int xj = j % AS;
      bool ok = mbar_try_wait(kXfull + 8 * xj, (j / AS) & 1);
      if (!__all_sync(0xFFFFFFFFu, ok)) {
        ok = mbar_wait_bounded(kXfull + 8 * xj, (j / AS) & 1, kSiteGemvFull);
        if (!__all_sync(0xFFFFFFFFu, ok)) return false;
      }
      const uint2 v = *reinterpret_cast<const uint2*>(x0 + (size_t)xj * L.xslot + L.xs + lane * 16 +
                                                      (kbj & 1) * 8);
      const uint32_t vv[8] = {v.x, v.x, v.x, v.x, v.y, v.y, v.y, v.y};
      tc::st_x8(tsf + 8u * (uint32_t)(j % kRing), vv);
      return true;
    };
    // K block of unit `it` and of unit it + kDBuf, advanced incrementally.
    const int kb_first = u0 % p.n_blocks;
    auto kb_step = [&](int kb) { return kb + 1 == p.n_blocks ? 0 : kb + 1; };
    int kb_ahead = kb_first;
    bool sf_ok = true;
    for (int j = 0; j < kDBuf && j < n_units; ++j, kb_ahead = kb_step(kb_ahead)) sf_ok = sf_ok && write_sf(j, kb_ahead);
    tc::wait_st();
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(kSfInit);
    __syncwarp();
    // The linear of unit `it`: its output, K blocks, first unit and first row
    // tile in the launch's numbering, row tiles (a grouped launch moves to the
    // next item when they are done; a single linear has one).
    OutView ov{p.out, p.ldo, p.out_bf16, p.n_rows, p.m};
    QuantView qv{};
    if constexpr (kQ) qv = QuantView{p.q_out, p.ldq, p.s_out, p.lds};
    int cur_nb = p.n_blocks, cur_unit0 = 0, cur_tile0 = 0, cur_tiles = 0, item = 0;
    auto load_item = [&](int l) {
      if constexpr (kGroup) {
        const GemvItem& gi = grp.items[l];
        ov = OutView{gi.out, gi.ldo, gi.out_bf16, gi.n_rows, gi.m};
        if constexpr (kQ) qv = QuantView{gi.q_out, gi.ldq, gi.s_out, gi.lds};
        cur_nb = gi.n_blocks;
        cur_unit0 = gi.unit0;
        cur_tile0 = gi.tile0;
        cur_tiles = (gi.n_rows + kRows - 1) / kRows;
      }
    };
    if constexpr (kGroup) {
      item = group_item(grp, u0, 0);
      load_item(item);
    }
    // Row tile (in the launch's numbering) holding unit u.
    auto tile_of = [&](int u) -> int {
      if constexpr (kGroup) {
        const int l = group_item(grp, u, 0);
        return grp.items[l].tile0 + (u - grp.items[l].unit0) / grp.items[l].n_blocks;
      } else {
        return u / p.n_blocks;
      }
    };
    const int first_tile = tile_of(u0);
    int seg_begin = u0;
    // K block and row tile (within its linear) of unit `it`.
    int kb_next = (u0 - cur_unit0) % cur_nb, rt_next = (u0 - cur_unit0) / cur_nb;
    // Q4_K: the activations' group sums of a unit, spread over the warp (lane
    // l holds kSF of them: token l / (8 / kSF), groups (l % (8 / kSF)) * kSF
    // on) and read with shuffles. The next unit's are loaded while this one
    // is processed, so their latency stays off the epilogue's path.
    constexpr int kSF = TOK / 4, kSLanes = 8 / kSF;
    float sum_cur[kSF], sum_next[kSF];
    auto load_sums = [&](int kb, float (&dst)[kSF]) {
      if constexpr (kQ4K) {
        const int t = lane / kSLanes;
        if (t < p.m) {
          const float* src = p.xsum + (size_t)t * p.ldsum + (size_t)kb * 8 + (lane % kSLanes) * kSF;
          if constexpr (kSF == 2) {
            const float2 v = __ldg(reinterpret_cast<const float2*>(src));
            dst[0] = v.x;
            dst[1] = v.y;
          } else {
#pragma unroll
            for (int j = 0; j < kSF; j += 4) {
              const float4 v = __ldg(reinterpret_cast<const float4*>(src + j));
              dst[j] = v.x;
              dst[j + 1] = v.y;
              dst[j + 2] = v.z;
              dst[j + 3] = v.w;
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < kSF; ++j) dst[j] = 0.f;
        }
      }
    };
    // Grouped Q4_K launches: the sums of unit uu come from its item (forward cursor).
    int sum_item = 0;
    auto load_sums_of = [&](int uu, int kb_single, float (&dst)[kSF]) {
      if constexpr (kQ4K && kGroup) {
        sum_item = group_item(grp, uu, sum_item);
        const GemvItem& gi = grp.items[sum_item];
        const int kb = (uu - gi.unit0) % gi.n_blocks;
        const int t = lane / kSLanes;
        if (t < gi.m) {
          const float* src = gi.xsum + (size_t)t * gi.ldsum + (size_t)kb * 8 + (lane % kSLanes) * kSF;
#pragma unroll
          for (int j = 0; j < kSF; j += 2) {
            const float2 v = __ldg(reinterpret_cast<const float2*>(src + j));
            dst[j] = v.x;
            dst[j + 1] = v.y;
          }
        } else {
#pragma unroll
          for (int j = 0; j < kSF; ++j) dst[j] = 0.f;
        }
      } else {
        load_sums(kb_single, dst);
      }
    };
    if constexpr (kQ4K) {
      if (u0 < u1) load_sums_of(u0, kb_next, sum_next);
    }
    int r = 0;  // ring slot of unit `it` and its phase
    uint32_t rph = 0;
    auto next_slot = [&]() {
      if (++r == kRing) {
        r = 0;
        rph ^= 1u;
      }
    };
    for (int it = 0, u = u0; sf_ok && u < u1; ++u, ++it, kb_ahead = kb_step(kb_ahead), next_slot()) {
      const int db = kDBuf == 2 ? (it & 1) : 0;
      const uint32_t mpar = kDBuf == 2 ? ((it >> 1) & 1) : (it & 1);
      bool ok = mbar_try_wait(kMdone + 8 * db, mpar);
      bool ok2 = mbar_try_wait(kAfull + 8 * r, rph);
      if (!__all_sync(0xFFFFFFFFu, ok && ok2)) {  // slow path, taken by the whole warp
        ok = mbar_wait_bounded(kMdone + 8 * db, mpar, kSiteGemvFull);
        ok = ok && mbar_wait_bounded(kAfull + 8 * r, rph, kSiteGemvFull);
        if (!__all_sync(0xFFFFFFFFu, ok)) break;
      }
      tc::fence_after_sync();
      const uint32_t tq = tq0 + (uint32_t)(db * 8 * NM);
      const uint8_t* aux = aux0 + (size_t)r * L.aux;
      if constexpr (kQ4K) {
        // Q4_K: out += P_g * d*s_g/2 - (dmin*m_g - 7.5*d*s_g) * (the token's sum of group g's activations),
        // P_g the group's product with the odd integers 2q - 15.
#pragma unroll
        for (int j = 0; j < kSF; ++j) sum_cur[j] = sum_next[j];
        if (u + 1 < u1) load_sums_of(u + 1, kb_step(kb_next), sum_next);
        // This unit's sums into the warp's copy [TOK][8] (lane l holds entries l*kSF..), read back as
        // broadcasts.
        float* scr = reinterpret_cast<float*>(tstage) + (warp - kEpiWarp0) * TOK * 8;
        __syncwarp();  // every lane has read the previous unit's copy
#pragma unroll
        for (int j = 0; j < kSF; j += 2)
          *reinterpret_cast<float2*>(scr + lane * kSF + j) = make_float2(sum_cur[j], sum_cur[j + 1]);
        __syncwarp();
        const float4* scr4 = reinterpret_cast<const float4*>(scr);
        const uint4 a4 = reinterpret_cast<const uint4*>(aux + L.w)[rl];
        const float dv = __half2float(__ushort_as_half((unsigned short)(a4.x & 0xFFFFu)));
        const float dmv = __half2float(__ushort_as_half((unsigned short)(a4.x >> 16)));
        const uint32_t b[3] = {a4.y, a4.z, a4.w};  // the 12 scale bytes
        auto byte = [&](int i) -> uint32_t { return (b[i >> 2] >> (8 * (i & 3))) & 0xFFu; };
        float wg[8], og[8];
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          const uint32_t sg = g < 4 ? byte(g) & 63u : (byte(g + 4) & 15u) | ((byte(g - 4) >> 6) << 4);
          const uint32_t mg = g < 4 ? byte(g + 4) & 63u : (byte(g + 4) >> 4) | ((byte(g) >> 6) << 4);
          // The MMA summed v = 2q - 15: d*s*q - dmin*m = (d*s/2)*v + (7.5*d*s - dmin*m).
          wg[g] = 0.5f * dv * (float)sg;
          og[g] = dmv * (float)mg - 7.5f * dv * (float)sg;
        }
        // One token's group sums from the warp's copy.
        auto sums_of = [&](int t, float (&sv)[8]) {
          const float4 lo = scr4[2 * t], hi = scr4[2 * t + 1];
          sv[0] = lo.x; sv[1] = lo.y; sv[2] = lo.z; sv[3] = lo.w;
          sv[4] = hi.x; sv[5] = hi.y; sv[6] = hi.z; sv[7] = hi.w;
        };
#pragma unroll
        for (int t0 = 0; t0 < TOK; t0 += 8) {
          if (t0 >= ov.m) break;  // warp-uniform
          uint32_t off[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) off[j] = (uint32_t)(j * NM + t0);
          float c[8][8];
          tc::ld_x8_multi<8>(tq, off, c);
          if (t0 + 8 <= ov.m) {
            // Eight tokens: two token pairs' sums at a time, the scale and the constant term in separate
            // paired accumulators (independent FMA chains).
#pragma unroll
            for (int t = 0; t < 8; t += 2) {
              float sa[8], sb[8];
              sums_of(t0 + t, sa);
              sums_of(t0 + t + 1, sb);
              float pa = 0.f, pb = 0.f, qa = 0.f, qb = 0.f;
#pragma unroll
              for (int g = 0; g < 8; ++g) {
                fma2(pa, pb, c[g][t], c[g][t + 1], wg[g], wg[g]);
                fma2(qa, qb, sa[g], sb[g], og[g], og[g]);
              }
              acc[t0 + t] += pa - qa;
              acc[t0 + t + 1] += pb - qb;
            }
          } else {
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              if (t0 + t < ov.m) {  // tokens past M are padding (warp-uniform branch)
                float sv[8];
                sums_of(t0 + t, sv);
                float pa = 0.f, qa = 0.f;
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                  pa = fmaf(c[g][t], wg[g], pa);
                  qa = fmaf(sv[g], og[g], qa);
                }
                acc[t0 + t] += pa - qa;
              }
            }
          }
        }
      } else {
        const uint2 dsc = reinterpret_cast<const uint2*>(aux + L.w)[rl];
        const float dv = __half2float(__ushort_as_half((unsigned short)dsc.x));
        const float dneg = -8388608.0f * dv;
        // 2*nibble+1 of group g is byte g/2 of tb[g&1]; float(2^23 + t)*d - 2^23*d = t*d exactly.
        const uint32_t tb0 = lop3_and_or(dsc.y << 1, 0x1E1E1E1Eu, 0x01010101u);
        const uint32_t tb1 = lop3_and_or(dsc.y >> 3, 0x1E1E1E1Eu, 0x01010101u);
        // Groups per batch of TMEM loads (one wait per batch), within the register budget.
        constexpr int GB = kDecWarps == 8 ? (TOK <= 8 ? 8 : TOK <= 16 ? 4 : 2) : 2;
  #pragma unroll
        for (int t0 = 0; t0 < TOK; t0 += 8) {
  #pragma unroll
          for (int g0 = 0; g0 < 8; g0 += GB) {
            uint32_t off[GB];
  #pragma unroll
            for (int j = 0; j < GB; ++j) off[j] = (uint32_t)((g0 + j) * NM + t0);
            float c[GB][8];
            tc::ld_x8_multi<GB>(tq, off, c);
            if constexpr (kGroup) {
              // Grouped launches (items of 1 to 8 tokens): the group factors first, then one
              // warp-uniform branch per token pair. (Single linears keep the loop below; the
              // same order would cost them 2-3 % in code layout, measured.)
              float wv[GB];
  #pragma unroll
              for (int j = 0; j < GB; ++j) {
                const int g = g0 + j;
                wv[j] = fmaf(__uint_as_float(prmt((g & 1) ? tb1 : tb0, 0x4B000000u, 0x7650u | (uint32_t)(g >> 1))),
                             dv, dneg);
              }
  #pragma unroll
              for (int t = 0; t < 8; t += 2) {
                if (t0 + t < ov.m) {
  #pragma unroll
                  for (int j = 0; j < GB; ++j)
                    fma2(acc[t0 + t], acc[t0 + t + 1], c[j][t], c[j][t + 1], wv[j], wv[j]);
                }
              }
            } else {
  #pragma unroll
              for (int j = 0; j < GB; ++j) {
                const int g = g0 + j;
                const float w = fmaf(__uint_as_float(prmt((g & 1) ? tb1 : tb0, 0x4B000000u, 0x7650u | (uint32_t)(g >> 1))),
                                     dv, dneg);
  #pragma unroll
                for (int t = 0; t < 8; t += 2) {
                  if (t0 + t < ov.m)  // tokens past M are padding (warp-uniform branch)
                    fma2(acc[t0 + t], acc[t0 + t + 1], c[j][t], c[j][t + 1], w, w);
                }
              }
            }
          }
        }
      }
      // The MMAs of unit it + kDBuf wait for this D buffer: their scales first.
      if (it + kDBuf < n_units && !write_sf(it + kDBuf, kb_ahead)) break;
      tc::wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(kEfree + 8 * r);
      __syncwarp();  // reconverge before the next waits

      const int kb = kb_next, rt = rt_next;
      const OutView ou = ov;  // this unit's linear (the cursor may move to the next item below)
      const QuantView qu = qv;
      const int nbu = cur_nb, unit0u = cur_unit0, tile = cur_tile0 + rt;
      if (++kb_next == cur_nb) {
        kb_next = 0;
        ++rt_next;
        if constexpr (kGroup) {
          if (rt_next == cur_tiles && u + 1 < u1) {
            load_item(++item);
            rt_next = 0;
          }
        }
      }
      if (!(kb == nbu - 1 || u == u1 - 1)) continue;
      const bool full_tile = (seg_begin == unit0u + rt * nbu) && (kb == nbu - 1);
      const int row = rt * kRows + rl;
      if (p.kparts > 1) {
        // Cluster K-split: ranks 1.. write their partials into rank 0's shared
        // memory and arrive on its barrier; rank 0 sums in rank order.
        const uint32_t rank = cluster_ctarank();
        if (rank != 0) {
          const uint32_t remote = mapa_shared(smem_u32(cpart) + (((rank - 1) * kRows + rl) * TOK) * 4u, 0);
#pragma unroll
          for (int t = 0; t < TOK; t += 4) st_cluster_v4(remote + 4u * t, acc[t], acc[t + 1], acc[t + 2], acc[t + 3]);
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(kCred, 0));
          __syncwarp();
        } else {
          if (__all_sync(0xFFFFFFFFu, mbar_wait_cluster_bounded(kCred, 0, kSiteGemvFull))) {
            for (int rk = 1; rk < p.kparts; ++rk) {
              const float* src = cpart + ((rk - 1) * kRows + rl) * TOK;
#pragma unroll
              for (int t = 0; t < TOK; ++t) acc[t] += src[t];
            }
            bool keep = true;
            if constexpr (kAR) keep = ar_exchange<TOK>(grp, ar_epoch, row, lane, acc);
            if (keep) {
#pragma unroll
              for (int t = 0; t < TOK; ++t) store_out_tm<kQ>(ou, qu, row, t, acc[t]);
            }
          }
        }
      } else if (full_tile) {
        bool keep = true;
        if constexpr (kAR) keep = ar_exchange<TOK>(grp, ar_epoch, row, lane, acc);
        if (keep) {
#pragma unroll
          for (int t = 0; t < TOK; ++t) store_out_tm<kQ>(ou, qu, row, t, acc[t]);
        }
      } else {
        // Stream-K: a row tile shared with other CTAs. The segment a CTA
        // finishes last is usually the last contribution: if every other
        // contributor has already published, sum at once; otherwise publish,
        // and the last to arrive sums (in CTA order either way).
        const int cta = blockIdx.x;
        const int tile_u0 = unit0u + rt * nbu;  // first unit of the row tile
        const int c_first = cta_of_unit(tile_u0);
        const int c_last = cta_of_unit(tile_u0 + nbu - 1);
        const int slot_id = (tile == first_tile) ? 0 : 1;
        int* counter = p.counters + (size_t)tile * kEpiWarps + q;
        int last = 0;
        if (u == u1 - 1) {
          if (lane == 0) last = ld_acquire_gpu(counter) == c_last - c_first;
          last = __shfl_sync(0xFFFFFFFFu, last, 0);
        }
        if (!last) {
          float* part = p.partials + ((size_t)(cta * 2 + slot_id) * kRows + rl) * TOK;
#pragma unroll
          for (int t = 0; t < TOK; t += 4)
            __stcg(reinterpret_cast<float4*>(part + t), make_float4(acc[t], acc[t + 1], acc[t + 2], acc[t + 3]));
          __syncwarp();
          if (lane == 0) last = atomic_add_acq_rel_gpu(counter, 1) == c_last - c_first;
          last = __shfl_sync(0xFFFFFFFFu, last, 0);
        }
        if (last) {
          if (lane == 0) *counter = 0;  // every contributor has arrived: leave it zeroed for the next launch
          sum_partials<TOK, kQ>(p.partials, unit_begin, ou, qu, tile, rl, row, cta, c_first, c_last, tile_of, acc);
        }
      }
#pragma unroll
      for (int t = 0; t < TOK; ++t) acc[t] = 0.f;
      seg_begin = u + 1;
    }
    if constexpr (kAR) {
      // The last CTA to finish advances the epoch for the next launch (which
      // reads it only after this grid has completed).
      if (warp == kEpiWarp0 && lane == 0) {
        uint32_t* ctl = reinterpret_cast<uint32_t*>(grp.base[grp.rank] + grp.ctl_offset);
        __threadfence();
        if (atomicAdd(ctl + 1, 1u) == gridDim.x - 1) {
          ctl[1] = 0;
          ctl[0] = ar_epoch + 1u;
          __threadfence();
        }
      }
    }
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(kEdone);
  }
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------
uint32_t gemv_tm_smem_bytes(int nt, int stages, int kparts, bool fused, bool q4k) {
  return tm_smem_bytes(nt, stages, kparts, fused, q4k);
}
int gemv_tm_max_stages() { return kMaxStagesTm; }

template <int NT, int kDecWarps, bool kQ = false, bool kQ4K = false>
static const void* tm_kernel() {
  return (const void*)iq3s_gemv_tm_kernel<NT, kDecWarps, GemvNoGroup, kQ, kQ4K>;
}
template <int NT, int kDecWarps, bool kQ = false>
static const void* tm_kernel_group() {
  return (const void*)iq3s_gemv_tm_kernel<NT, kDecWarps, GemvGroup, kQ>;
}
template <int NT, bool kQ = false, bool kQ4K = false>
static const void* tm_kernel_group_pre() {
  return (const void*)iq3s_gemv_tm_kernel<NT, 8, GemvGroupPre, kQ, kQ4K>;
}

static int query_max_clusters(int nt, int dec_warps, int stages, int kparts, bool q4k);

static const void* tm_kernel_for(int nt, int dec_warps, bool q4k = false) {
  if (q4k) return nt == 1 ? tm_kernel<1, 8, false, true>() : nt == 2 ? tm_kernel<2, 8, false, true>()
                                                                    : tm_kernel<4, 8, false, true>();
  if (dec_warps == 16) return nt == 1 ? tm_kernel<1, 16>() : nt == 2 ? tm_kernel<2, 16>() : tm_kernel<4, 16>();
  return nt == 1 ? tm_kernel<1, 8>() : nt == 2 ? tm_kernel<2, 8>() : tm_kernel<4, 8>();
}

int gemv_tm_max_clusters(int nt, int dec_warps, int stages, int kparts, bool q4k) {
  // Cached per (device, configuration): the query runs once.
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, bool>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const auto key = std::make_tuple(dev, nt, dec_warps, stages, kparts, q4k);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const int n = query_max_clusters(nt, dec_warps, stages, kparts, q4k);
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = n;
  return n;
}

static int query_max_clusters(int nt, int dec_warps, int stages, int kparts, bool q4k) {
  const void* kern = tm_kernel_for(nt, dec_warps, q4k);
  const uint32_t smem = tm_smem_bytes(nt, stages, kparts, false, q4k);
  if (ensure_smem_attribute(kern, smem) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kparts * 16);
  cfg.blockDim = dim3(tm_threads(dec_warps));
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)kparts;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

template <int NT, int kDecWarps>
static cudaError_t launch_gemv_tm_t(const GemvTmParams& p, const GemvTmMaps& maps, int grid, cudaStream_t stream,
                                    bool q4k = false) {
  const uint32_t smem = tm_smem_bytes(NT, p.stages, p.kparts, p.x_bf16 != nullptr, q4k);
  const void* kern = q4k ? tm_kernel<NT, 8, false, true>()
                     : p.q_out != nullptr ? tm_kernel<NT, kDecWarps, true>() : tm_kernel<NT, kDecWarps, false>();
  cudaError_t e = ensure_smem_attribute(kern, smem);
  if (e != cudaSuccess) return e;
  const GemvNoGroup none{0};
  return launch_pdl_cluster(kern, dim3(grid), dim3(tm_threads(kDecWarps)), smem, stream, p.kparts > 1 ? p.kparts : 1,
                            p, maps, none);
}

// Grouped launches use 8 decoder warps and stream-K.
template <int NT>
static cudaError_t launch_gemv_tm_group_t(const GemvTmParams& p, const GemvGroup& g, int grid, cudaStream_t stream) {
  const uint32_t smem = tm_smem_bytes(NT, p.stages, 0, true);
  bool quant = false;  // some item also writes its output's MXFP8 quantization
  for (int i = 0; i < g.count; ++i) quant = quant || g.items[i].q_out != nullptr;
  const void* kern = quant ? tm_kernel_group<NT, 8, true>() : tm_kernel_group<NT, 8, false>();
  cudaError_t e = ensure_smem_attribute(kern, smem);
  if (e != cudaSuccess) return e;
  GemvTmMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  return launch_pdl_cluster(kern, dim3(grid), dim3(tm_threads(8)), smem, stream, 1, p, maps, g);
}

template <int NT>
static cudaError_t launch_gemv_tm_group_pre_t(const GemvTmParams& p, const GemvGroupPre& g, int grid,
                                              cudaStream_t stream, bool q4k) {
  const uint32_t smem = tm_smem_bytes(NT, p.stages, 0, true, q4k);
  bool quant = false;  // some item also writes its output's MXFP8 quantization
  for (int i = 0; i < g.count; ++i) quant = quant || g.items[i].q_out != nullptr;
  if (q4k && quant) return cudaErrorInvalidValue;
  const void* kern = q4k ? tm_kernel_group_pre<NT, false, true>()
                         : quant ? tm_kernel_group_pre<NT, true>() : tm_kernel_group_pre<NT, false>();
  cudaError_t e = ensure_smem_attribute(kern, smem);
  if (e != cudaSuccess) return e;
  GemvTmMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  return launch_pdl_cluster(kern, dim3(grid), dim3(tm_threads(8)), smem, stream, 1, p, maps, g);
}

cudaError_t launch_gemv_tm_group_pre(const GemvTmParams& p, const GemvGroupPre& g, int nt, int grid,
                                     cudaStream_t stream, bool q4k) {
  if (p.kparts != 0) return cudaErrorInvalidValue;
  switch (nt) {
    case 1: return launch_gemv_tm_group_pre_t<1>(p, g, grid, stream, q4k);
    case 2: return launch_gemv_tm_group_pre_t<2>(p, g, grid, stream, q4k);
    default: return launch_gemv_tm_group_pre_t<4>(p, g, grid, stream, q4k);
  }
}

cudaError_t launch_gemv_tm_group(const GemvTmParams& p, const GemvGroup& g, int nt, int dec_warps, int grid,
                                 cudaStream_t stream) {
  if (dec_warps != 8 || p.kparts != 0) return cudaErrorInvalidValue;
  switch (nt) {
    case 1: return launch_gemv_tm_group_t<1>(p, g, grid, stream);
    case 2: return launch_gemv_tm_group_t<2>(p, g, grid, stream);
    default: return launch_gemv_tm_group_t<4>(p, g, grid, stream);
  }
}

template <int NT>
static cudaError_t launch_gemv_tm_n(const GemvTmParams& p, int dec_warps, const GemvTmMaps& maps, int grid,
                                    cudaStream_t stream, bool q4k) {
  if (q4k) return launch_gemv_tm_t<NT, 8>(p, maps, grid, stream, true);
  if (dec_warps == 16) return launch_gemv_tm_t<NT, 16>(p, maps, grid, stream);
  return launch_gemv_tm_t<NT, 8>(p, maps, grid, stream);
}

cudaError_t launch_gemv_tm(const GemvTmParams& p, int nt, int dec_warps, const GemvTmMaps& maps, int grid,
                           cudaStream_t stream, bool q4k) {
  if (q4k && (dec_warps != 8 || p.x_bf16 != nullptr || p.q_out != nullptr || !p.packed || !p.xsum))
    return cudaErrorInvalidValue;
  switch (nt) {
    case 1: return launch_gemv_tm_n<1>(p, dec_warps, maps, grid, stream, q4k);
    case 2: return launch_gemv_tm_n<2>(p, dec_warps, maps, grid, stream, q4k);
    default: return launch_gemv_tm_n<4>(p, dec_warps, maps, grid, stream, q4k);
  }
}

uint32_t q4k_gemv_smem_bytes(int nt, int stages, int kparts) { return tm_smem_bytes(nt, stages, kparts, false, true); }

// Row-split linear with its all-reduce fused: 8 decoder warps, bf16 rows
// quantized in the kernel, whole row tiles or cluster K splits (kparts >= 1:
// every row's final sum is formed in one CTA, where the exchange runs).
template <int NT>
static cudaError_t launch_gemv_tm_ar_t(const GemvTmParams& p, const GemvAr& ar, const GemvTmMaps& maps, int grid,
                                       cudaStream_t stream) {
  const uint32_t smem = tm_smem_bytes(NT, p.stages, p.kparts, true);
  const void* kern = (const void*)iq3s_gemv_tm_kernel<NT, 8, GemvAr, false>;
  cudaError_t e = ensure_smem_attribute(kern, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl_cluster(kern, dim3(grid), dim3(tm_threads(8)), smem, stream, p.kparts > 1 ? p.kparts : 1, p,
                            maps, ar);
}

cudaError_t launch_gemv_tm_ar(const GemvTmParams& p, const GemvAr& ar, int nt, const GemvTmMaps& maps, int grid,
                              cudaStream_t stream) {
  if (p.kparts < 1 || p.x_bf16 == nullptr || p.q_out != nullptr || ar.world < 1 || ar.world > kGemvArMaxRanks)
    return cudaErrorInvalidValue;
  switch (nt) {
    case 1: return launch_gemv_tm_ar_t<1>(p, ar, maps, grid, stream);
    case 2: return launch_gemv_tm_ar_t<2>(p, ar, maps, grid, stream);
    default: return launch_gemv_tm_ar_t<4>(p, ar, maps, grid, stream);
  }
}

}  // namespace mambo
