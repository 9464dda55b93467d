// IQ3_S x MXFP8 GEMM for prefill-sized M with FP16 tensor-core operands, one
// accumulator per 256-wide K block.
//
// The per-32-weight-group scale d * (1 + 2*nibble) is not a power of two, so
// the reference's large-M kernel (src/python/mambo/kernels/iq3_s_fp8.py:262-275)
// forms one FP8 product per group and rescales it in FP32; on a tensor core
// that turns every 32-deep MMA into a round trip through the CUDA cores. Here
// the group factor moves into the weight operand instead, exactly:
//   A = sign * grid * (1 + 2*nibble)   (|A| <= 15 * 31 = 465: 9 significant
//                                       bits, exact in FP16)
//   B = E4M3(x) * 2^(e(x, g) - e_max(token))   (FP16, exact while the group's
//                                       exponent is within 12 of the token's
//                                       largest; below that, FP16 rounding of
//                                       parts 2^12 smaller than the row's
//                                       largest group)
// so one FP32 accumulator covers a whole K block: out += D * d per block, and
// out *= 2^e_max(token) at the end (exact powers of two).
//
// Tiles: 128 weight rows x 128 tokens, persistent CTAs as in the FP8 GEMM.
// Roles: weight producer (bulk copies of tile-major records), activation
// producer (3-D TMA of 128 x 128 FP16 half-blocks), 8 decoder warps (codebook
// gather -> E4M3 -> FP16 x (1+2*nibble) -> tcgen05.st, A ring of 2 blocks =
// 256 TMEM columns), MMA warp (16 x kind::f16 M=128 N=128 K=16 per block into
// one of two D buffers), 8 epilogue warps (two per TMEM lane quadrant).
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "kernels.cuh"
#include "tcgen05.cuh"
#include "iq3s_tm.cuh"
#include "mxfp8.cuh"

namespace mambo {

namespace {

constexpr int kRowsH = 128, kTokH = 128;
constexpr int kDecWarpsH = 8, kEpiWarpsH = 8;
constexpr int kARingH = 2;   // decoded A blocks in TMEM (128 columns each)
constexpr int kDRingH = 2;   // D buffers (128 columns each)
// FP16 activation half-blocks (the CTA's tokens x 128 K) in flight: 3 of 32 KB
// for a single CTA (128 tokens), 6 of 16 KB for a CTA of a pair (64 tokens).
constexpr int kXStagesMaxH = 6;
constexpr int kMaxWStagesH = 6;
constexpr uint32_t kXRingBytesH = 3u * kTokH * 128u * 2u;  // 96 KB either way
__host__ __device__ constexpr int x_stages_h(bool pair) { return pair ? 6 : 3; }
__host__ __device__ constexpr uint32_t x_half_bytes_h(bool pair) { return (pair ? 64u : 128u) * 256u; }
// Rows' d of a block, in a ring of 4 with its own barriers (dfull, count 4:
// the part-0 decoder warps). The decoders write slot it % 4 after the MMAs of
// block it - 2 completed, which waited for the epilogue to release block
// it - 4's D buffer: the epilogue has read that slot, and the decoders are
// never 4 blocks ahead of it, so the barrier phases cannot alias.
constexpr int kAuxRingH = 4;
constexpr uint32_t kAuxH = kRowsH * 4;
constexpr uint32_t kBarBytesH = 512;
constexpr uint32_t kTmA = 0, kTmD = 128u * kARingH;
constexpr uint32_t kTmColsH = 512;
static_assert(kTmD + kDRingH * (uint32_t)kTokH <= kTmColsH, "TMEM plan exceeds 512 columns");
constexpr int kThreadsH = (3 + kDecWarpsH + kEpiWarpsH) * 32;
static_assert(2 * (kMaxWStagesH + kXStagesMaxH + kARingH + kDRingH) + 1 + kAuxRingH + 2 + 1 <= (int)(kBarBytesH / 8),
              "barrier area");
constexpr int kEpiWarp0H = 2 + kDecWarpsH, kXWarpH = kEpiWarp0H + kEpiWarpsH;

__host__ __device__ constexpr uint32_t align_up_h(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// With out_stage: a 32 KB bf16 tile (128 tokens x 128 rows) for the TMA store, after the barriers.
constexpr uint32_t kOutStageBytesH = kTokH * kRowsH * 2u;
__host__ __device__ inline uint32_t gemm_f16_smem(int wstages, bool out_stage = false) {
  return tm::kTableBytes + 1024 + align_up_h((uint32_t)wstages * tm::kRecordBytes, 1024) + kXRingBytesH +
         kAuxRingH * kAuxH + tm::kTableStageBytes + kBarBytesH + (out_stage ? 128u + kOutStageBytesH : 0u);
}

// Two E4M3 values (bytes 0 and 1 of each half of v) -> two FP16 pairs.
__device__ __forceinline__ void e4m3x4_to_f16x4(uint32_t v, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(v));
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ void store_out_h(const GemmF16Params& p, int row, int tok, float v) {
  if (row < p.n_rows && tok < p.m) {
    if (p.out_bf16) {
      reinterpret_cast<__nv_bfloat16*>(p.out)[(int64_t)tok * p.ldo + row] = __float2bfloat16_rn(v);
    } else {
      reinterpret_cast<float*>(p.out)[(int64_t)tok * p.ldo + row] = v;
    }
  }
}

}  // namespace

// kPair: tiles of 256 weight rows x 128 tokens on a cluster of two CTAs. Each
// CTA decodes its 128 rows into its own TMEM and loads its 64 tokens of every
// activation half-block; rank 0 issues M=256 MMAs over both (one activation
// tile serves 256 weight rows: half the L2 traffic per FLOP) and its commits
// arrive in both CTAs; rank 1's decoders and epilogue arrive on rank 0's
// barriers. Otherwise 128 x 128 tiles on single CTAs.
// kFold: the block scale d folded, rounded, into the FP16 weight operand with
// each row's exponent taken out (GemmF16Params::row_exp), so one accumulator
// covers the tile's whole K range: the epilogue runs once per tile instead of
// once per K block, and the MMAs never wait for it inside a tile. Each weight
// carries one FP16 rounding (about 2^-12 relative).
// kPair and kFold together (the wide GEMM): tiles of 256 weight rows x 256
// tokens on a CTA pair, each CTA loading 128 tokens of every activation
// half-block and holding its rows' 128 x 256 accumulator (all of TMEM beside
// the A ring, so one accumulator per tile). Each decoded weight block feeds
// twice the tensor work of a 128-token tile, and each activation tile serves
// 256 weight rows.
template <bool kPair, bool kFold = false>
__global__ void __launch_bounds__(kThreadsH, 1)
    iq3s_gemm_f16_kernel(const __grid_constant__ GemmF16Params p, const __grid_constant__ GemmF16Maps maps) {
  constexpr bool kWide = kPair && kFold;
  constexpr int kTokT = kWide ? 2 * kTokH : kTokH;  // tokens of a tile
  constexpr int kPasses = kWide ? 2 : 1;            // epilogue passes of 128 tokens per tile
  // B half-block (the CTA's tokens x 128 K): two [tokens][128 bytes] boxes in
  // the 128-byte-swizzled K-major layout (8-row atoms 1024 bytes apart); an
  // MMA's 16 K (32 bytes) start 32 bytes further into the row.
  constexpr int kTokLoad = kPair && !kWide ? 64 : kTokH;
  constexpr int kXS = x_stages_h(kPair && !kWide);
  constexpr uint32_t kXHalf = x_half_bytes_h(kPair && !kWide);
  constexpr uint32_t kBoxBytes = kTokLoad * 128u;
  constexpr uint32_t kIdesc = tc::idesc_f16_f32(kPair ? 2 * kRowsH : kRowsH, kTokT);
  static_assert(!kWide || kTmD + (uint32_t)kTokT <= kTmColsH, "wide GEMM: one 256-column accumulator beside the A ring");
  constexpr uint16_t kBoth = 0x3;  // CTA mask of a pair

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* table = smem_raw;
  uint8_t* st0 = smem_raw + tm::kTableBytes + ((1024u - ((smem_u32(smem_raw) + tm::kTableBytes) & 1023u)) & 1023u);
  const int SW = p.wstages;
  uint8_t* x0 = st0 + align_up_h((uint32_t)SW * tm::kRecordBytes, 1024);
  uint8_t* aux0 = x0 + (size_t)kXRingBytesH;
  uint32_t* tstage = reinterpret_cast<uint32_t*>(aux0 + kAuxRingH * kAuxH);
  uint64_t* bars = reinterpret_cast<uint64_t*>(aux0 + kAuxRingH * kAuxH + tm::kTableStageBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxWStagesH + 2 * kXStagesMaxH + 2 * kARingH +
                                                    2 * kDRingH + 1 + kAuxRingH + 2);
  uint8_t* ostage = reinterpret_cast<uint8_t*>(bars) + kBarBytesH;  // bf16 output tile (out_tma)
  ostage += (128u - (smem_u32(ostage) & 127u)) & 127u;
  const uint32_t bar0 = smem_u32(bars);
  // Barriers as in the FP8 GEMM, with activation slots per half block.
  const uint32_t kWfull = bar0, kWempty = bar0 + 8 * kMaxWStagesH;
  const uint32_t kXfull = bar0 + 16 * kMaxWStagesH, kXempty = kXfull + 8 * kXStagesMaxH;
  const uint32_t kAfull = kXempty + 8 * kXStagesMaxH, kAempty = kAfull + 8 * kARingH;
  const uint32_t kMdone = kAempty + 8 * kARingH, kEfree = kMdone + 8 * kDRingH;
  const uint32_t kEdone = kEfree + 8 * kDRingH, kDfull = kEdone + 8;
  // Output staging (out_tma): free for writing (the previous TMA store has
  // read it), and written by all epilogue warps.
  const uint32_t kOfree = kDfull + 8 * kAuxRingH, kOfull = kOfree + 8;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  // Work items: (row group, token tile, K part), a row group being one row
  // tile (single CTAs) or two (pairs: rank r takes row tile 2*group + r); the
  // K parts of an output tile are consecutive items, so CTAs running at the
  // same time share its weight and activation rows. Item t of this CTA covers
  // K blocks [kb_begin(t), kb_end(t)).
  const int nb = p.n_blocks;
  const int ks = kPair ? 1 : p.ksplit;
  const int groups = kPair ? (p.row_tiles + 1) / 2 : p.row_tiles;
  const int n_tiles = groups * p.tok_tiles * ks;
  const int cl = kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ncl = kPair ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int my_tiles = cl < n_tiles ? (n_tiles - 1 - cl) / ncl + 1 : 0;
  auto out_tile = [&](int t) { return ks == 1 ? cl + t * ncl : (cl + t * ncl) / ks; };
  auto row_tile = [&](int t) { return (out_tile(t) / p.tok_tiles) * (kPair ? 2 : 1) + (int)rank; };
  auto tok_tile = [&](int t) { return out_tile(t) % p.tok_tiles; };
  auto kpart = [&](int t) { return ks == 1 ? 0 : (cl + t * ncl) % ks; };
  auto kb_begin = [&](int t) { return ks == 1 ? 0 : kpart(t) * nb / ks; };  // nb * ks < 2^31
  auto kb_end = [&](int t) { return ks == 1 ? nb : (kpart(t) + 1) * nb / ks; };
  // Rank 0's copy of a barrier (rank 1 arrives there).
  auto lead = [&](uint32_t bar) { return kPair ? mapa_shared(bar, 0) : bar; };

  uint32_t tw[512 / (kDecWarpsH * 32)];
  if (warp >= 2 && warp < kEpiWarp0H) {
#pragma unroll
    for (int j = 0; j < 512 / (kDecWarpsH * 32); ++j) tw[j] = __ldg(p.table + (threadIdx.x - 64) + j * kDecWarpsH * 32);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < SW; ++s) {
      mbar_init(kWfull + 8 * s, 1);
      mbar_init(kWempty + 8 * s, kDecWarpsH);
    }
    for (int x = 0; x < kXS; ++x) {
      mbar_init(kXfull + 8 * x, 1);
      mbar_init(kXempty + 8 * x, 1);
    }
    for (int r = 0; r < kARingH; ++r) {
      mbar_init(kAfull + 8 * r, kPair ? 2 * kDecWarpsH : kDecWarpsH);
      mbar_init(kAempty + 8 * r, 1);
    }
    for (int d = 0; d < kDRingH; ++d) {
      mbar_init(kMdone + 8 * d, 1);
      mbar_init(kEfree + 8 * d, kPair ? 2 * kEpiWarpsH : kEpiWarpsH);
    }
    mbar_init(kEdone, kEpiWarpsH);
    for (int a = 0; a < kAuxRingH; ++a) mbar_init(kDfull + 8 * a, 4);
    mbar_init(kOfree, 1);
    mbar_init(kOfull, kEpiWarpsH);
    fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tc::alloc_pair(smem_u32(tmem_slot), kTmColsH);
      tc::relinquish_pair();
    } else {
      tc::alloc(smem_u32(tmem_slot), kTmColsH);
      tc::relinquish();
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if constexpr (kPair) cluster_sync_all();  // both CTAs' barriers and TMEM ready before any remote use
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // -------------------------------------------------------------- weight producer
    if (lane == 0) {
      int it = 0, s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = 0; ok && t < my_tiles; ++t) {
        const int rt = row_tile(t);
        const bool have = rt < p.row_tiles;  // a pair's second row tile may not exist
        const uint8_t* rec = p.packed + (size_t)(have ? rt : 0) * nb * tm::kRecordBytes;
        for (int kb = kb_begin(t), kbe = kb_end(t); kb < kbe; ++kb, ++it) {
          if (it >= SW && !mbar_wait_bounded(kWempty + 8 * s, ph ^ 1, kSiteGemvEmpty)) {
            ok = false;
            break;
          }
          if (have) {
            mbar_arrive_expect_tx(kWfull + 8 * s, tm::kRecordBytes);
            bulk_load(smem_u32(st0 + (size_t)s * tm::kRecordBytes), rec + (size_t)kb * tm::kRecordBytes,
                      tm::kRecordBytes, kWfull + 8 * s);
          } else {
            mbar_arrive(kWfull + 8 * s);  // nothing to load: the decoded rows are never stored
          }
          if (++s == SW) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == kXWarpH) {
    // -------------------------------------------------------------- activation producer
    if (lane == 0) {
      tma_prefetch_desc(&maps.x16);
      const uint64_t keep = l2_policy_evict_last();
      pdl_wait();
      int hj = 0, x = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = 0; ok && t < my_tiles; ++t) {
        const int tok0 = tok_tile(t) * kTokT + (int)rank * kTokLoad;
        for (int kb = kb_begin(t), kbe = kb_end(t); ok && kb < kbe; ++kb) {
          for (int h = 0; h < 2; ++h, ++hj) {
            if (hj >= kXS && !mbar_wait_bounded(kXempty + 8 * x, ph ^ 1, kSiteGemvEmpty)) {
              ok = false;
              break;
            }
            const uint32_t full = kXfull + 8 * x;
            const uint32_t dst = smem_u32(x0 + (size_t)x * kXHalf);
            if constexpr (kPair) {
              // Both halves complete on rank 0's barrier, which expects them.
              if (rank == 0) mbar_arrive_expect_tx(full, 2 * kXHalf);
              tma_load_2d_pair(dst, &maps.x16, kb * 256 + h * 128, tok0, lead(full), keep);
              tma_load_2d_pair(dst + kBoxBytes, &maps.x16, kb * 256 + h * 128 + 64, tok0, lead(full), keep);
            } else {
              mbar_arrive_expect_tx(full, kXHalf);
              tma_load_2d(dst, &maps.x16, kb * 256 + h * 128, tok0, full, keep);
              tma_load_2d(dst + kBoxBytes, &maps.x16, kb * 256 + h * 128 + 64, tok0, full, keep);
            }
            if (++x == kXS) {
              x = 0;
              ph ^= 1;
            }
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA (rank 0 of a pair)
    int it = 0, hj = 0;
    bool ok = rank == 0;
    for (int t = 0; ok && t < my_tiles; ++t) {
      // Folded: D buffer t % 2 holds tile t for its whole K range; it is free
      // once the epilogue has read tile t - 2.
      // Wide: the one accumulator is free once both CTAs' epilogues have read tile t - 1.
      if constexpr (kWide) {
        if (t >= 1) ok = tm::warp_wait_cluster(kEfree, (uint32_t)(t - 1) & 1u, kSiteGemvEmpty);
        if (!ok) break;
      } else if constexpr (kFold) {
        if (t >= kDRingH) ok = tm::warp_wait(kEfree + 8 * (t & 1), ((t >> 1) & 1) ^ 1, kSiteGemvEmpty);
        if (!ok) break;
      }
      const int kb0 = kb_begin(t), kbe = kb_end(t);
      for (int kb = kb0; ok && kb < kbe; ++kb, ++it) {
        const int r = it % kARingH, db = kWide ? 0 : kFold ? (t & 1) : (it & 1);
        ok = kPair ? tm::warp_wait_cluster(kAfull + 8 * r, (it / kARingH) & 1, kSiteGemvFull)
                   : tm::warp_wait(kAfull + 8 * r, (it / kARingH) & 1, kSiteGemvFull);
        // The D buffer is free once the epilogue(s) have read block it - 2.
        if (!kFold && ok && it >= kDRingH)
          ok = kPair ? tm::warp_wait_cluster(kEfree + 8 * db, ((it >> 1) & 1) ^ 1, kSiteGemvEmpty)
                     : tm::warp_wait(kEfree + 8 * db, ((it >> 1) & 1) ^ 1, kSiteGemvEmpty);
        if (!ok) break;
        const uint32_t dcol = tmem + kTmD + (uint32_t)(db * kTokH), acol = tmem + kTmA + 128u * (uint32_t)r;
#pragma unroll 1
        for (int h = 0; h < 2; ++h, ++hj) {
          const int x = hj % kXS;
          ok = kPair ? tm::warp_wait_cluster(kXfull + 8 * x, (hj / kXS) & 1, kSiteGemvFull)
                     : tm::warp_wait(kXfull + 8 * x, (hj / kXS) & 1, kSiteGemvFull);
          if (!ok) break;
          tc::fence_after_sync();
          const uint64_t bdesc = tc::smem_desc_sw128(smem_u32(x0 + (size_t)x * kXHalf), 1024u);
          if (tm::elect_one()) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint64_t bj = bdesc + (uint64_t)(((j >> 2) * kBoxBytes + (j & 3) * 32u) >> 4);
              if constexpr (kPair) {
                tc::mma_f16_ts_pair(dcol, acol + (uint32_t)((8 * h + j) * 8), bj, kIdesc,
                                    kFold ? (kb != kb0 || (h | j) != 0) : (h | j) != 0);
              } else {
                // Folded: accumulate over the tile's K blocks (a fresh sum at its first MMA).
                tc::mma_f16_ts(dcol, acol + (uint32_t)((8 * h + j) * 8), bj, kIdesc,
                               kFold ? (kb != kb0 || (h | j) != 0) : (h | j) != 0);
              }
            }
            if constexpr (kPair) {
              tc::commit_pair(kXempty + 8 * x, kBoth);
            } else {
              tc::commit(kXempty + 8 * x);
            }
          }
          __syncwarp();
        }
        if (!ok) break;
        if (tm::elect_one()) {
          if constexpr (kPair) {
            tc::commit_pair(kAempty + 8 * r, kBoth);
            if (!kFold || kb == kbe - 1) tc::commit_pair(kMdone + 8 * db, kBoth);  // wide: once the tile is summed
          } else {
            tc::commit(kAempty + 8 * r);
            if (!kFold || kb == kbe - 1) tc::commit(kMdone + 8 * db);  // folded: once the tile is summed
          }
        }
        __syncwarp();
      }
    }
    // Free the TMEM once this CTA's epilogue has read its last results.
    mbar_wait_bounded(kEdone, 0, kSiteGemvFull);
    __syncwarp();
    tc::fence_after_sync();
    if constexpr (kPair) {
      tc::dealloc_pair(tmem, kTmColsH);
    } else {
      tc::dealloc(tmem, kTmColsH);
    }
  } else if (warp < kEpiWarp0H) {
    // -------------------------------------------------------------- decoders
    const int dw = warp - 2;
    const int q = warp & 3;
    const int part = dw >> 2;  // groups 4*part .. 4*part+3 of the block
    const int rl = 32 * q + lane;
    tm::build_table(table, tstage, tw, (int)threadIdx.x - 64, kDecWarpsH * 32);
    const uint32_t l4 = (uint32_t)(lane << 2) * 0x01010101u;
    // FP16 A: column c of a block holds K elements 2c, 2c+1; this thread's
    // half of the block is columns 64*part .. 64*part+63.
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + kTmA + (uint32_t)(part * 64);
    const uint32_t off_q0 = tm::kRecQs + (uint32_t)(2 * part) * 2048u + (uint32_t)rl * 16u;
    const uint32_t off_q1 = off_q0 + 2048u;
    const uint32_t off_sg = tm::kRecSigns + (uint32_t)part * 2048u + (uint32_t)rl * 16u;
    const uint32_t off_qh = tm::kRecQh + (uint32_t)part * 512u + (uint32_t)rl * 4u;
    int it = 0, s = 0;
    uint32_t sph = 0;
    bool ok = true;
    for (int t = 0; ok && t < my_tiles; ++t) {
      // Folded: 2^-e of this row (rows past N read the tail's zero entries).
      float fold = 1.f;
      if constexpr (kFold) fold = ldexpf(1.f, -(int)__ldg(p.row_exp + (size_t)row_tile(t) * kRowsH + rl));
      for (int kb = kb_begin(t), kbe = kb_end(t); kb < kbe; ++kb, ++it) {
        const int r = it % kARingH;
        ok = tm::warp_wait(kWfull + 8 * s, sph, kSiteGemvFull);
        if (ok && it >= kARingH) ok = tm::warp_wait(kAempty + 8 * r, ((it / kARingH) & 1) ^ 1, kSiteGemvEmpty);
        if (!ok) break;
        const uint8_t* st = st0 + (size_t)s * tm::kRecordBytes;
        const uint4 a = *reinterpret_cast<const uint4*>(st + off_q0);
        const uint4 c = *reinterpret_cast<const uint4*>(st + off_q1);
        const uint4 gs = *reinterpret_cast<const uint4*>(st + off_sg);
        const uint32_t hw = *reinterpret_cast<const uint32_t*>(st + off_qh);
        const uint32_t scw = *reinterpret_cast<const uint32_t*>(st + tm::kRecScales + rl * 4);
        const uint32_t qw[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
        const uint32_t sw[4] = {gs.x, gs.y, gs.z, gs.w};
        float dfold = 0.f;  // folded: this block's d * 2^-e (exact)
        if constexpr (kFold) {
          dfold = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(st + tm::kRecD + rl * 2))) * fold;
        } else if (part == 0) {
          // The row's d for the epilogue.
          reinterpret_cast<uint32_t*>(aux0 + (size_t)(it % kAuxRingH) * kAuxH)[rl] =
              *reinterpret_cast<const uint16_t*>(st + tm::kRecD + rl * 2);
          __syncwarp();
          if (lane == 0) mbar_arrive(kDfull + 8 * (it % kAuxRingH));
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint32_t e[8];
          tm::decode_group_packed(table, qw[2 * g], qw[2 * g + 1], hw, 2u * (uint32_t)g, sw[g], l4, e);
          // (1 + 2*nibble) of group 4*part + g as an FP16 pair (an odd integer <= 31: exact);
          // folded, times d * 2^-e, rounded to FP16.
          const uint32_t mult = 1u + 2u * ((scw >> (4 * (4 * part + g))) & 0xFu);
          const uint32_t mh = kFold ? (uint32_t)__half_as_ushort(__float2half_rn(dfold * (float)mult))
                                    : (uint32_t)__half_as_ushort(__uint2half_rn(mult));
          const uint32_t m2 = mh | (mh << 16);
          uint32_t v[16];
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {
            uint32_t lo, hi;
            e4m3x4_to_f16x4(e[cc], lo, hi);
            v[2 * cc] = hmul2(lo, m2);
            v[2 * cc + 1] = hmul2(hi, m2);
          }
          tc::st_cols<16>(tq + (uint32_t)(r * 128 + g * 16), v);
        }
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          if (kPair && rank != 0) {
            mbar_arrive_cluster(lead(kAfull + 8 * r));
          } else {
            mbar_arrive(kAfull + 8 * r);
          }
          mbar_arrive(kWempty + 8 * s);
        }
        __syncwarp();
        if (++s == SW) {
          s = 0;
          sph ^= 1;
        }
      }
    }
  } else if constexpr (kWide) {
    // -------------------------------------------------------------- epilogue (wide tiles)
    // Each CTA's 128 rows x 256 tokens leave in two passes of 128 tokens; the
    // two warps of a lane quadrant take 64 tokens each a pass. The one
    // accumulator is released (to both CTAs' MMA issuer) after the second
    // pass's reads.
    const int e = warp - kEpiWarp0H;
    const int q = warp & 3;
    const int h = e >> 2;
    const int rl = 32 * q + lane;
    const uint32_t tq0 = tmem + ((uint32_t)(32 * q) << 16) + kTmD + (uint32_t)(h * 64);
    pdl_wait();  // tok_scale and the output may belong to the previous kernel
    pdl_launch_dependents();
    bool ok = true;
    for (int t = 0; ok && t < my_tiles; ++t) {
      const int rt = row_tile(t), tt = tok_tile(t);
      if (!tm::warp_wait(kMdone, (uint32_t)t & 1u, kSiteGemvFull)) break;
      tc::fence_after_sync();
      const float rs = ldexpf(1.f, (int)__ldg(p.row_exp + (size_t)rt * kRowsH + rl));
      const int row = rt * kRowsH + rl;
      for (int pass = 0; pass < 2; ++pass) {
        float acc[64];
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 16) {
          const uint32_t off[2] = {(uint32_t)c0, (uint32_t)c0 + 8u};
          float cv[2][8];
          tc::ld_x8_multi<2>(tq0 + (uint32_t)(pass * kTokH), off, cv);
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[c0 + 8 * j + i] = cv[j][i] * rs;
        }
        if (pass == 1) {
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) {
            if (rank != 0) {
              mbar_arrive_cluster(lead(kEfree));
            } else {
              mbar_arrive(kEfree);
            }
          }
          __syncwarp();
        }
        const int tok0 = tt * kTokT + pass * kTokH + h * 64;
        const float4* ts = reinterpret_cast<const float4*>(p.tok_scale + tok0);
        if (p.out_tma) {
          // As the single-CTA epilogue: bf16 tile of 128 tokens in shared memory, one TMA store.
          const uint32_t ph = (uint32_t)(2 * t + pass) & 1u;
          if (e == 0 && lane == 0) {
            bulk_wait_group_read0();
            mbar_arrive(kOfree);
          }
          if (!tm::warp_wait(kOfree, ph, kSiteGemvEmpty)) {
            ok = false;
            break;
          }
          __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(ostage) + (size_t)(h * 64) * kRowsH + rl;
#pragma unroll
          for (int c = 0; c < 64; c += 4) {
            const float4 sc = __ldg(ts + c / 4);
            stg[(size_t)(c + 0) * kRowsH] = __float2bfloat16_rn(acc[c + 0] * sc.x);
            stg[(size_t)(c + 1) * kRowsH] = __float2bfloat16_rn(acc[c + 1] * sc.y);
            stg[(size_t)(c + 2) * kRowsH] = __float2bfloat16_rn(acc[c + 2] * sc.z);
            stg[(size_t)(c + 3) * kRowsH] = __float2bfloat16_rn(acc[c + 3] * sc.w);
          }
          fence_proxy_async_shared();  // the TMA store reads the tile through the async proxy
          __syncwarp();
          if (lane == 0) mbar_arrive(kOfull);
          if (e == 0) {
            if (!tm::warp_wait(kOfull, ph, kSiteGemvFull)) {
              ok = false;
              break;
            }
            if (lane == 0) {
              tma_store_2d(&maps.out, rt * kRowsH, tt * kTokT + pass * kTokH, smem_u32(ostage));
              bulk_commit_group();
            }
          }
          __syncwarp();
        } else {
#pragma unroll
          for (int c = 0; c < 64; c += 4) {
            const float4 sc = __ldg(ts + c / 4);
            store_out_h(p, row, tok0 + c + 0, acc[c + 0] * sc.x);
            store_out_h(p, row, tok0 + c + 1, acc[c + 1] * sc.y);
            store_out_h(p, row, tok0 + c + 2, acc[c + 2] * sc.z);
            store_out_h(p, row, tok0 + c + 3, acc[c + 3] * sc.w);
          }
        }
      }
    }
    if (p.out_tma && e == 0 && lane == 0) bulk_wait_group0();  // the last tile's store is written
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(kEdone);
    __syncwarp();
  } else {
    // -------------------------------------------------------------- epilogue
    const int e = warp - kEpiWarp0H;
    const int q = warp & 3;
    const int h = e >> 2;  // tokens h*64 .. h*64+63 of the tile
    const int rl = 32 * q + lane;
    const uint32_t tq0 = tmem + ((uint32_t)(32 * q) << 16) + kTmD + (uint32_t)(h * 64);
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.f;
    pdl_wait();  // tok_scale and the output may belong to the previous kernel
    pdl_launch_dependents();
    int it = 0;
    bool ok = true;
    for (int t = 0; ok && t < my_tiles; ++t) {
      const int rt = row_tile(t), tt = tok_tile(t);
      if constexpr (kFold) {
        // The tile's sum over its whole K range, in D buffer t % 2, times 2^e of the row.
        const int db = t & 1;
        if (!tm::warp_wait(kMdone + 8 * db, (t >> 1) & 1, kSiteGemvFull)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const float rs = ldexpf(1.f, (int)__ldg(p.row_exp + (size_t)rt * kRowsH + rl));
        const uint32_t tq = tq0 + (uint32_t)(db * kTokH);
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 16) {
          const uint32_t off[2] = {(uint32_t)c0, (uint32_t)c0 + 8u};
          float cv[2][8];
          tc::ld_x8_multi<2>(tq, off, cv);
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[c0 + 8 * j + i] = cv[j][i] * rs;
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(kEfree + 8 * db);
        __syncwarp();
      }
      for (int kb = kb_begin(t), kbe = kb_end(t); !kFold && kb < kbe; ++kb, ++it) {
        const int db = it & 1;
        if (!tm::warp_wait(kDfull + 8 * (it % kAuxRingH), (it / kAuxRingH) & 1, kSiteGemvFull) ||
            !tm::warp_wait(kMdone + 8 * db, (it >> 1) & 1, kSiteGemvFull)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const float dv = __half2float(__ushort_as_half(
            (unsigned short)reinterpret_cast<const uint32_t*>(aux0 + (size_t)(it % kAuxRingH) * kAuxH)[rl]));
        const uint32_t tq = tq0 + (uint32_t)(db * kTokH);
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 16) {
          const uint32_t off[2] = {(uint32_t)c0, (uint32_t)c0 + 8u};
          float cv[2][8];
          tc::ld_x8_multi<2>(tq, off, cv);
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int i = 0; i < 8; i += 2)
              fma2(acc[c0 + 8 * j + i], acc[c0 + 8 * j + i + 1], cv[j][i], cv[j][i + 1], dv, dv);
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          if (kPair && rank != 0) {
            mbar_arrive_cluster(lead(kEfree + 8 * db));
          } else {
            mbar_arrive(kEfree + 8 * db);
          }
        }
        __syncwarp();
      }
      if (!ok) break;
      if (ks > 1) {
        // K split: publish this warp's partial (32 rows x 64 tokens, FP32,
        // token quads major so that a warp's 16-byte stores are contiguous)
        // and count in; the last contributor of the tile sums the partials
        // in K-part order (its own from registers) and goes on to the store.
        const int ot = out_tile(t), kp = kpart(t);
        // Element (part j, token quad c/4 of this warp's half, row rl) of the tile's partials.
        float4* part = reinterpret_cast<float4*>(p.partials) + (size_t)ot * ks * (kTokH / 4) * kRowsH +
                       (h * 16) * kRowsH + rl;
        constexpr int kPartStride = (kTokH / 4) * kRowsH;  // float4s per part
#pragma unroll
        for (int c = 0; c < 64; c += 4)
          __stcg(part + kp * kPartStride + (c / 4) * kRowsH, make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]));
        __threadfence();  // every lane's partial is visible GPU-wide before the count goes up
        __syncwarp();
        int* counter = p.split_counters + (size_t)ot * kEpiWarpsH + e;
        int last = 0;
        if (lane == 0) last = atomic_add_acq_rel_gpu(counter, 1) == ks - 1;
        last = __shfl_sync(0xFFFFFFFFu, last, 0);
        if (!last) {
#pragma unroll
          for (int i = 0; i < 64; ++i) acc[i] = 0.f;
          continue;
        }
        if (lane == 0) *counter = 0;  // every part has arrived: zero again for the next launch
        __threadfence();              // the other parts' partials are read after the count was seen
        // Sum in part order (this warp's own part read back: it is in L2).
#pragma unroll
        for (int c = 0; c < 64; c += 4) {
          float4 sum = __ldcg(part + (c / 4) * kRowsH);
#pragma unroll 1
          for (int j = 1; j < ks; ++j) {
            const float4 v = __ldcg(part + j * kPartStride + (c / 4) * kRowsH);
            sum.x += v.x;
            sum.y += v.y;
            sum.z += v.z;
            sum.w += v.w;
          }
          acc[c] = sum.x;
          acc[c + 1] = sum.y;
          acc[c + 2] = sum.z;
          acc[c + 3] = sum.w;
        }
      }
      // The tile's 64 tokens, 8 at a time: their scales as two float4 loads
      // (tok_scale is padded to whole tiles), issued before the previous
      // chunk's stores so that the load latency overlaps them.
      const int row = rt * kRowsH + rl, tok0 = tt * kTokH + h * 64;
      const float4* ts = reinterpret_cast<const float4*>(p.tok_scale + tok0);
      if (p.out_tma) {
        // bf16 tile into shared memory ([token][row], as the TMA box), then one
        // TMA store: the epilogue moves on to the next tile at once. The
        // previous tile's store must have read the staging tile first.
        if (e == 0 && lane == 0) {
          bulk_wait_group_read0();
          mbar_arrive(kOfree);
        }
        if (!tm::warp_wait(kOfree, (uint32_t)t & 1u, kSiteGemvEmpty)) break;
        __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(ostage) + (size_t)(h * 64) * kRowsH + rl;
        float4 n4a = __ldg(ts), n4b = __ldg(ts + 1);
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
          const float sc[8] = {n4a.x, n4a.y, n4a.z, n4a.w, n4b.x, n4b.y, n4b.z, n4b.w};
          if (c + 8 < 64) {
            n4a = __ldg(ts + (c + 8) / 4);
            n4b = __ldg(ts + (c + 8) / 4 + 1);
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            stg[(size_t)(c + i) * kRowsH] = __float2bfloat16_rn(acc[c + i] * sc[i]);
            acc[c + i] = 0.f;
          }
        }
        fence_proxy_async_shared();  // the TMA store reads the tile through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive(kOfull);
        if (e == 0) {
          if (!tm::warp_wait(kOfull, (uint32_t)t & 1u, kSiteGemvFull)) break;
          if (lane == 0) {
            tma_store_2d(&maps.out, rt * kRowsH, tt * kTokH, smem_u32(ostage));
            bulk_commit_group();
          }
        }
        __syncwarp();
        continue;
      }
      const bool odd = (lane & 1) != 0;
      const bool pack4 = (p.ldo % 4 == 0) && ((uintptr_t)p.out % (p.out_bf16 ? 8u : 16u) == 0);
      const bool pack2 = (p.ldo % 2 == 0) && ((uintptr_t)p.out % (p.out_bf16 ? 4u : 8u) == 0);
      float4 n4a = __ldg(ts), n4b = __ldg(ts + 1);
#pragma unroll
      for (int c = 0; c < 64; c += 8) {
        const float sc[8] = {n4a.x, n4a.y, n4a.z, n4a.w, n4b.x, n4b.y, n4b.z, n4b.w};
        if (c + 8 < 64) {
          n4a = __ldg(ts + (c + 8) / 4);
          n4b = __ldg(ts + (c + 8) / 4 + 1);
        }
        if (pack4) {
          // Four rows per store: a 4 x 4 transpose within each quad of lanes
          // (two exchange rounds) leaves lane L holding token i + (L & 3) for
          // rows (L & ~3) .. (L & ~3) + 3 (N % 8 == 0: all four exist).
          const int ql = lane & 3;
          const bool hi2 = ql >= 2, qodd = (ql & 1) != 0;
#pragma unroll
          for (int i = 0; i < 8; i += 4) {
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = acc[c + i + j] * sc[i + j];
            // Exchange step 1 (lane ^ 2): lanes 0-1 keep tokens 0-1, lanes 2-3 tokens 2-3.
            const float a0 = hi2 ? v[2] : v[0], a1 = hi2 ? v[3] : v[1];
            const float r0 = __shfl_xor_sync(0xFFFFFFFFu, hi2 ? v[0] : v[2], 2);
            const float r1 = __shfl_xor_sync(0xFFFFFFFFu, hi2 ? v[1] : v[3], 2);
            // Exchange step 2 (lane ^ 1): even lanes keep the first of their two tokens.
            const float g0 = __shfl_xor_sync(0xFFFFFFFFu, qodd ? a0 : a1, 1);  // row L^1
            const float g1 = __shfl_xor_sync(0xFFFFFFFFu, qodd ? r0 : r1, 1);  // row L^3
            const float own = qodd ? a1 : a0, own2 = qodd ? r1 : r0;           // rows L, L^2
            float o[4];
#pragma unroll
            for (int pos = 0; pos < 4; ++pos)
              o[pos] = pos == ql ? own : pos == (ql ^ 2) ? own2 : pos == (ql ^ 1) ? g0 : g1;
            const int tok = tok0 + c + i + ql, r0w = row - ql;
            if (r0w < p.n_rows && tok < p.m) {
              const int64_t at = (int64_t)tok * p.ldo + r0w;
              if (p.out_bf16) {
                const __nv_bfloat162 b01 = __floats2bfloat162_rn(o[0], o[1]), b23 = __floats2bfloat162_rn(o[2], o[3]);
                *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + at) =
                    make_uint2(*reinterpret_cast<const uint32_t*>(&b01), *reinterpret_cast<const uint32_t*>(&b23));
              } else {
                *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + at) = make_float4(o[0], o[1], o[2], o[3]);
              }
            }
          }
        } else if (pack2) {
          // Two rows per store: lanes L and L^1 trade one value, so that the
          // even lane holds rows L, L+1 of token i and the odd lane rows L-1, L
          // of token i+1 (N % 8 == 0: both rows exist when the first does).
#pragma unroll
          for (int i = 0; i < 8; i += 2) {
            const float v0 = acc[c + i] * sc[i], v1 = acc[c + i + 1] * sc[i + 1];
            const float got = __shfl_xor_sync(0xFFFFFFFFu, odd ? v0 : v1, 1);
            const int tok = tok0 + c + i + (odd ? 1 : 0), r0 = row - (odd ? 1 : 0);
            if (r0 < p.n_rows && tok < p.m) {
              const int64_t at = (int64_t)tok * p.ldo + r0;
              if (p.out_bf16) {
                *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(p.out) + at) =
                    __floats2bfloat162_rn(odd ? got : v0, odd ? v1 : got);
              } else {
                *reinterpret_cast<float2*>(reinterpret_cast<float*>(p.out) + at) =
                    make_float2(odd ? got : v0, odd ? v1 : got);
              }
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) store_out_h(p, row, tok0 + c + i, acc[c + i] * sc[i]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[c + i] = 0.f;
      }
    }
    if (p.out_tma && e == 0 && lane == 0) bulk_wait_group0();  // the last tile's store is written
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(kEdone);
    __syncwarp();
  }
  // Neither CTA of a pair leaves while the other may still use its shared
  // memory or TMEM (remote arrivals, the pair MMAs).
  if constexpr (kPair) cluster_sync_all();
}

// Eight E4M3 values (bytes of raw, in order) -> eight FP16 values of E4M3 * f
// (f = 2^(e_g - e_max), or NaN), each rounded to nearest once.
__device__ __forceinline__ uint4 x16_from_e4m3x8(uint2 raw, float f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t two = ((i < 2 ? raw.x : raw.y) >> (16 * (i & 1))) & 0xFFFFu;
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)two, __NV_E4M3);
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&hr));
    const __half2 o = __floats2half2_rn(v.x * f, v.y * f);
    w[i] = *reinterpret_cast<const uint32_t*>(&o);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// The largest scale code of a row (0xFF, a NaN group, counts as 0), reduced
// over the CTA; every thread returns it. `codes` holds the row's k/32 codes.
__device__ __forceinline__ int row_max_code(const uint8_t* codes, int64_t groups) {
  int emax = 0;
  for (int64_t g = threadIdx.x; g < groups; g += blockDim.x) {
    const int e = codes[g];
    emax = max(emax, e == 0xFF ? 0 : e);
  }
  for (int o = 16; o > 0; o >>= 1) emax = max(emax, __shfl_xor_sync(0xFFFFFFFFu, emax, o));
  __shared__ int wmax[32];
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = emax;
  __syncthreads();
  if (threadIdx.x < 32) {
    int v = threadIdx.x < (blockDim.x >> 5) ? wmax[threadIdx.x] : 0;
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    if (threadIdx.x == 0) wmax[0] = v;
  }
  __syncthreads();
  return wmax[0];
}

// One CTA per token row: e_max over the row's UE8M0 scales, then every E4M3
// value times 2^(e_g - e_max) rounded to FP16; tok_scale = 2^(e_max - 127).
// A scale code 0xFF (NaN) makes its group NaN.
__global__ void iq3s_x16_kernel(const uint8_t* __restrict__ xq, int64_t ldxq, const uint8_t* __restrict__ xs,
                                int64_t ldxs, int64_t k, uint16_t* __restrict__ x16, int64_t ld,
                                float* __restrict__ tok_scale) {
  const int64_t t = blockIdx.x;
  const uint8_t* srow = xs + t * ldxs;
  const int emax = row_max_code(srow, k / 32);
  if (threadIdx.x == 0) tok_scale[t] = e8m0_to_float((uint32_t)emax);
  const uint8_t* qrow = xq + t * ldxq;
  uint16_t* orow = x16 + t * ld;
  for (int64_t c = threadIdx.x; c < k / 8; c += blockDim.x) {  // 8 values per step
    const int e = srow[c / 4];
    const uint2 raw = *reinterpret_cast<const uint2*>(qrow + c * 8);
    const float f = e == 0xFF ? __uint_as_float(0x7FC00000u) : ldexpf(1.0f, e - emax);
    *reinterpret_cast<uint4*>(orow + c * 8) = x16_from_e4m3x8(raw, f);
  }
}

uint32_t gemm_f16_smem_bytes(int wstages, bool out_stage) { return gemm_f16_smem(wstages, out_stage); }
int gemm_f16_max_wstages() { return kMaxWStagesH; }

cudaError_t launch_x16(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int m, int64_t k,
                       uint16_t* x16, int64_t ld, float* tok_scale, cudaStream_t stream) {
  iq3s_x16_kernel<<<(unsigned)m, 256, 0, stream>>>(xq, ldxq, xs, ldxs, k, x16, ld, tok_scale);
  return cudaGetLastError();
}

// Activation quantization fused into the FP16 conversion: bf16 (T = uint16_t)
// or f32 rows -> the MXFP8 codes mambo_quantize_mxfp8 forms (round to nearest
// even: quad of lanes per 32-value group, as quantize_mxfp8_kernel) -> the
// FP16 operand and token scale iq3s_x16_kernel forms from those codes. One
// CTA per token; the row's E4M3 bytes and scale codes wait in shared memory
// (k + k/32 bytes) while the CTA finds the largest code. Rows 16-byte aligned;
// k % 256 == 0, so every warp's lanes stay together through the quad shuffles.
template <typename T>
__global__ void __launch_bounds__(256) iq3s_x16_quant_kernel(const T* __restrict__ x, int64_t ldx, int64_t k,
                                                             uint16_t* __restrict__ x16, int64_t ld,
                                                             float* __restrict__ tok_scale) {
  extern __shared__ __align__(16) uint8_t qsm[];
  uint8_t* qrow = qsm;      // [k] E4M3 bytes
  uint8_t* srow = qsm + k;  // [k/32] scale codes
  const int64_t t = blockIdx.x;
  const T* xrow = x + t * ldx;
  pdl_wait();  // the activations may come from the previous kernel
  for (int64_t c = threadIdx.x; c < k / 8; c += blockDim.x) {  // chunk of 8 values; group c/4
    float v[8];
    if constexpr (sizeof(T) == 2) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(xrow + c * 8));
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      }
    } else {
      const float4 a = __ldg(reinterpret_cast<const float4*>(xrow + c * 8));
      const float4 b = __ldg(reinterpret_cast<const float4*>(xrow + c * 8) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    uint2 q;
    const uint32_t code = mxfp8_quad_rne(v, q);
    *reinterpret_cast<uint2*>(qrow + c * 8) = q;
    if ((c & 3) == 0) srow[c / 4] = (uint8_t)code;
  }
  __syncthreads();
  const int emax = row_max_code(srow, k / 32);
  pdl_launch_dependents();
  if (threadIdx.x == 0) tok_scale[t] = e8m0_to_float((uint32_t)emax);
  uint16_t* orow = x16 + t * ld;
  for (int64_t c = threadIdx.x; c < k / 8; c += blockDim.x) {
    const int e = srow[c / 4];
    const uint2 raw = *reinterpret_cast<const uint2*>(qrow + c * 8);
    const float f = e == 0xFF ? __uint_as_float(0x7FC00000u) : ldexpf(1.0f, e - emax);
    *reinterpret_cast<uint4*>(orow + c * 8) = x16_from_e4m3x8(raw, f);
  }
}

size_t x16_quant_smem_bytes(int64_t k) { return (size_t)k + (size_t)(k / 32); }

cudaError_t launch_x16_quant(const void* x, int x_dtype, int64_t ldx, int m, int64_t k, uint16_t* x16, int64_t ld,
                             float* tok_scale, cudaStream_t stream) {
  const size_t smem = x16_quant_smem_bytes(k);
  const void* kern = x_dtype == MAMBO_BF16 ? (const void*)iq3s_x16_quant_kernel<uint16_t>
                                           : (const void*)iq3s_x16_quant_kernel<float>;
  cudaError_t e = ensure_smem_attribute(kern, smem);
  if (e != cudaSuccess) return e;
  if (x_dtype == MAMBO_BF16)
    return launch_pdl(kern, dim3((unsigned)m), dim3(256), smem, stream, (const uint16_t*)x, ldx, k, x16, ld,
                      tok_scale);
  return launch_pdl(kern, dim3((unsigned)m), dim3(256), smem, stream, (const float*)x, ldx, k, x16, ld, tok_scale);
}

cudaError_t launch_gemm_f16(const GemmF16Params& p, const GemmF16Maps& maps, int grid, cudaStream_t stream,
                            bool fold) {
  const uint32_t smem = gemm_f16_smem(p.wstages, p.out_tma != 0);
  const void* kern = fold ? (const void*)iq3s_gemm_f16_kernel<false, true> : (const void*)iq3s_gemm_f16_kernel<false>;
  cudaError_t e = ensure_smem_attribute(kern, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(kThreadsH), smem, stream, p, maps);
}

int gemm_f16_pair_max_clusters(int wstages, bool out_stage) {
  const void* kern = (const void*)iq3s_gemm_f16_kernel<true>;
  const uint32_t smem = gemm_f16_smem(wstages, out_stage);
  if (ensure_smem_attribute(kern, smem) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(kThreadsH);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
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

cudaError_t launch_gemm_f16_pair(const GemmF16Params& p, const GemmF16Maps& maps, int clusters, cudaStream_t stream,
                                 bool wide) {
  const uint32_t smem = gemm_f16_smem(p.wstages, p.out_tma != 0);
  const void* kern = wide ? (const void*)iq3s_gemm_f16_kernel<true, true> : (const void*)iq3s_gemm_f16_kernel<true>;
  cudaError_t e = ensure_smem_attribute(kern, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl_cluster(kern, dim3(2 * clusters), dim3(kThreadsH), smem, stream, 2, p, maps);
}

}  // namespace mambo
