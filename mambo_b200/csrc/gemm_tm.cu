// IQ3_S x MXFP8 GEMM for prefill-sized M on the 5th-generation tensor cores
// (tcgen05, sm_100a), with the decoded weight operand kept in tensor memory.
//
// Same arithmetic as the reference's large-M kernel
// (src/python/mambo/kernels/iq3_s_fp8.py:225-276): per 32-weight group g,
// P_g = sum_k E4M3(w) * E4M3(x) * 2^e(x, g) is formed by the tensor core in
// FP32 (block-scaled MMA: the activation's UE8M0 scale is applied in the MMA,
// the weight side's scale is 2^0), then out += P_g * d * (1 + 2*nibble_g) in
// FP32, group by group.
//
// Tiles: 128 weight rows (MMA M, TMEM lanes) x 128 tokens (MMA N). One
// persistent CTA per SM takes tiles blockIdx.x, + gridDim.x, ...; a tile walks
// every K block (a "unit": 128 rows x 256 K). Roles:
//  * warp 0, weight producer: one bulk copy of the unit's tile-major record
//    (14080 bytes) into a ring of weight stages, refilled once decoded.
//  * activation producer warp: after the previous kernel has finished
//    (programmatic dependent launch), two 2D TMA copies of the unit's 128 x 256
//    activation block in 128-byte swizzled rows (rows past M read as zero) and one
//    bulk copy of its scales, already in the tensor core's scale-factor atom
//    layout (written by iq3s_xs_atoms_kernel), into a ring of 3 slots.
//  * decoder warps (8): as in the GEMV, a thread owns a weight row (its TMEM
//    lane) and half of the K block, expands the codes through the lane-private
//    codebook and writes E4M3 bytes to its lane with tcgen05.st (A ring of 2).
//  * warp 1, MMA: per unit, two tcgen05.cp move the activation scales to TMEM
//    (replicated into the four lane quadrants); per group one block-scaled
//    tcgen05.mma (M=128, N=128, K=32) into one of two D buffers, committed to
//    that buffer's barrier.
//  * 8 epilogue warps, two per TMEM lane quadrant (64 tokens each): a thread
//    owns a weight row, reads its group partials with tcgen05.ld and
//    accumulates P_g * d*(1+2*nibble) in FP32 registers; at the end of the
//    tile it stores its row of the output (32 consecutive rows per warp and
//    token: coalesced).
#include "kernels.cuh"
#include "tcgen05.cuh"
#include "iq3s_tm.cuh"

namespace mambo {

namespace {

constexpr int kRowsG = 128;  // weight rows per tile = MMA M = TMEM lanes
constexpr int kTokG = 128;   // tokens per tile = MMA N
constexpr int kDecWarpsG = 8, kEpiWarpsG = 8;
constexpr int kARingG = 2;     // decoded A operands in TMEM
constexpr int kDRingG = 2;     // per-group D buffers in TMEM
constexpr int kXStagesG = 3;   // activation slots
constexpr int kMaxWStagesG = 6;
constexpr uint32_t kBTileG = kTokG * 256u;  // B operand of a unit: 32 KB
constexpr uint32_t kSfBytesG = 1024;        // a unit's activation scales: two 32 x 16-byte atoms
constexpr uint32_t kXSlotG = kBTileG + kSfBytesG;
constexpr uint32_t kAuxG = kRowsG * 8;  // rows' (d, scale word) of a unit
constexpr uint32_t kBarBytesG = 512;
// TMEM columns: A ring, D ring, the weights' scale factors (all 2^0), then a
// scale-factor slot (8 columns) per activation slot. The MMA reads a
// scale-factor matrix from 4 columns at the address it is given (column +
// row / 32), so every such address is a multiple of 4.
constexpr uint32_t kTmA = 0, kTmD = 64u * kARingG, kTmSfa = kTmD + kDRingG * (uint32_t)kTokG, kTmSfb = kTmSfa + 16u;
constexpr uint32_t kTmColsG = 512;
static_assert(kTmSfb + 8u * kXStagesG <= kTmColsG, "TMEM plan exceeds 512 columns");
static_assert(kTmSfa % 16u == 0 && kTmSfb % 8u == 0, "scale-factor columns must stay aligned");
// Warps: weight producer, MMA, decoders, epilogue, activation producer.
constexpr int kThreadsG = (3 + kDecWarpsG + kEpiWarpsG) * 32;
constexpr int kEpiWarp0G = 2 + kDecWarpsG, kXWarpG = kEpiWarp0G + kEpiWarpsG;

__host__ __device__ constexpr uint32_t align_up_g(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline uint32_t gemm_smem(int wstages) {
  return tm::kTableBytes + 1024 + align_up_g((uint32_t)wstages * tm::kRecordBytes, 1024) + kXStagesG * kXSlotG +
         kARingG * kAuxG + tm::kTableStageBytes + kBarBytesG;
}

__device__ __forceinline__ void store_out_g(const GemmTmParams& p, int row, int tok, float v) {
  if (row < p.n_rows && tok < p.m) {
    if (p.out_bf16) {
      reinterpret_cast<__nv_bfloat16*>(p.out)[(int64_t)tok * p.ldo + row] = __float2bfloat16_rn(v);
    } else {
      reinterpret_cast<float*>(p.out)[(int64_t)tok * p.ldo + row] = v;
    }
  }
}

}  // namespace

__global__ void __launch_bounds__(kThreadsG, 1)
    iq3s_gemm_tm_kernel(const __grid_constant__ GemmTmParams p, const __grid_constant__ GemmTmMaps maps) {
  // B tile: two [128 tokens][128 bytes] boxes in the 128-byte-swizzled
  // K-major layout (8-row atoms 1024 bytes apart); group g (32 bytes of K)
  // starts 32*(g%4) bytes into box g/4's rows.
  constexpr uint32_t kBoxBytes = kTokG * 128u;
  constexpr uint32_t kIdesc = tc::idesc_mx_e4m3(kRowsG, kTokG, 0, 0);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The codebook sits at the start of dynamic shared memory; the stages
  // follow, aligned to 1024 bytes at run time.
  uint8_t* table = smem_raw;
  uint8_t* st0 = smem_raw + tm::kTableBytes + ((1024u - ((smem_u32(smem_raw) + tm::kTableBytes) & 1023u)) & 1023u);
  const int SW = p.wstages;
  uint8_t* x0 = st0 + align_up_g((uint32_t)SW * tm::kRecordBytes, 1024);  // activation slots
  uint8_t* aux0 = x0 + (size_t)kXStagesG * kXSlotG;
  uint32_t* tstage = reinterpret_cast<uint32_t*>(aux0 + kARingG * kAuxG);
  uint64_t* bars = reinterpret_cast<uint64_t*>(aux0 + kARingG * kAuxG + tm::kTableStageBytes);
  uint32_t* tmem_slot =
      reinterpret_cast<uint32_t*>(bars + 2 * kMaxWStagesG + 2 * kXStagesG + 2 * kARingG + 2 * kDRingG + 1);
  const uint32_t bar0 = smem_u32(bars);
  // Barriers: per weight stage wfull (landed) / wempty (decoded); per
  // activation slot xfull (landed) / xempty (its MMAs complete); per A slot
  // afull (decoded, rows' scales written) / aempty (its MMAs complete); per D
  // buffer mdone (MMA complete) / efree (read by the epilogue); edone.
  const uint32_t kWfull = bar0, kWempty = bar0 + 8 * kMaxWStagesG;
  const uint32_t kXfull = bar0 + 16 * kMaxWStagesG, kXempty = kXfull + 8 * kXStagesG;
  const uint32_t kAfull = kXempty + 8 * kXStagesG, kAempty = kAfull + 8 * kARingG;
  const uint32_t kMdone = kAempty + 8 * kARingG, kEfree = kMdone + 8 * kDRingG;
  const uint32_t kEdone = kEfree + 8 * kDRingG;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.n_blocks, n_tiles = p.row_tiles * p.tok_tiles;
  const int my_tiles = (int)blockIdx.x < n_tiles ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

  // Decoder threads fetch the 2 KB codebook now, so that its latency overlaps
  // the set-up below.
  uint32_t tw[512 / (kDecWarpsG * 32)];
  if (warp >= 2 && warp < kEpiWarp0G) {
#pragma unroll
    for (int j = 0; j < 512 / (kDecWarpsG * 32); ++j) tw[j] = __ldg(p.table + (threadIdx.x - 64) + j * kDecWarpsG * 32);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < SW; ++s) {
      mbar_init(kWfull + 8 * s, 1);
      mbar_init(kWempty + 8 * s, kDecWarpsG);
    }
    for (int x = 0; x < kXStagesG; ++x) {
      mbar_init(kXfull + 8 * x, 1);
      mbar_init(kXempty + 8 * x, 1);
    }
    for (int r = 0; r < kARingG; ++r) {
      mbar_init(kAfull + 8 * r, kDecWarpsG);
      mbar_init(kAempty + 8 * r, 1);
    }
    for (int d = 0; d < kDRingG; ++d) {
      mbar_init(kMdone + 8 * d, 1);
      mbar_init(kEfree + 8 * d, kEpiWarpsG);
    }
    mbar_init(kEdone, kEpiWarpsG);
    fence_barrier_init();
  }
  if (warp == 1) {
    tc::alloc(smem_u32(tmem_slot), kTmColsG);
    tc::relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  // ------------------------------------------------------------------ weight producer
  if (warp == 0) {
    if (lane == 0) {
      int it = 0, s = 0;
      uint32_t ph = 0;  // phase of stage s
      for (int t = 0; t < my_tiles; ++t) {
        const int rt = ((int)blockIdx.x + t * (int)gridDim.x) / p.tok_tiles;
        const uint8_t* rec = p.packed + (size_t)rt * nb * tm::kRecordBytes;
        for (int kb = 0; kb < nb; ++kb, ++it) {
          if (it >= SW && !mbar_wait_bounded(kWempty + 8 * s, ph ^ 1, kSiteGemvEmpty)) return;
          mbar_arrive_expect_tx(kWfull + 8 * s, tm::kRecordBytes);
          bulk_load(smem_u32(st0 + (size_t)s * tm::kRecordBytes), rec + (size_t)kb * tm::kRecordBytes,
                    tm::kRecordBytes, kWfull + 8 * s);
          if (++s == SW) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------------ activation producer
  if (warp == kXWarpG) {
    if (lane == 0) {
      tma_prefetch_desc(&maps.x);
      const uint64_t keep = l2_policy_evict_last();  // every row tile reads them
      pdl_wait();
      const int nq = 2 * nb;  // K quads (4 groups of 32)
      int it = 0, x = 0;
      uint32_t ph = 0;
      for (int t = 0; t < my_tiles; ++t) {
        const int tt = ((int)blockIdx.x + t * (int)gridDim.x) % p.tok_tiles;
        for (int kb = 0; kb < nb; ++kb, ++it) {
          if (it >= kXStagesG && !mbar_wait_bounded(kXempty + 8 * x, ph ^ 1, kSiteGemvEmpty)) return;
          const uint32_t full = kXfull + 8 * x, slot = smem_u32(x0 + (size_t)x * kXSlotG);
          mbar_arrive_expect_tx(full, kXSlotG);
          tma_load_2d(slot, &maps.x, kb * 256, tt * kTokG, full, keep);
          tma_load_2d(slot + kBoxBytes, &maps.x, kb * 256 + 128, tt * kTokG, full, keep);
          bulk_load_hint(slot + kBTileG, p.xs_atoms + ((size_t)tt * nq + 2 * kb) * 512, kSfBytesG, full, keep);
          if (++x == kXStagesG) {
            x = 0;
            ph ^= 1;
          }
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------------ MMA
  if (warp == 1) {
    int it = 0, gi = 0;
    bool ok = true;
    for (int t = 0; ok && t < my_tiles; ++t) {
      for (int kb = 0; kb < nb; ++kb, ++it) {
        const int r = it % kARingG, x = it % kXStagesG;
        ok = tm::warp_wait(kAfull + 8 * r, (it / kARingG) & 1, kSiteGemvFull) &&
             tm::warp_wait(kXfull + 8 * x, (it / kXStagesG) & 1, kSiteGemvFull);
        if (!ok) break;
        tc::fence_after_sync();
        const uint32_t xslot = smem_u32(x0 + (size_t)x * kXSlotG);
        const uint64_t bdesc = tc::smem_desc_sw128(xslot, 1024u);
        const uint32_t sfb = tmem + kTmSfb + 8u * (uint32_t)x, acol = tmem + kTmA + 64u * (uint32_t)r;
        if (tm::elect_one()) {
          // Groups 0-3 and 4-7 of the unit: 32 rows x 16 bytes each, 8-row core
          // matrices 128 bytes apart. Ordered before this thread's MMAs.
          tc::cp_32x128b_warpx4(sfb, tc::smem_desc(xslot + kBTileG, 128u, 128u));
          tc::cp_32x128b_warpx4(sfb + 4u, tc::smem_desc(xslot + kBTileG + 512u, 128u, 128u));
        }
        __syncwarp();
#pragma unroll 1
        for (int g = 0; g < 8; ++g, ++gi) {
          const int ds = gi & 1;
          if (gi >= kDRingG && !tm::warp_wait(kEfree + 8 * ds, ((gi >> 1) & 1) ^ 1, kSiteGemvEmpty)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          if (tm::elect_one()) {
            tc::mma_mx_e4m3_ts(tmem + kTmD + (uint32_t)(ds * kTokG), acol + (uint32_t)(g * 8),
                               bdesc + (uint64_t)((((uint32_t)g >> 2) * kBoxBytes + ((uint32_t)g & 3u) * 32u) >> 4),
                               kIdesc | ((uint32_t)(g & 3) << 4),
                               tmem + kTmSfa, sfb + 4u * (uint32_t)(g >> 2), 0);
            tc::commit(kMdone + 8 * ds);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (tm::elect_one()) {
          tc::commit(kAempty + 8 * r);
          tc::commit(kXempty + 8 * x);
        }
        __syncwarp();
      }
    }
    // Free the TMEM once every epilogue warp has read its last partials.
    mbar_wait_bounded(kEdone, 0, kSiteGemvFull);
    __syncwarp();
    tc::fence_after_sync();
    tc::dealloc(tmem, kTmColsG);
    return;
  }

  // ------------------------------------------------------------------ decoders
  if (warp < kEpiWarp0G) {
    const int dw = warp - 2;
    const int q = warp & 3;        // TMEM lane quadrant this warp may access
    const int part = dw >> 2;      // which half of the K block
    const int rl = 32 * q + lane;  // weight row within the tile = TMEM lane
    const int nthreads = kDecWarpsG * 32;
    tm::build_table(table, tstage, tw, (int)threadIdx.x - 64, nthreads);
    const uint32_t l4 = (uint32_t)(lane << 2) * 0x01010101u;
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + kTmA + (uint32_t)(part * 32);
    // The weights' MMA scale factors are all 2^0 (UE8M0 127); the first afull
    // arrival orders these stores before the first MMA.
    if (part == 0)
      tc::st_x4(tmem + ((uint32_t)(32 * q) << 16) + kTmSfa, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
    // This thread's bytes in a chunk-major record.
    const uint32_t off_q0 = tm::kRecQs + (uint32_t)(2 * part) * 2048u + (uint32_t)rl * 16u;
    const uint32_t off_q1 = off_q0 + 2048u;
    const uint32_t off_sg = tm::kRecSigns + (uint32_t)part * 2048u + (uint32_t)rl * 16u;
    const uint32_t off_qh = tm::kRecQh + (uint32_t)part * 512u + (uint32_t)rl * 4u;
    int it = 0;
    for (int t = 0; t < my_tiles; ++t) {
      for (int kb = 0; kb < nb; ++kb, ++it) {
        const int s = it % SW, r = it % kARingG;
        // A slot r is free once the MMAs of unit it - kARingG have completed.
        bool ok = tm::warp_wait(kWfull + 8 * s, (it / SW) & 1, kSiteGemvFull);
        if (ok && it >= kARingG) ok = tm::warp_wait(kAempty + 8 * r, ((it / kARingG) & 1) ^ 1, kSiteGemvEmpty);
        if (!ok) return;
        const uint8_t* st = st0 + (size_t)s * tm::kRecordBytes;
        const uint4 a = *reinterpret_cast<const uint4*>(st + off_q0);
        const uint4 c = *reinterpret_cast<const uint4*>(st + off_q1);
        const uint4 gs = *reinterpret_cast<const uint4*>(st + off_sg);
        const uint32_t hw = *reinterpret_cast<const uint32_t*>(st + off_qh);
        const uint32_t qw[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
        const uint32_t sw[4] = {gs.x, gs.y, gs.z, gs.w};
        if (part == 0) {
          // The row's d and scale nibbles for the epilogue (it forms d * (1 + 2*nibble)).
          reinterpret_cast<uint2*>(aux0 + (size_t)r * kAuxG)[rl] =
              make_uint2(*reinterpret_cast<const uint16_t*>(st + tm::kRecD + rl * 2),
                         *reinterpret_cast<const uint32_t*>(st + tm::kRecScales + rl * 4));
        }
        uint32_t v[32];
#pragma unroll
        for (int g = 0; g < 4; ++g)
          tm::decode_group_packed(table, qw[2 * g], qw[2 * g + 1], hw, 2u * (uint32_t)g, sw[g], l4, v + 8 * g);
        tc::st_cols<32>(tq + (uint32_t)(r * 64), v);
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(kAfull + 8 * r);
          mbar_arrive(kWempty + 8 * s);
        }
        __syncwarp();
      }
    }
    return;
  }

  // ------------------------------------------------------------------ epilogue
  {
    const int e = warp - kEpiWarp0G;
    const int q = warp & 3;        // TMEM lane quadrant of this warp
    const int h = e >> 2;          // tokens h*64 .. h*64+63 of the tile
    const int rl = 32 * q + lane;  // weight row within the tile = TMEM lane
    const uint32_t tq0 = tmem + ((uint32_t)(32 * q) << 16) + kTmD + (uint32_t)(h * 64);
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.f;
    pdl_wait();  // the output may still be in use by the previous kernel
    pdl_launch_dependents();
    int it = 0, gi = 0;
    bool ok = true;
    for (int t = 0; ok && t < my_tiles; ++t) {
      const int ti = (int)blockIdx.x + t * (int)gridDim.x;
      const int rt = ti / p.tok_tiles, tt = ti % p.tok_tiles;
      for (int kb = 0; kb < nb; ++kb, ++it) {
        const int r = it % kARingG;
        if (!tm::warp_wait(kAfull + 8 * r, (it / kARingG) & 1, kSiteGemvFull)) {
          ok = false;
          break;
        }
        // Read once per unit, before any D buffer of the unit is released: the
        // decoders refill slot r only after this unit's MMAs have completed.
        const uint2 dsc = reinterpret_cast<const uint2*>(aux0 + (size_t)r * kAuxG)[rl];
        const float dv = __half2float(__ushort_as_half((unsigned short)dsc.x));
        const float dneg = -8388608.0f * dv;
        // 2*nibble+1 of group g is byte g/2 of tb[g&1]; float(2^23 + t)*d - 2^23*d = t*d exactly.
        const uint32_t tb0 = lop3_and_or(dsc.y << 1, 0x1E1E1E1Eu, 0x01010101u);
        const uint32_t tb1 = lop3_and_or(dsc.y >> 3, 0x1E1E1E1Eu, 0x01010101u);
#pragma unroll 1
        for (int g = 0; g < 8; ++g, ++gi) {
          const int ds = gi & 1;
          if (!tm::warp_wait(kMdone + 8 * ds, (gi >> 1) & 1, kSiteGemvFull)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const float w = fmaf(__uint_as_float(prmt((g & 1) ? tb1 : tb0, 0x4B000000u, 0x7650u | (uint32_t)(g >> 1))),
                               dv, dneg);
          const uint32_t tq = tq0 + (uint32_t)(ds * kTokG);
#pragma unroll
          for (int c0 = 0; c0 < 64; c0 += 16) {
            const uint32_t off[2] = {(uint32_t)c0, (uint32_t)c0 + 8u};
            float cv[2][8];
            tc::ld_x8_multi<2>(tq, off, cv);
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
              for (int i = 0; i < 8; i += 2)
                fma2(acc[c0 + 8 * j + i], acc[c0 + 8 * j + i + 1], cv[j][i], cv[j][i + 1], w, w);
          }
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(kEfree + 8 * ds);
          __syncwarp();
        }
        if (!ok) break;
      }
      if (!ok) break;
      const int row = rt * kRowsG + rl, tok0 = tt * kTokG + h * 64;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        store_out_g(p, row, tok0 + i, acc[i]);
        acc[i] = 0.f;
      }
    }
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(kEdone);
  }
}

// Writes activation scales xs [m][nq*4] (UE8M0, one per 32 K) as the tensor
// core's scale-factor atoms: for token tile tt (128 tokens) and K quad q (4
// groups), 512 bytes whose row n0 (16 bytes) holds, at byte 4*n1 + j, the
// scale of token tt*128 + 32*n1 + n0 and group 4q + j. Tokens past m get 0.
__global__ void iq3s_xs_atoms_kernel(const uint8_t* __restrict__ xs, int64_t ldxs, int m, int nq, int tok_tiles,
                                     uint8_t* __restrict__ atoms) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one 16-byte row
  const int64_t total = (int64_t)tok_tiles * nq * 32;
  if (idx >= total) return;
  const int n0 = (int)(idx & 31);
  const int64_t tq = idx >> 5;
  const int q = (int)(tq % nq), tt = (int)(tq / nq);
  uint32_t w[4];
#pragma unroll
  for (int n1 = 0; n1 < 4; ++n1) {
    const int tok = tt * 128 + 32 * n1 + n0;
    uint32_t v = 0;
    if (tok < m) {
      const uint8_t* src = xs + (int64_t)tok * ldxs + 4 * q;
      v = (uint32_t)src[0] | ((uint32_t)src[1] << 8) | ((uint32_t)src[2] << 16) | ((uint32_t)src[3] << 24);
    }
    w[n1] = v;
  }
  reinterpret_cast<uint4*>(atoms)[idx] = make_uint4(w[0], w[1], w[2], w[3]);
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------
uint32_t gemm_tm_smem_bytes(int wstages) { return gemm_smem(wstages); }
int gemm_tm_max_wstages() { return kMaxWStagesG; }
int gemm_tm_tile_tokens() { return kTokG; }

cudaError_t launch_xs_atoms(const uint8_t* xs, int64_t ldxs, int m, int n_blocks, uint8_t* atoms,
                            cudaStream_t stream) {
  const int tok_tiles = (m + kTokG - 1) / kTokG, nq = 2 * n_blocks;
  const int64_t rows = (int64_t)tok_tiles * nq * 32;
  const int threads = 256;
  iq3s_xs_atoms_kernel<<<(unsigned)((rows + threads - 1) / threads), threads, 0, stream>>>(xs, ldxs, m, nq, tok_tiles,
                                                                                         atoms);
  return cudaGetLastError();
}

cudaError_t launch_gemm_tm(const GemmTmParams& p, const GemmTmMaps& maps, int grid, cudaStream_t stream) {
  const uint32_t smem = gemm_smem(p.wstages);
  const void* kern = (const void*)iq3s_gemm_tm_kernel;
  cudaError_t e = ensure_smem_attribute(kern, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(kThreadsG), smem, stream, p, maps);
}

}  // namespace mambo
