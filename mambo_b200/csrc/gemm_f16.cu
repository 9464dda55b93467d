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

namespace mambo {

namespace {

constexpr int kRowsH = 128, kTokH = 128;
constexpr int kDecWarpsH = 8, kEpiWarpsH = 8;
constexpr int kARingH = 2;   // decoded A blocks in TMEM (128 columns each)
constexpr int kDRingH = 2;   // D buffers (128 columns each)
constexpr int kXStagesH = 3;  // FP16 activation half-blocks (128 tokens x 128 K)
constexpr int kMaxWStagesH = 6;
constexpr uint32_t kXHalfBytes = kTokH * 128u * 2u;  // 32 KB
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
constexpr int kEpiWarp0H = 2 + kDecWarpsH, kXWarpH = kEpiWarp0H + kEpiWarpsH;

__host__ __device__ constexpr uint32_t align_up_h(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline uint32_t gemm_f16_smem(int wstages) {
  return tm::kTableBytes + 1024 + align_up_h((uint32_t)wstages * tm::kRecordBytes, 1024) + kXStagesH * kXHalfBytes +
         kAuxRingH * kAuxH + tm::kTableStageBytes + kBarBytesH;
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

__global__ void __launch_bounds__(kThreadsH, 1)
    iq3s_gemm_f16_kernel(const __grid_constant__ GemmF16Params p, const __grid_constant__ GemmF16Maps maps) {
  // B half-block (128 tokens x 128 K): two [128 tokens][128 bytes] boxes in
  // the 128-byte-swizzled K-major layout (8-row atoms 1024 bytes apart); an
  // MMA's 16 K (32 bytes) start 32 bytes further into the row.
  constexpr uint32_t kBoxBytes = kTokH * 128u;
  constexpr uint32_t kIdesc = tc::idesc_f16_f32(kRowsH, kTokH);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* table = smem_raw;
  uint8_t* st0 = smem_raw + tm::kTableBytes + ((1024u - ((smem_u32(smem_raw) + tm::kTableBytes) & 1023u)) & 1023u);
  const int SW = p.wstages;
  uint8_t* x0 = st0 + align_up_h((uint32_t)SW * tm::kRecordBytes, 1024);
  uint8_t* aux0 = x0 + (size_t)kXStagesH * kXHalfBytes;
  uint32_t* tstage = reinterpret_cast<uint32_t*>(aux0 + kAuxRingH * kAuxH);
  uint64_t* bars = reinterpret_cast<uint64_t*>(aux0 + kAuxRingH * kAuxH + tm::kTableStageBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxWStagesH + 2 * kXStagesH + 2 * kARingH +
                                                    2 * kDRingH + 1 + kAuxRingH);
  const uint32_t bar0 = smem_u32(bars);
  // Barriers as in the FP8 GEMM, with activation slots per half block.
  const uint32_t kWfull = bar0, kWempty = bar0 + 8 * kMaxWStagesH;
  const uint32_t kXfull = bar0 + 16 * kMaxWStagesH, kXempty = kXfull + 8 * kXStagesH;
  const uint32_t kAfull = kXempty + 8 * kXStagesH, kAempty = kAfull + 8 * kARingH;
  const uint32_t kMdone = kAempty + 8 * kARingH, kEfree = kMdone + 8 * kDRingH;
  const uint32_t kEdone = kEfree + 8 * kDRingH, kDfull = kEdone + 8;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.n_blocks, n_tiles = p.row_tiles * p.tok_tiles;
  const int my_tiles = (int)blockIdx.x < n_tiles ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

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
    for (int x = 0; x < kXStagesH; ++x) {
      mbar_init(kXfull + 8 * x, 1);
      mbar_init(kXempty + 8 * x, 1);
    }
    for (int r = 0; r < kARingH; ++r) {
      mbar_init(kAfull + 8 * r, kDecWarpsH);
      mbar_init(kAempty + 8 * r, 1);
    }
    for (int d = 0; d < kDRingH; ++d) {
      mbar_init(kMdone + 8 * d, 1);
      mbar_init(kEfree + 8 * d, kEpiWarpsH);
    }
    mbar_init(kEdone, kEpiWarpsH);
    for (int a = 0; a < kAuxRingH; ++a) mbar_init(kDfull + 8 * a, 4);
    fence_barrier_init();
  }
  if (warp == 1) {
    tc::alloc(smem_u32(tmem_slot), kTmColsH);
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
      uint32_t ph = 0;
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
  if (warp == kXWarpH) {
    if (lane == 0) {
      tma_prefetch_desc(&maps.x16);
      const uint64_t keep = l2_policy_evict_last();
      pdl_wait();
      int hj = 0, x = 0;
      uint32_t ph = 0;
      for (int t = 0; t < my_tiles; ++t) {
        const int tt = ((int)blockIdx.x + t * (int)gridDim.x) % p.tok_tiles;
        for (int kb = 0; kb < nb; ++kb) {
          for (int h = 0; h < 2; ++h, ++hj) {
            if (hj >= kXStagesH && !mbar_wait_bounded(kXempty + 8 * x, ph ^ 1, kSiteGemvEmpty)) return;
            const uint32_t full = kXfull + 8 * x;
            mbar_arrive_expect_tx(full, kXHalfBytes);
            const uint32_t dst = smem_u32(x0 + (size_t)x * kXHalfBytes);
            tma_load_2d(dst, &maps.x16, kb * 256 + h * 128, tt * kTokH, full, keep);
            tma_load_2d(dst + kBoxBytes, &maps.x16, kb * 256 + h * 128 + 64, tt * kTokH, full, keep);
            if (++x == kXStagesH) {
              x = 0;
              ph ^= 1;
            }
          }
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------------ MMA
  if (warp == 1) {
    int it = 0, hj = 0;
    bool ok = true;
    for (int t = 0; ok && t < my_tiles; ++t) {
      for (int kb = 0; ok && kb < nb; ++kb, ++it) {
        const int r = it % kARingH, db = it & 1;
        ok = tm::warp_wait(kAfull + 8 * r, (it / kARingH) & 1, kSiteGemvFull);
        // The D buffer is free once the epilogue has read block it - 2.
        if (ok && it >= kDRingH) ok = tm::warp_wait(kEfree + 8 * db, ((it >> 1) & 1) ^ 1, kSiteGemvEmpty);
        if (!ok) break;
        const uint32_t dcol = tmem + kTmD + (uint32_t)(db * kTokH), acol = tmem + kTmA + 128u * (uint32_t)r;
#pragma unroll 1
        for (int h = 0; h < 2; ++h, ++hj) {
          const int x = hj % kXStagesH;
          if (!tm::warp_wait(kXfull + 8 * x, (hj / kXStagesH) & 1, kSiteGemvFull)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint64_t bdesc = tc::smem_desc_sw128(smem_u32(x0 + (size_t)x * kXHalfBytes), 1024u);
          if (tm::elect_one()) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              tc::mma_f16_ts(dcol, acol + (uint32_t)((8 * h + j) * 8),
                             bdesc + (uint64_t)(((j >> 2) * kBoxBytes + (j & 3) * 32u) >> 4), kIdesc, (h | j) != 0);
            tc::commit(kXempty + 8 * x);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (tm::elect_one()) {
          tc::commit(kAempty + 8 * r);
          tc::commit(kMdone + 8 * db);
        }
        __syncwarp();
      }
    }
    mbar_wait_bounded(kEdone, 0, kSiteGemvFull);
    __syncwarp();
    tc::fence_after_sync();
    tc::dealloc(tmem, kTmColsH);
    return;
  }

  // ------------------------------------------------------------------ decoders
  if (warp < kEpiWarp0H) {
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
    for (int t = 0; t < my_tiles; ++t) {
      for (int kb = 0; kb < nb; ++kb, ++it) {
        const int r = it % kARingH;
        bool ok = tm::warp_wait(kWfull + 8 * s, sph, kSiteGemvFull);
        if (ok && it >= kARingH) ok = tm::warp_wait(kAempty + 8 * r, ((it / kARingH) & 1) ^ 1, kSiteGemvEmpty);
        if (!ok) return;
        const uint8_t* st = st0 + (size_t)s * tm::kRecordBytes;
        const uint4 a = *reinterpret_cast<const uint4*>(st + off_q0);
        const uint4 c = *reinterpret_cast<const uint4*>(st + off_q1);
        const uint4 gs = *reinterpret_cast<const uint4*>(st + off_sg);
        const uint32_t hw = *reinterpret_cast<const uint32_t*>(st + off_qh);
        const uint32_t scw = *reinterpret_cast<const uint32_t*>(st + tm::kRecScales + rl * 4);
        const uint32_t qw[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
        const uint32_t sw[4] = {gs.x, gs.y, gs.z, gs.w};
        if (part == 0) {
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
          // (1 + 2*nibble) of group 4*part + g as an FP16 pair (an odd integer <= 31: exact).
          const uint32_t mult = 1u + 2u * ((scw >> (4 * (4 * part + g))) & 0xFu);
          const uint32_t mh = (uint32_t)__half_as_ushort(__uint2half_rn(mult));
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
          mbar_arrive(kAfull + 8 * r);
          mbar_arrive(kWempty + 8 * s);
        }
        __syncwarp();
        if (++s == SW) {
          s = 0;
          sph ^= 1;
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------------ epilogue
  {
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
      const int ti = (int)blockIdx.x + t * (int)gridDim.x;
      const int rt = ti / p.tok_tiles, tt = ti % p.tok_tiles;
      for (int kb = 0; kb < nb; ++kb, ++it) {
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
        if (lane == 0) mbar_arrive(kEfree + 8 * db);
        __syncwarp();
      }
      if (!ok) break;
      const int row = rt * kRowsH + rl, tok0 = tt * kTokH + h * 64;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const int tok = tok0 + i;
        const float sc = tok < p.m ? __ldg(p.tok_scale + tok) : 0.f;
        store_out_h(p, row, tok, acc[i] * sc);
        acc[i] = 0.f;
      }
    }
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(kEdone);
  }
}

// One CTA per token row: e_max over the row's UE8M0 scales, then every E4M3
// value times 2^(e_g - e_max) rounded to FP16; tok_scale = 2^(e_max - 127).
// A scale code 0xFF (NaN) makes its group NaN.
__global__ void iq3s_x16_kernel(const uint8_t* __restrict__ xq, int64_t ldxq, const uint8_t* __restrict__ xs,
                                int64_t ldxs, int64_t k, uint16_t* __restrict__ x16, int64_t ld,
                                float* __restrict__ tok_scale) {
  const int64_t t = blockIdx.x;
  const int64_t groups = k / 32;
  const uint8_t* srow = xs + t * ldxs;
  int emax = 0;
  for (int64_t g = threadIdx.x; g < groups; g += blockDim.x) {
    const int e = srow[g];
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
  emax = wmax[0];
  if (threadIdx.x == 0) tok_scale[t] = e8m0_to_float((uint32_t)emax);
  const uint8_t* qrow = xq + t * ldxq;
  uint16_t* orow = x16 + t * ld;
  for (int64_t c = threadIdx.x; c < k / 8; c += blockDim.x) {  // 8 values per step
    const int e = srow[c / 4];
    const uint2 raw = *reinterpret_cast<const uint2*>(qrow + c * 8);
    const float f = e == 0xFF ? __uint_as_float(0x7FC00000u) : ldexpf(1.0f, e - emax);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t two = ((i < 2 ? raw.x : raw.y) >> (16 * (i & 1))) & 0xFFFFu;
      const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)two, __NV_E4M3);
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&hr));
      const __half2 o = __floats2half2_rn(v.x * f, v.y * f);
      w[i] = *reinterpret_cast<const uint32_t*>(&o);
    }
    *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------
uint32_t gemm_f16_smem_bytes(int wstages) { return gemm_f16_smem(wstages); }
int gemm_f16_max_wstages() { return kMaxWStagesH; }

cudaError_t launch_x16(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int m, int64_t k,
                       uint16_t* x16, int64_t ld, float* tok_scale, cudaStream_t stream) {
  iq3s_x16_kernel<<<(unsigned)m, 256, 0, stream>>>(xq, ldxq, xs, ldxs, k, x16, ld, tok_scale);
  return cudaGetLastError();
}

cudaError_t launch_gemm_f16(const GemmF16Params& p, const GemmF16Maps& maps, int grid, cudaStream_t stream) {
  const uint32_t smem = gemm_f16_smem(p.wstages);
  const void* kern = (const void*)iq3s_gemm_f16_kernel;
  cudaError_t e = ensure_smem_attribute(kern, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(kThreadsH), smem, stream, p, maps);
}

}  // namespace mambo
