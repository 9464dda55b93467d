// IQ3_S x MXFP8 weight-streaming linear for decode-sized M (sm_100a).
//
// Computes out[M,N] = sum_k x[m,k] * w[n,k] where x = E4M3 * 2^e (UE8M0 per
// 32 along K) and w = d * (1 + 2*nibble) * (+-grid magnitude), with the
// reference's exact decomposition (src/python/mambo/kernels/iq3_s_fp8.py:279-333):
// each 32-weight group's E4M3 x E4M3 product is summed by the tensor core in
// FP32 and then scaled by the group's FP32 weight scale d*(1+2*nibble) and the
// activation's power-of-two scale.
//
// Design (B200):
//  * Work unit = (row tile of R = 16*warps weight rows, one 256-wide K block).
//    Persistent CTAs (one per SM) walk a contiguous range of units
//    (row-tile major, stream-K), so every SM streams the same number of
//    weight bytes whatever the shape.
//  * One producer thread stages units through a ring of shared-memory stages
//    with asynchronous copies completing on an mbarrier: five TMA tensor copies
//    for the weight fields (qs/signs swizzled so consumer reads are bank-conflict
//    free) and one bulk copy per token row of the MXFP8 activation slice.
//  * The activation scales are converted to float once per CTA.
//  * Consumer warps decode straight into mma.sync m16n8k32 A fragments: the
//    fragment puts 4 consecutive K of one row in one register, which is exactly
//    one IQ3_S code (4 weights sharing one codebook entry). The codebook lives
//    in shared memory replicated per lane (entry e of lane l in bank l), so the
//    512-entry gather is conflict free. Weights are the 16-row A operand
//    (swap-AB); tokens are the n8 B operand.
//  * Row tiles split between CTAs write FP32 partials to a workspace; per
//    (row tile, warp) an acq_rel atomic counter elects the last warp to finish,
//    which sums the partials in CTA order (deterministic) and resets the counter.
#include "kernels.cuh"

namespace mambo {

constexpr int kTableBytes = 512 * 32 * 4;  // lane-private codebook
constexpr int kMaxStages = 12;
constexpr int kXRowBytes = 272;  // 256-byte activation rows padded to 272 (conflict-free B-fragment reads)

__host__ __device__ constexpr uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

struct StageLayout {
  uint32_t qs, signs, qh, d, scales, x, bytes;
};

__host__ __device__ inline StageLayout gemv_stage_layout(int rows, int nt) {
  StageLayout L{};
  uint32_t off = 0;
  L.qs = off;
  off = align_up(off + rows * 64, 1024);
  L.signs = off;
  off = align_up(off + rows * 32, 128);
  L.qh = off;
  off = align_up(off + rows * 8, 128);
  L.d = off;
  off = align_up(off + rows * 2, 128);
  L.scales = off;
  off = align_up(off + rows * 4, 128);
  L.x = off;
  off = align_up(off + 8 * nt * kXRowBytes, 1024);
  L.bytes = off;
  return L;
}

__host__ __device__ inline uint32_t gemv_xs_bytes(int n_blocks, int nt) {
  return align_up((uint32_t)n_blocks * 8u * 8u * nt * 4u, 128);
}

__host__ __device__ inline uint32_t gemv_smem_bytes(int rows, int nt, int stages, int n_blocks) {
  return 1024 + kTableBytes + stages * gemv_stage_layout(rows, nt).bytes + gemv_xs_bytes(n_blocks, nt) + 2048 +
         2 * kMaxStages * 8;
}

__device__ __forceinline__ int unit_begin(int cta, int grid, int units) {
  return (int)(((int64_t)cta * units) / grid);
}

__device__ __forceinline__ int cta_of_unit(int u, int grid, int units) {
  return (int)((((int64_t)u + 1) * grid - 1) / units);
}

// Swizzled byte offsets of the weight fields inside a stage (match TMA SWIZZLE_64B / SWIZZLE_32B).
__device__ __forceinline__ uint32_t qs_off(uint32_t row, uint32_t byte) {
  return row * 64 + ((((byte >> 4) ^ (row >> 1)) & 3) << 4) + (byte & 15);
}
__device__ __forceinline__ uint32_t signs_off(uint32_t row, uint32_t byte) {
  return row * 32 + ((((byte >> 4) ^ (row >> 2)) & 1) << 4) + (byte & 15);
}

__device__ __forceinline__ void mma_e4m3(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  // Pure register-to-register: not volatile, so the compiler may overlap groups.
  asm("mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

template <int NT, bool kTma>
__device__ void gemv_producer(const GemvParams& p, const GemvMaps* maps, uint8_t* stage0, const StageLayout& L,
                              uint32_t full0, uint32_t empty0, int u0, int u1) {
  const int lane = threadIdx.x & 31;
  const int rows = p.warps * 16;
  const int tokens = 8 * NT;
  const bool async_all = kTma && p.x_bulk;
  if (async_all && lane != 0) return;  // one thread drives every copy
  uint64_t policy = 0;
  if constexpr (kTma) {
    if (lane == 0) {
      policy = l2_policy_evict_first();
      tma_prefetch_desc(&maps->qs);
      tma_prefetch_desc(&maps->signs);
      tma_prefetch_desc(&maps->qh);
      tma_prefetch_desc(&maps->d);
      tma_prefetch_desc(&maps->scales);
    }
  }
  // Weights do not depend on the previous kernel: with the fully asynchronous
  // path, issue the first stages' weight copies before waiting for it.
  int issued_weights = 0;
  if (async_all) {
    issued_weights = min(p.stages, u1 - u0);
    for (int it = 0; it < issued_weights; ++it) {
      const int u = u0 + it;
      const uint32_t full = full0 + 8 * it;
      uint8_t* st = stage0 + (size_t)it * L.bytes;
      const int rt = u / p.n_blocks, kb = u % p.n_blocks;
      const int n0 = rt * rows;
      mbar_expect_tx(full, (uint32_t)rows * 110u + (uint32_t)p.m * 256u);
      tma_load_3d(smem_u32(st + L.qs), &maps->qs, 0, n0, kb, full, policy);
      tma_load_3d(smem_u32(st + L.signs), &maps->signs, 0, n0, kb, full, policy);
      tma_load_2d(smem_u32(st + L.qh), &maps->qh, n0, kb, full, policy);
      tma_load_2d(smem_u32(st + L.d), &maps->d, n0, kb, full, policy);
      tma_load_2d(smem_u32(st + L.scales), &maps->scales, n0, kb, full, policy);
    }
  }
  pdl_wait();  // activations come from the previous kernel
  for (int u = u0, it = 0; u < u1; ++u, ++it) {
    const int s = it % p.stages;
    const uint32_t full = full0 + 8 * s, empty = empty0 + 8 * s;
    if (it < issued_weights) {
      uint8_t* st = stage0 + (size_t)s * L.bytes;
      const int kb = u % p.n_blocks;
      for (int tok = 0; tok < p.m; ++tok)
        bulk_load(smem_u32(st + L.x + tok * kXRowBytes), p.xq + (int64_t)tok * p.ldxq + (int64_t)kb * 256, 256, full);
      mbar_arrive(full);
      continue;
    }
    if (it >= p.stages) {
      if (!mbar_wait_bounded(empty, ((it / p.stages) & 1) ^ 1, kSiteGemvEmpty)) return;
    }
    uint8_t* st = stage0 + (size_t)s * L.bytes;
    const int rt = u / p.n_blocks, kb = u % p.n_blocks;
    const int n0 = rt * rows;
    if constexpr (kTma) {
      if (lane == 0) {
        mbar_expect_tx(full, (uint32_t)rows * 110u + (p.x_bulk ? (uint32_t)p.m * 256u : 0u));
        tma_load_3d(smem_u32(st + L.qs), &maps->qs, 0, n0, kb, full, policy);
        tma_load_3d(smem_u32(st + L.signs), &maps->signs, 0, n0, kb, full, policy);
        tma_load_2d(smem_u32(st + L.qh), &maps->qh, n0, kb, full, policy);
        tma_load_2d(smem_u32(st + L.d), &maps->d, n0, kb, full, policy);
        tma_load_2d(smem_u32(st + L.scales), &maps->scales, n0, kb, full, policy);
        if (p.x_bulk) {
          for (int tok = 0; tok < p.m; ++tok)
            bulk_load(smem_u32(st + L.x + tok * kXRowBytes), p.xq + (int64_t)tok * p.ldxq + (int64_t)kb * 256, 256,
                      full);
        }
      }
    } else {
      // Plain loads into the same swizzled layout (any N, any field alignment).
      for (int i = lane; i < rows * 4; i += 32) {  // qs: 4 x 16 bytes per row
        const int r = i >> 2, c = i & 3;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (n0 + r < p.n_rows)
          v = *reinterpret_cast<const uint4*>(p.qs + ((int64_t)kb * p.n_rows + n0 + r) * 64 + c * 16);
        *reinterpret_cast<uint4*>(st + L.qs + qs_off(r, c * 16)) = v;
      }
      for (int i = lane; i < rows * 2; i += 32) {  // signs: 2 x 16 bytes per row
        const int r = i >> 1, c = i & 1;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (n0 + r < p.n_rows)
          v = *reinterpret_cast<const uint4*>(p.signs + ((int64_t)kb * p.n_rows + n0 + r) * 32 + c * 16);
        *reinterpret_cast<uint4*>(st + L.signs + signs_off(r, c * 16)) = v;
      }
      for (int r = lane; r < rows; r += 32) {
        uint2 qh = make_uint2(0, 0);
        uint32_t dd = 0, sc = 0;
        if (n0 + r < p.n_rows) {
          const int64_t blk = (int64_t)kb * p.n_rows + n0 + r;
          qh = *reinterpret_cast<const uint2*>(p.qh + blk * 8);
          dd = *reinterpret_cast<const uint16_t*>(p.d + blk * 2);
          sc = *reinterpret_cast<const uint32_t*>(p.scales + blk * 4);
        }
        *reinterpret_cast<uint2*>(st + L.qh + r * 8) = qh;
        *reinterpret_cast<uint16_t*>(st + L.d + r * 2) = (uint16_t)dd;
        *reinterpret_cast<uint32_t*>(st + L.scales + r * 4) = sc;
      }
    }
    if (!async_all) {
      // Activation slice [tokens x 256] E4M3 with plain loads (rows >= M are zero).
      for (int i = lane; i < tokens * 16; i += 32) {
        const int tok = i >> 4, c = i & 15;
        uint32_t w[4] = {0, 0, 0, 0};
        if (tok < p.m) {
          const uint8_t* src = p.xq + (int64_t)tok * p.ldxq + (int64_t)kb * 256 + c * 16;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            w[j] = (uint32_t)src[4 * j] | ((uint32_t)src[4 * j + 1] << 8) | ((uint32_t)src[4 * j + 2] << 16) |
                   ((uint32_t)src[4 * j + 3] << 24);
        }
        *reinterpret_cast<uint4*>(st + L.x + tok * kXRowBytes + c * 16) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    mbar_arrive(full);
  }
}

__device__ __forceinline__ void store_out(const GemvParams& p, int row, int tok, float v) {
  if (row < p.n_rows && tok < p.m) {
    if (p.out_bf16) {
      reinterpret_cast<__nv_bfloat16*>(p.out)[(int64_t)tok * p.ldo + row] = __float2bfloat16_rn(v);
    } else {
      reinterpret_cast<float*>(p.out)[(int64_t)tok * p.ldo + row] = v;
    }
  }
}

template <int NT>
__device__ void gemv_consumer(const GemvParams& p, const uint8_t* table, const float* xsf, uint8_t* stage0,
                              const StageLayout& L, uint32_t full0, uint32_t empty0, int u0, int u1) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int rows = p.warps * 16;
  const int tokens = 8 * NT;
  const uint32_t lane4x = (uint32_t)(lane << 2) * 0x01010101u;
  const int rl0 = warp * 16 + gid;  // local rows rl0 and rl0 + 8
  // Swizzled in-stage offsets of this thread's qs halfwords and sign bytes,
  // per row h and group g (the group's low bits ride in a constant).
  uint32_t qs_o[2][4], sg_o[2][2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t r = rl0 + 8 * h;
#pragma unroll
    for (int j = 0; j < 4; ++j) qs_o[h][j] = L.qs + qs_off(r, 16 * j + 2 * tig);
#pragma unroll
    for (int j = 0; j < 2; ++j) sg_o[h][j] = L.signs + signs_off(r, 16 * j + tig);
  }

  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;

  int seg_begin = u0;
  for (int u = u0, it = 0; u < u1; ++u, ++it) {
    const int s = it % p.stages;
    const uint32_t full = full0 + 8 * s, empty = empty0 + 8 * s;
    if (!mbar_wait_bounded(full, (it / p.stages) & 1, kSiteGemvFull)) return;
    const uint8_t* st = stage0 + (size_t)s * L.bytes;
    const int rt = u / p.n_blocks, kb = u % p.n_blocks;

    // Per-row metadata of this block for rows rl0 (h=0) and rl0+8 (h=1).
    uint32_t e0[2][2], e1[2][2];  // [h][groups 0-3 / 4-7]: byte g = (high code bit << 7) | lane<<2
    uint32_t tb[2][2];            // [h][even/odd groups]: byte j = 2*nibble+1
    float dv[2], dneg[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = rl0 + 8 * h;
      const uint2 qh = *reinterpret_cast<const uint2*>(st + L.qh + r * 8);
      const uint64_t q64 = ((uint64_t)qh.y << 32 | qh.x) >> (2 * tig);
      const uint32_t lo = (uint32_t)q64, hi = (uint32_t)(q64 >> 32);
      e0[h][0] = lop3_and_or(lo << 7, 0x80808080u, lane4x);
      e0[h][1] = lop3_and_or(hi << 7, 0x80808080u, lane4x);
      e1[h][0] = lop3_and_or(lo << 6, 0x80808080u, lane4x);
      e1[h][1] = lop3_and_or(hi << 6, 0x80808080u, lane4x);
      const uint32_t sc = *reinterpret_cast<const uint32_t*>(st + L.scales + r * 4);
      tb[h][0] = lop3_and_or(sc << 1, 0x1E1E1E1Eu, 0x01010101u);
      tb[h][1] = lop3_and_or(sc >> 3, 0x1E1E1E1Eu, 0x01010101u);
      const uint16_t dh = *reinterpret_cast<const uint16_t*>(st + L.d + r * 2);
      dv[h] = __half2float(__ushort_as_half(dh));
      dneg[h] = -8388608.0f * dv[h];
    }
    const float* xs_kb = xsf + (size_t)kb * 8 * tokens;
    const uint8_t* xrow = st + L.x + gid * kXRowBytes + 8 * tig;

#pragma unroll
    for (int g = 0; g < 8; ++g) {
      uint32_t a[4];  // a0: row gid code 2tig, a1: row gid+8 code 2tig, a2/a3: code 2tig+1
      float w[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t q = *reinterpret_cast<const uint16_t*>(st + qs_o[h][g >> 1] + 8 * (g & 1));
        const uint32_t sb = st[sg_o[h][g >> 2] + 4 * (g & 3)];
        const uint32_t sel = (uint32_t)(4 + (g & 3)) | 0x2200u;
        const uint32_t addr0 = prmt(q, e0[h][g >> 2], sel);
        const uint32_t addr1 = prmt(q, e1[h][g >> 2], sel | 0x10u);
        const uint32_t m0 = *reinterpret_cast<const uint32_t*>(table + addr0);
        const uint32_t m1 = *reinterpret_cast<const uint32_t*>(table + addr1);
        a[h] = lop3_and_or((sb & 0xFu) * 0x10204080u, 0x80808080u, m0);
        a[2 + h] = lop3_and_or((sb >> 4) * 0x10204080u, 0x80808080u, m1);
        // weight scale d*(2*nibble+1): float(2^23 + t) * d - 2^23 * d, exact
        const uint32_t tf = prmt(tb[h][g & 1], 0x4B000000u, 0x7650u | (uint32_t)(g >> 1));
        w[h] = fmaf(__uint_as_float(tf), dv[h], dneg[h]);
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const uint2 b = *reinterpret_cast<const uint2*>(xrow + t * 8 * kXRowBytes + 32 * g);
        float c[4];
        mma_e4m3(c, a[0], a[1], a[2], a[3], b.x, b.y);
        const float2 xsc = *reinterpret_cast<const float2*>(xs_kb + g * tokens + 8 * t + 2 * tig);
        // acc += (c * activation scale) * weight scale; c * 2^e is exact.
        mul2(c[0], c[1], c[0], c[1], xsc.x, xsc.y);
        mul2(c[2], c[3], c[2], c[3], xsc.x, xsc.y);
        fma2(acc[t][0], acc[t][1], c[0], c[1], w[0], w[0]);
        fma2(acc[t][2], acc[t][3], c[2], c[3], w[1], w[1]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty);

    // End of a row-tile segment?
    const bool seg_end = (kb == p.n_blocks - 1) || (u == u1 - 1);
    if (!seg_end) continue;
    const int seg_first_kb = seg_begin % p.n_blocks;
    const bool full_tile = (seg_first_kb == 0) && (kb == p.n_blocks - 1);
    const int row0 = rt * rows;
    if (full_tile) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int tok = 8 * t + 2 * tig;
        store_out(p, row0 + rl0, tok, acc[t][0]);
        store_out(p, row0 + rl0, tok + 1, acc[t][1]);
        store_out(p, row0 + rl0 + 8, tok, acc[t][2]);
        store_out(p, row0 + rl0 + 8, tok + 1, acc[t][3]);
      }
    } else {
      // Partial: slot 0 = first row tile of this CTA, slot 1 = its last one.
      // Each warp owns its 16 rows: it publishes its partial, and the warp
      // that arrives last on the (row tile, warp) counter sums all partials
      // of those rows in CTA order. No CTA-wide barrier is involved.
      const int cta = blockIdx.x, grid = gridDim.x;
      const int slot = (rt == u0 / p.n_blocks) ? 0 : 1;
      float* part = p.partials + ((size_t)(cta * 2 + slot) * rows) * tokens;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int tok = 8 * t + 2 * tig;
        __stcg(reinterpret_cast<float2*>(part + (size_t)rl0 * tokens + tok), make_float2(acc[t][0], acc[t][1]));
        __stcg(reinterpret_cast<float2*>(part + (size_t)(rl0 + 8) * tokens + tok), make_float2(acc[t][2], acc[t][3]));
      }
      __syncwarp();
      const int c_first = cta_of_unit(rt * p.n_blocks, grid, p.total_units);
      const int c_last = cta_of_unit(rt * p.n_blocks + p.n_blocks - 1, grid, p.total_units);
      int last = 0;
      if (lane == 0) {
        int* counter = p.counters + (size_t)rt * p.warps + warp;
        const int old = atomic_add_acq_rel_gpu(counter, 1);
        last = (old == c_last - c_first);
        if (last) *counter = 0;  // leave the counter zeroed for the next launch
      }
      last = __shfl_sync(0xFFFFFFFFu, last, 0);
      if (last) {
        float sum[NT][4];
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int i = 0; i < 4; ++i) sum[t][i] = 0.f;
        // Issue the loads of up to kBatch segments before summing them (in CTA order).
        constexpr int kBatch = 8 / NT;
        for (int c0 = c_first; c0 <= c_last; c0 += kBatch) {
          float2 v[kBatch][NT][2];
#pragma unroll
          for (int j = 0; j < kBatch; ++j) {
            const int c = c0 + j;
            if (c <= c_last) {
              const int c_slot = (rt == unit_begin(c, grid, p.total_units) / p.n_blocks) ? 0 : 1;
              const float* src = p.partials + ((size_t)(c * 2 + c_slot) * rows) * tokens;
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                const int tok = 8 * t + 2 * tig;
                v[j][t][0] = __ldcg(reinterpret_cast<const float2*>(src + (size_t)rl0 * tokens + tok));
                v[j][t][1] = __ldcg(reinterpret_cast<const float2*>(src + (size_t)(rl0 + 8) * tokens + tok));
              }
            }
          }
#pragma unroll
          for (int j = 0; j < kBatch; ++j) {
            if (c0 + j <= c_last) {
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                sum[t][0] += v[j][t][0].x;
                sum[t][1] += v[j][t][0].y;
                sum[t][2] += v[j][t][1].x;
                sum[t][3] += v[j][t][1].y;
              }
            }
          }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const int tok = 8 * t + 2 * tig;
          store_out(p, row0 + rl0, tok, sum[t][0]);
          store_out(p, row0 + rl0, tok + 1, sum[t][1]);
          store_out(p, row0 + rl0 + 8, tok, sum[t][2]);
          store_out(p, row0 + rl0 + 8, tok + 1, sum[t][3]);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;
    seg_begin = u + 1;
  }
}

template <int NT, int kWarps, bool kTma>
__global__ void __launch_bounds__((kWarps + 1) * 32, 1)
    iq3s_gemv_kernel(const __grid_constant__ GemvParams p, const __grid_constant__ GemvMaps maps) {
  extern __shared__ uint8_t smem_raw[];
  // An offset from smem_raw (not integer arithmetic) keeps the pointer in the shared address space.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* table = smem;
  const int rows = p.warps * 16;
  const int tokens = 8 * NT;
  const StageLayout L = gemv_stage_layout(rows, NT);
  uint8_t* stage0 = smem + kTableBytes;
  float* xsf = reinterpret_cast<float*>(stage0 + (size_t)p.stages * L.bytes);
  uint32_t* tstage = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(xsf) + gemv_xs_bytes(p.n_blocks, NT));
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(tstage) + 2048);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kMaxStages);
  const bool async_all = kTma && p.x_bulk;

  const int u0 = unit_begin(blockIdx.x, gridDim.x, p.total_units);
  const int u1 = unit_begin(blockIdx.x + 1, gridDim.x, p.total_units);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(full0 + 8 * s, async_all ? 1 : 32);  // producer arrivals (+ copy bytes)
      mbar_init(empty0 + 8 * s, p.warps);            // one arrival per consumer warp
    }
    fence_barrier_init();
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  if (warp == p.warps) {
    gemv_producer<NT, kTma>(p, &maps, stage0, L, full0, empty0, u0, u1);
    return;
  }
  // Consumers: codebook, activation scales and zero padding rows, then the main loop.
  const int nthreads = p.warps * 32;
  // Stage the 2 KB codebook (two independent loads per thread at most), then
  // expand it to the lane-private copy: entry (q | h<<8) of lane l at byte
  // (q<<8)|(h<<7)|(l<<2). Consecutive threads write consecutive banks.
  for (int i = threadIdx.x; i < 512; i += nthreads) tstage[i] = __ldg(p.table + i);
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
  for (int i = threadIdx.x; i < 512 * 32; i += nthreads) {
    const uint32_t code = i >> 5, l = i & 31;
    const uint32_t off = ((code & 0xFFu) << 8) | ((code >> 8) << 7) | (l << 2);
    *reinterpret_cast<uint32_t*>(table + off) = tstage[code];
  }
  if (async_all) {
    // The bulk copies fill rows < M only: zero the padding rows of every stage once.
    const int per_stage = (tokens - p.m) * (kXRowBytes / 16);
    for (int i = threadIdx.x; i < p.stages * per_stage; i += nthreads) {
      const int s = i / per_stage, j = i - s * per_stage;
      const int tok = p.m + j / (kXRowBytes / 16), c = j % (kXRowBytes / 16);
      *reinterpret_cast<uint4*>(stage0 + (size_t)s * L.bytes + L.x + tok * kXRowBytes + c * 16) =
          make_uint4(0, 0, 0, 0);
    }
  }
  pdl_wait();  // the activation scales come from the previous kernel
  // Activation scales as floats, laid out [k group][token]; padding tokens get 1.
  for (int i = threadIdx.x; i < p.n_blocks * 8 * tokens; i += nthreads) {
    const int kg = i / tokens, tok = i - kg * tokens;
    xsf[i] = tok < p.m ? e8m0_to_float(p.xs[(int64_t)tok * p.ldxs + kg]) : 1.0f;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
  pdl_launch_dependents();
  gemv_consumer<NT>(p, table, xsf, stage0, L, full0, empty0, u0, u1);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
  }
  return fn;
}

static bool encode(EncodeTiledFn fn, CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base,
                   const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                   CUtensorMapSwizzle swz) {
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, type, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Builds the five weight tensor maps. Returns false when the TMA path does not apply.
bool make_gemv_maps(const GemvParams& p, GemvMaps* maps) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  const uint64_t N = (uint64_t)p.n_rows, B = (uint64_t)p.n_blocks;
  const uint32_t R = (uint32_t)p.warps * 16;
  if (N % 8 != 0 || R > 256) return false;
  const uintptr_t ptrs[5] = {(uintptr_t)p.qs, (uintptr_t)p.signs, (uintptr_t)p.qh, (uintptr_t)p.d,
                             (uintptr_t)p.scales};
  for (uintptr_t a : ptrs)
    if (a % 16) return false;
  {
    cuuint64_t dims[3] = {64, N, B};
    cuuint64_t str[2] = {64, N * 64};
    cuuint32_t box[3] = {64, R, 1};
    if (!encode(fn, &maps->qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, p.qs, dims, str, box, CU_TENSOR_MAP_SWIZZLE_64B))
      return false;
  }
  {
    cuuint64_t dims[3] = {32, N, B};
    cuuint64_t str[2] = {32, N * 32};
    cuuint32_t box[3] = {32, R, 1};
    if (!encode(fn, &maps->signs, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, p.signs, dims, str, box,
                CU_TENSOR_MAP_SWIZZLE_32B))
      return false;
  }
  {
    cuuint64_t dims[2] = {N, B};
    cuuint64_t str[1] = {N * 8};
    cuuint32_t box[2] = {R, 1};
    if (!encode(fn, &maps->qh, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, p.qh, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return false;
  }
  {
    cuuint64_t dims[2] = {N, B};
    cuuint64_t str[1] = {N * 2};
    cuuint32_t box[2] = {R, 1};
    if (!encode(fn, &maps->d, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, p.d, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return false;
  }
  {
    cuuint64_t dims[2] = {N, B};
    cuuint64_t str[1] = {N * 4};
    cuuint32_t box[2] = {R, 1};
    if (!encode(fn, &maps->scales, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, p.scales, dims, str, box,
                CU_TENSOR_MAP_SWIZZLE_NONE))
      return false;
  }
  return true;
}

bool make_gemv_x_map(const uint8_t* xq, int64_t ldxq, int m, int n_blocks, int box_tokens, CUtensorMap* map) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn || (uintptr_t)xq % 16 || ldxq % 16 || m < 1 || box_tokens > 256) return false;
  // [K/16 chunks][m tokens][16 bytes]: each box lands as 16-byte K chunks of
  // box_tokens rows, the K-major no-swizzle layout of the MMA's B operand.
  cuuint64_t dims[3] = {16, (cuuint64_t)m, (cuuint64_t)n_blocks * 16};
  cuuint64_t str[2] = {(cuuint64_t)ldxq, 16};
  cuuint32_t box[3] = {16, (cuuint32_t)box_tokens, 16};
  return encode(fn, map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, xq, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

bool make_gemv_xb_map(const uint16_t* x, int64_t ldx, int m, int64_t k, int box_tokens, CUtensorMap* map) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn || (uintptr_t)x % 16 || ldx % 8 || m < 1 || k % 256 || box_tokens > 256) return false;
  // [m tokens][K bf16]: a box of box_tokens rows x 256 values (one K block,
  // 512 bytes a row, unswizzled); rows past m are zero-filled.
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
  cuuint64_t str[1] = {(cuuint64_t)(ldx * 2)};
  cuuint32_t box[2] = {256, (cuuint32_t)box_tokens};
  return encode(fn, map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, x, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

bool make_gemm_out_map(void* out, int64_t ldo, int n_rows, int m, CUtensorMap* map) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn || (uintptr_t)out % 16 || ldo % 8 || n_rows < 1 || m < 1) return false;
  // [m tokens][n_rows bf16]: a 128-row x 128-token tile, rows contiguous (unswizzled).
  cuuint64_t dims[2] = {(cuuint64_t)n_rows, (cuuint64_t)m};
  cuuint64_t str[1] = {(cuuint64_t)(ldo * 2)};
  cuuint32_t box[2] = {128, 128};
  return encode(fn, map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, out, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

bool make_gemm_x8_map(const uint8_t* xq, int64_t ldxq, int m, int64_t k, CUtensorMap* map) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn || (uintptr_t)xq % 16 || ldxq % 16 || m < 1 || k % 128) return false;
  // [m tokens][K bytes]: a box of 128 tokens x 128 bytes lands as eight
  // 1024-byte atoms of the K-major 128-byte-swizzled UMMA layout.
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
  cuuint64_t str[1] = {(cuuint64_t)ldxq};
  cuuint32_t box[2] = {128, 128};
  return encode(fn, map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, xq, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

bool make_gemm_x16_map(const uint16_t* x16, int64_t ld, int m, int64_t k, int box_tokens, CUtensorMap* map) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn || (uintptr_t)x16 % 16 || (ld * 2) % 16 || m < 1 || k % 128 || box_tokens % 8 || box_tokens > 256)
    return false;
  // [m tokens][K halves]: a box of box_tokens tokens x 64 halves (128 bytes)
  // lands as 1024-byte atoms (8 tokens each) of the K-major 128-byte-swizzled
  // UMMA layout.
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
  cuuint64_t str[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_tokens};
  return encode(fn, map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, x16, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

bool make_gemv_xs_map(const uint8_t* xs, int64_t ldxs, int m, int n_blocks, int box_tokens, CUtensorMap* map) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn || (uintptr_t)xs % 16 || ldxs % 16 || m < 1 || box_tokens > 256) return false;
  // Boxes of 16 scale bytes (the groups of two K blocks) x box_tokens rows.
  cuuint64_t dims[2] = {(cuuint64_t)n_blocks * 8, (cuuint64_t)m};
  cuuint64_t str[1] = {(cuuint64_t)ldxs};
  cuuint32_t box[2] = {16, (cuuint32_t)box_tokens};
  return encode(fn, map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, xs, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

uint32_t gemv_smem_bytes_host(int rows, int nt, int stages, int n_blocks) {
  return gemv_smem_bytes(rows, nt, stages, n_blocks);
}

template <int NT, int kWarps, bool kTma>
static cudaError_t launch_gemv_t(const GemvParams& p, const GemvMaps& maps, int grid, cudaStream_t stream) {
  const uint32_t smem = gemv_smem_bytes(p.warps * 16, NT, p.stages, p.n_blocks);
  auto kern = iq3s_gemv_kernel<NT, kWarps, kTma>;
  cudaError_t e = ensure_smem_attribute((const void*)kern, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl((const void*)kern, dim3(grid), dim3((p.warps + 1) * 32), smem, stream, p, maps);
}

template <int NT, bool kTma>
static cudaError_t launch_gemv_w(const GemvParams& p, const GemvMaps& maps, int grid, cudaStream_t stream) {
  switch (p.warps) {
    case 4: return launch_gemv_t<NT, 4, kTma>(p, maps, grid, stream);
    case 8: return launch_gemv_t<NT, 8, kTma>(p, maps, grid, stream);
    case 12: return launch_gemv_t<NT, 12, kTma>(p, maps, grid, stream);
    default: return launch_gemv_t<NT, 16, kTma>(p, maps, grid, stream);
  }
}

cudaError_t launch_gemv(const GemvParams& p, int nt, bool use_tma, const GemvMaps& maps, int grid,
                        cudaStream_t stream) {
  if (use_tma) {
    switch (nt) {
      case 1: return launch_gemv_w<1, true>(p, maps, grid, stream);
      case 2: return launch_gemv_w<2, true>(p, maps, grid, stream);
      default: return launch_gemv_w<4, true>(p, maps, grid, stream);
    }
  }
  switch (nt) {
    case 1: return launch_gemv_w<1, false>(p, maps, grid, stream);
    case 2: return launch_gemv_w<2, false>(p, maps, grid, stream);
    default: return launch_gemv_w<4, false>(p, maps, grid, stream);
  }
}

}  // namespace mambo
