// IQ3_S x MXFP8 weight-streaming linear on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Same arithmetic as the reference (src/python/mambo/kernels/iq3_s_fp8.py:279-333):
// per 32-weight group g, P_g = sum_k E4M3(x) * E4M3(+-grid) is summed by the
// tensor core in FP32, then out += P_g * 2^e(x, g) * d * (1 + 2*nibble_g) in FP32.
//
// Design (one persistent CTA per SM, 22 warps):
//  * warp 0, producer: per work unit (128 weight rows x one 256-wide K block,
//    stream-K order) five TMA tensor copies of the IQ3_S fields plus one bulk
//    copy of the packed activation slice, into a ring of stages.
//  * warps 2-17, decoders: expand each 4-weight IQ3_S code through a lane-private
//    shared-memory codebook into E4M3 bytes, written as the K-major no-swizzle
//    UMMA operand (8 x 16-byte core matrices); copy the activation tile and
//    scales and the rows' d and scale nibbles.
//  * warp 1, MMA: one thread issues 8 tcgen05.mma (M=128 rows, N=16/32 tokens,
//    K=32 each, one per group) into TMEM, double buffered, and commits them to
//    an mbarrier; the warp owns the TMEM allocation.
//  * warps 18-21, epilogue: each thread owns one weight row (its TMEM lane),
//    loads the group partials with tcgen05.ld, scales them by the activation
//    scale and d * (1 + 2*nibble) and accumulates them in FP32 registers; finished rows go to the output, or to a split-K workspace
//    whose last contributor (acq_rel counter) sums them in CTA order.
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace mambo {

namespace {

constexpr int kRows = 128;  // weight rows per unit = MMA M
constexpr int kTableBytes = 512 * 32 * 4;
constexpr int kEpiWarps = 4;
__host__ __device__ constexpr int tc_threads(int dec_warps) { return (2 + dec_warps + kEpiWarps) * 32; }
constexpr int kMaxStagesTc = 6;

__host__ __device__ constexpr uint32_t align_up_tc(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }
__host__ __device__ constexpr int nmma_for(int nt) { return nt * 8 < 16 ? 16 : nt * 8; }

// Raw stage: weight fields at the offsets of the TMA boxes, then the packed activation slice.
struct TcLayout {
  uint32_t qs, signs, qh, d, scales, xpack, raw_bytes;  // within a raw stage
  uint32_t a, bt, xs, w, slot_bytes;                    // within an operand slot
  uint32_t pack_bytes;
};

__host__ __device__ inline TcLayout tc_layout(int nt) {
  TcLayout L{};
  const int nm = nmma_for(nt);
  L.qs = 0;
  L.signs = kRows * 64;             // 8192, 1024-aligned (SWIZZLE_32B destination)
  L.qh = L.signs + kRows * 32;      // 12288
  L.d = L.qh + kRows * 8;           // 13312
  L.scales = L.d + kRows * 2;       // 13568
  L.xpack = align_up_tc(L.scales + kRows * 4, 128);
  L.pack_bytes = nm * 256 + 8 * nm * 4;
  L.raw_bytes = align_up_tc(L.xpack + L.pack_bytes, 1024);
  L.a = 0;
  L.bt = kRows * 256;               // 32 KB decoded E4M3 tile
  L.xs = L.bt + nm * 256;
  L.w = L.xs + 8 * nm * 4;  // per row: d (fp16 bits) in the low half, scale nibbles word next: 2 x u32
  L.slot_bytes = align_up_tc(L.w + 2 * kRows * 4, 1024);
  return L;
}

__host__ __device__ inline uint32_t tc_smem_bytes(int nt, int stages) {
  const TcLayout L = tc_layout(nt);
  return 1024 + kTableBytes + stages * L.raw_bytes + 2 * L.slot_bytes + 256;
}

__device__ __forceinline__ uint32_t qs_off_tc(uint32_t row, uint32_t byte) {
  return row * 64 + ((((byte >> 4) ^ (row >> 1)) & 3) << 4) + (byte & 15);
}
__device__ __forceinline__ uint32_t signs_off_tc(uint32_t row, uint32_t byte) {
  return row * 32 + ((((byte >> 4) ^ (row >> 2)) & 1) << 4) + (byte & 15);
}

__device__ __forceinline__ int unit_begin_tc(int cta, int grid, int units) {
  return (int)(((int64_t)cta * units) / grid);
}
__device__ __forceinline__ int cta_of_unit_tc(int u, int grid, int units) {
  return (int)((((int64_t)u + 1) * grid - 1) / units);
}

__device__ __forceinline__ void store_out_tc(const GemvTcParams& p, int row, int tok, float v) {
  if (row < p.n_rows && tok < p.m) {
    if (p.out_bf16) {
      reinterpret_cast<__nv_bfloat16*>(p.out)[(int64_t)tok * p.ldo + row] = __float2bfloat16_rn(v);
    } else {
      reinterpret_cast<float*>(p.out)[(int64_t)tok * p.ldo + row] = v;
    }
  }
}

struct TcBarriers {
  uint32_t full, empty, afull, mdone, tfree, edone;  // base addresses (8 bytes per entry)
};

}  // namespace

// --------------------------------------------------------------------------
// Activation packing: MXFP8 [M,K] (+ scales) -> per K block, the UMMA B tile
// (NMMA tokens x 256 bytes, 8-token x 16-byte core matrices: token group tg,
// K chunk kc at tg*2048 + kc*128 + (tok%8)*16) followed by the scales as
// floats [8 groups][NMMA tokens]. Tokens >= M are zero with scale 1.
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(256) pack_activations_kernel(const PackParams p) {
  pdl_wait();  // inputs come from, and the buffer may still be read by, the previous kernel
  pdl_launch_dependents();
  const int nm = p.nmma;
  const int chunks = nm * 16;                 // 16-byte chunks of one B tile
  const int per_block = chunks + 8 * nm;      // + one float per (group, token)
  const int64_t total = (int64_t)p.n_blocks * per_block;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int kb = (int)(i / per_block);
    const int j = (int)(i - (int64_t)kb * per_block);
    uint8_t* dst = p.pack + (size_t)kb * p.pack_bytes;
    if (j < chunks) {
      const int tok = j >> 4, kc = j & 15;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (tok < p.m) {
        const uint8_t* src = p.xq + (int64_t)tok * p.ldxq + (int64_t)kb * 256 + kc * 16;
        if (p.x_vec) {
          v = __ldg(reinterpret_cast<const uint4*>(src));
        } else {
          uint32_t w[4];
#pragma unroll
          for (int b = 0; b < 4; ++b)
            w[b] = (uint32_t)src[4 * b] | ((uint32_t)src[4 * b + 1] << 8) | ((uint32_t)src[4 * b + 2] << 16) |
                   ((uint32_t)src[4 * b + 3] << 24);
          v = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      *reinterpret_cast<uint4*>(dst + (tok >> 3) * 2048 + kc * 128 + (tok & 7) * 16) = v;
    } else {
      const int e = j - chunks, g = e / nm, tok = e - g * nm;
      const float v = tok < p.m ? e8m0_to_float(p.xs[(int64_t)tok * p.ldxs + (int64_t)kb * 8 + g]) : 1.0f;
      reinterpret_cast<float*>(dst + nm * 256)[g * nm + tok] = v;
    }
  }
}

cudaError_t launch_pack_activations(const PackParams& p, int num_sms, cudaStream_t stream) {
  const int64_t total = (int64_t)p.n_blocks * (p.nmma * 16 + 8 * p.nmma);
  int64_t blocks = (total + 255) / 256;
  if (blocks > (int64_t)num_sms * 4) blocks = (int64_t)num_sms * 4;
  if (blocks < 1) blocks = 1;
  return launch_pdl((const void*)pack_activations_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, p);
}

// --------------------------------------------------------------------------
// The linear kernel
// --------------------------------------------------------------------------
template <int NT, int kDecWarps>
__global__ void __launch_bounds__(tc_threads(kDecWarps), 1)
    iq3s_gemv_tc_kernel(const __grid_constant__ GemvTcParams p, const __grid_constant__ GemvMaps maps) {
  constexpr int NM = nmma_for(NT);       // MMA N (tokens, padded to 16)
  constexpr int TOK = 8 * NT;            // tokens the epilogue keeps
  constexpr uint32_t kIdesc = tc::idesc_e4m3_f32(kRows, NM);
  constexpr uint32_t kTmemCols = 2 * 8 * NM;  // two buffers of 8 group partials

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const TcLayout L = tc_layout(NT);
  // The codebook sits at the start of dynamic shared memory (a link-time
  // constant address, so lookups need no base register); the TMA stages
  // after it are aligned to 1024 bytes at run time.
  uint8_t* table = smem_raw;
  uint8_t* raw0 = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw + kTableBytes) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* slot0 = raw0 + (size_t)p.stages * L.raw_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(slot0 + 2 * L.slot_bytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStagesTc + 7);
  const uint32_t bar0 = smem_u32(bars);
  const TcBarriers B{bar0, bar0 + 8 * kMaxStagesTc, bar0 + 16 * kMaxStagesTc, bar0 + 16 * kMaxStagesTc + 16,
                     bar0 + 16 * kMaxStagesTc + 32, bar0 + 16 * kMaxStagesTc + 48};

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u0 = unit_begin_tc(blockIdx.x, gridDim.x, p.total_units);
  const int u1 = unit_begin_tc(blockIdx.x + 1, gridDim.x, p.total_units);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(B.full + 8 * s, 1);
      mbar_init(B.empty + 8 * s, kDecWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(B.afull + 8 * b, kDecWarps);
      mbar_init(B.mdone + 8 * b, 1);
      mbar_init(B.tfree + 8 * b, kEpiWarps);
    }
    mbar_init(B.edone, kEpiWarps);
    fence_barrier_init();
  }
  if (warp == 1) {
    tc::alloc(smem_u32(tmem_slot), kTmemCols);
    tc::relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  // ------------------------------------------------------------------ producer
  if (warp == 0) {
    if (lane != 0) return;
    const uint64_t policy = l2_policy_evict_first();
    tma_prefetch_desc(&maps.qs);
    tma_prefetch_desc(&maps.signs);
    tma_prefetch_desc(&maps.qh);
    tma_prefetch_desc(&maps.d);
    tma_prefetch_desc(&maps.scales);
    const int pre = min(p.stages, u1 - u0);
    auto issue_weights = [&](int it, int u) {
      const uint32_t full = B.full + 8 * (it % p.stages);
      uint8_t* st = raw0 + (size_t)(it % p.stages) * L.raw_bytes;
      const int n0 = (u / p.n_blocks) * kRows, kb = u % p.n_blocks;
      mbar_expect_tx(full, (uint32_t)kRows * 110u + L.pack_bytes);
      tma_load_3d(smem_u32(st + L.qs), &maps.qs, 0, n0, kb, full, policy);
      tma_load_3d(smem_u32(st + L.signs), &maps.signs, 0, n0, kb, full, policy);
      tma_load_2d(smem_u32(st + L.qh), &maps.qh, n0, kb, full, policy);
      tma_load_2d(smem_u32(st + L.d), &maps.d, n0, kb, full, policy);
      tma_load_2d(smem_u32(st + L.scales), &maps.scales, n0, kb, full, policy);
    };
    auto issue_pack = [&](int it, int u) {
      const uint32_t full = B.full + 8 * (it % p.stages);
      uint8_t* st = raw0 + (size_t)(it % p.stages) * L.raw_bytes;
      bulk_load(smem_u32(st + L.xpack), p.xpack + (size_t)(u % p.n_blocks) * L.pack_bytes, L.pack_bytes, full);
      mbar_arrive(full);
    };
    // Weights are independent of the previous kernel: start streaming them first.
    for (int it = 0; it < pre; ++it) issue_weights(it, u0 + it);
    pdl_wait();
    for (int it = 0; it < pre; ++it) issue_pack(it, u0 + it);
    for (int it = pre, u = u0 + pre; u < u1; ++u, ++it) {
      if (!mbar_wait_bounded(B.empty + 8 * (it % p.stages), ((it / p.stages) & 1) ^ 1, kSiteGemvEmpty)) return;
      issue_weights(it, u);
      issue_pack(it, u);
    }
    return;
  }

  // ------------------------------------------------------------------ MMA
  if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      for (int it = 0, u = u0; u < u1 && ok; ++u, ++it) {
        const int b = it & 1;
        ok = mbar_wait_bounded(B.afull + 8 * b, (it >> 1) & 1, kSiteGemvFull);
        if (ok && it >= 2) ok = mbar_wait_bounded(B.tfree + 8 * b, ((it >> 1) & 1) ^ 1, kSiteGemvEmpty);
        if (!ok) break;
        tc::fence_after_sync();
        const uint32_t sa = smem_u32(slot0 + (size_t)b * L.slot_bytes + L.a);
        const uint32_t sb = smem_u32(slot0 + (size_t)b * L.slot_bytes + L.bt);
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          const uint64_t da = tc::smem_desc(sa + 256 * g, 128, 2048);
          const uint64_t db = tc::smem_desc(sb + 256 * g, 128, 2048);
          tc::mma_e4m3(tmem + (uint32_t)(b * 8 * NM + g * NM), da, db, kIdesc, 0);
        }
        tc::commit(B.mdone + 8 * b);
      }
      // Free the TMEM once every epilogue warp has read its last partials.
      mbar_wait_bounded(B.edone, 0, kSiteGemvFull);
      tc::fence_after_sync();
    }
    __syncwarp();
    tc::dealloc(tmem, kTmemCols);
    return;
  }

  // ------------------------------------------------------------------ decoders
  if (warp < 2 + kDecWarps) {
    const int dw = warp - 2;
    const int nthreads = kDecWarps * 32;
    const int tid = threadIdx.x - 64;
    // Codebook: stage 2 KB, then expand to the lane-private copy (entry
    // (q | h<<8) of lane l at byte (q<<8)|(h<<7)|(l<<2)); consecutive threads
    // write consecutive banks.
    uint32_t* tstage = reinterpret_cast<uint32_t*>(slot0);  // operand slot 0, free until the first unit
    for (int i = tid; i < 512; i += nthreads) tstage[i] = __ldg(p.table + i);
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
    for (int i = tid; i < 512 * 32; i += nthreads) {
      const uint32_t code = i >> 5, l = i & 31;
      *reinterpret_cast<uint32_t*>(table + (((code & 0xFFu) << 8) | ((code >> 8) << 7) | (l << 2))) = tstage[code];
    }
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");

    const uint32_t lane2x = (uint32_t)(lane << 2) * 0x0101u;
    // Task i of this thread: weight row row0 + kRowStep*i, 16-weight chunk kc
    // (kDecWarps is a multiple of 4, so the chunk and every swizzle term are
    // the same for all i and each address is a base plus a constant).
    constexpr int kTasks = (64 + kDecWarps - 1) / kDecWarps;
    constexpr int kRowStep = 8 * (kDecWarps / 4);
    static_assert(kDecWarps % 4 == 0, "decoder warps must be a multiple of 4");
    const int row0 = (dw >> 2) * 8 + (lane & 7);
    const int kc = (dw & 3) * 4 + (lane >> 3);
    const uint32_t qs_base = L.qs + qs_off_tc(row0, 4 * kc);
    const uint32_t qh_base = L.qh + row0 * 8 + (kc >> 1);
    const uint32_t sg_base = L.signs + signs_off_tc(row0, 2 * kc);
    const uint32_t a_base = L.a + (row0 >> 3) * 2048 + kc * 128 + (row0 & 7) * 16;
    const uint32_t h_shift = (kc & 1) * 4;
    for (int it = 0, u = u0; u < u1; ++u, ++it) {
      const int s = it % p.stages, b = it & 1;
      if (!mbar_wait_bounded(B.full + 8 * s, (it / p.stages) & 1, kSiteGemvFull)) return;
      if (it >= 2 && !mbar_wait_bounded(B.tfree + 8 * b, ((it >> 1) & 1) ^ 1, kSiteGemvEmpty)) return;
      const uint8_t* st = raw0 + (size_t)s * L.raw_bytes;
      uint8_t* slot = slot0 + (size_t)b * L.slot_bytes;
      // All gathers first, then all stores: a store may alias later loads as
      // far as the compiler knows, so interleaving them would serialize the tasks.
      uint4 v[kTasks];
#pragma unroll
      for (int i = 0; i < kTasks; ++i) {
        if (64 % kDecWarps != 0 && dw + kDecWarps * i >= 64) break;
        const uint32_t q = *reinterpret_cast<const uint32_t*>(st + qs_base + i * (kRowStep * 64));
        const uint32_t hn = (st[qh_base + i * (kRowStep * 8)] >> h_shift) & 0xFu;
        const uint32_t sg = *reinterpret_cast<const uint16_t*>(st + sg_base + i * (kRowStep * 32));
        const uint32_t e0 = lop3_and_or((hn & 3u) * 0x4080u, 0x8080u, lane2x);
        const uint32_t e1 = lop3_and_or((hn >> 2) * 0x4080u, 0x8080u, lane2x);
        const uint32_t m0 = *reinterpret_cast<const uint32_t*>(table + prmt(q, e0, 0x6604u));
        const uint32_t m1 = *reinterpret_cast<const uint32_t*>(table + prmt(q, e0, 0x6615u));
        const uint32_t m2 = *reinterpret_cast<const uint32_t*>(table + prmt(q, e1, 0x6624u));
        const uint32_t m3 = *reinterpret_cast<const uint32_t*>(table + prmt(q, e1, 0x6635u));
        v[i].x = lop3_and_or((sg & 0xFu) * 0x10204080u, 0x80808080u, m0);
        v[i].y = lop3_and_or(((sg >> 4) & 0xFu) * 0x10204080u, 0x80808080u, m1);
        v[i].z = lop3_and_or(((sg >> 8) & 0xFu) * 0x10204080u, 0x80808080u, m2);
        v[i].w = lop3_and_or((sg >> 12) * 0x10204080u, 0x80808080u, m3);
      }
#pragma unroll
      for (int i = 0; i < kTasks; ++i) {
        if (64 % kDecWarps != 0 && dw + kDecWarps * i >= 64) break;
        *reinterpret_cast<uint4*>(slot + a_base + i * (kRowStep / 8) * 2048) = v[i];
      }
      // Rows' d and scale nibbles for the epilogue (it forms d * (1 + 2*nibble)).
      for (int r = tid; r < kRows; r += nthreads) {
        reinterpret_cast<uint2*>(slot + L.w)[r] =
            make_uint2(*reinterpret_cast<const uint16_t*>(st + L.d + r * 2),
                       *reinterpret_cast<const uint32_t*>(st + L.scales + r * 4));
      }
      // Activation tile and scales to the operand slot.
      for (int c = tid; c < (int)(L.pack_bytes / 16); c += nthreads)
        reinterpret_cast<uint4*>(slot + L.bt)[c] = reinterpret_cast<const uint4*>(st + L.xpack)[c];
      fence_proxy_async_shared();  // generic-proxy writes -> tensor-core reads
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(B.afull + 8 * b);
        mbar_arrive(B.empty + 8 * s);
      }
    }
    return;
  }

  // ------------------------------------------------------------------ epilogue
  {
    const int q = warp & 3;               // TMEM lane quadrant of this warp
    const int rl = 32 * q + lane;         // local weight row = TMEM lane
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
    float acc[TOK];
#pragma unroll
    for (int t = 0; t < TOK; ++t) acc[t] = 0.f;
    pdl_wait();  // the workspace and output may still be in use by the previous kernel
    pdl_launch_dependents();
    int seg_begin = u0;
    bool ok = true;
    for (int it = 0, u = u0; u < u1; ++u, ++it) {
      const int b = it & 1;
      if (!mbar_wait_bounded(B.mdone + 8 * b, (it >> 1) & 1, kSiteGemvFull)) { ok = false; break; }
      tc::fence_after_sync();
      const uint8_t* slot = slot0 + (size_t)b * L.slot_bytes;
      const float* xs = reinterpret_cast<const float*>(slot + L.xs);
      const uint2 dsc = reinterpret_cast<const uint2*>(slot + L.w)[rl];
      const float dv = __half2float(__ushort_as_half((unsigned short)dsc.x));
      const float dneg = -8388608.0f * dv;
      // 2*nibble+1 of group g is byte g/2 of tb[g&1]; float(2^23 + t)*d - 2^23*d = t*d exactly.
      const uint32_t tb0 = lop3_and_or(dsc.y << 1, 0x1E1E1E1Eu, 0x01010101u);
      const uint32_t tb1 = lop3_and_or(dsc.y >> 3, 0x1E1E1E1Eu, 0x01010101u);
#pragma unroll
      for (int g = 0; g < 8; g += 2) {
#pragma unroll
        for (int tb = 0; tb < TOK; tb += 8) {
          float c0[8], c1[8];
          tc::ld_x8_pair(tq + (uint32_t)(b * 8 * NM + g * NM + tb), tq + (uint32_t)(b * 8 * NM + (g + 1) * NM + tb),
                         c0, c1);
          const float w0 = fmaf(__uint_as_float(prmt(tb0, 0x4B000000u, 0x7650u | (uint32_t)(g >> 1))), dv, dneg);
          const float w1 = fmaf(__uint_as_float(prmt(tb1, 0x4B000000u, 0x7650u | (uint32_t)(g >> 1))), dv, dneg);
#pragma unroll
          for (int t = 0; t < 8; t += 2) {
            float p0, p1;
            mul2(p0, p1, c0[t], c0[t + 1], xs[g * NM + tb + t], xs[g * NM + tb + t + 1]);
            fma2(acc[tb + t], acc[tb + t + 1], p0, p1, w0, w0);
            mul2(p0, p1, c1[t], c1[t + 1], xs[(g + 1) * NM + tb + t], xs[(g + 1) * NM + tb + t + 1]);
            fma2(acc[tb + t], acc[tb + t + 1], p0, p1, w1, w1);
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(B.tfree + 8 * b);

      const int kb = u % p.n_blocks, rt = u / p.n_blocks;
      if (!(kb == p.n_blocks - 1 || u == u1 - 1)) continue;
      const bool full_tile = (seg_begin % p.n_blocks == 0) && (kb == p.n_blocks - 1);
      const int row = rt * kRows + rl;
      if (full_tile) {
#pragma unroll
        for (int t = 0; t < TOK; ++t) store_out_tc(p, row, t, acc[t]);
      } else {
        const int cta = blockIdx.x, grid = gridDim.x;
        const int slot_id = (rt == u0 / p.n_blocks) ? 0 : 1;
        float* part = p.partials + ((size_t)(cta * 2 + slot_id) * kRows + rl) * TOK;
#pragma unroll
        for (int t = 0; t < TOK; t += 4) __stcg(reinterpret_cast<float4*>(part + t), make_float4(acc[t], acc[t + 1], acc[t + 2], acc[t + 3]));
        __syncwarp();
        const int c_first = cta_of_unit_tc(rt * p.n_blocks, grid, p.total_units);
        const int c_last = cta_of_unit_tc(rt * p.n_blocks + p.n_blocks - 1, grid, p.total_units);
        int last = 0;
        if (lane == 0) {
          int* counter = p.counters + (size_t)rt * kEpiWarps + q;
          last = (atomic_add_acq_rel_gpu(counter, 1) == c_last - c_first);
          if (last) *counter = 0;  // leave the counter zeroed for the next launch
        }
        last = __shfl_sync(0xFFFFFFFFu, last, 0);
        if (last) {
          float sum[TOK];
#pragma unroll
          for (int t = 0; t < TOK; ++t) sum[t] = 0.f;
          constexpr int kBatch = TOK <= 8 ? 4 : (TOK <= 16 ? 2 : 1);
          for (int c0 = c_first; c0 <= c_last; c0 += kBatch) {
            float4 v[kBatch][TOK / 4];
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
              const int c = c0 + j;
              if (c <= c_last) {
                const int cs = (rt == unit_begin_tc(c, grid, p.total_units) / p.n_blocks) ? 0 : 1;
                const float* src = p.partials + ((size_t)(c * 2 + cs) * kRows + rl) * TOK;
#pragma unroll
                for (int t = 0; t < TOK / 4; ++t) v[j][t] = __ldcg(reinterpret_cast<const float4*>(src) + t);
              }
            }
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
              if (c0 + j <= c_last) {
#pragma unroll
                for (int t = 0; t < TOK / 4; ++t) {
                  sum[4 * t] += v[j][t].x;
                  sum[4 * t + 1] += v[j][t].y;
                  sum[4 * t + 2] += v[j][t].z;
                  sum[4 * t + 3] += v[j][t].w;
                }
              }
            }
          }
#pragma unroll
          for (int t = 0; t < TOK; ++t) store_out_tc(p, row, t, sum[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < TOK; ++t) acc[t] = 0.f;
      seg_begin = u + 1;
    }
    (void)ok;
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(B.edone);
  }
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------
uint32_t gemv_tc_smem_bytes(int nt, int stages) { return tc_smem_bytes(nt, stages); }
uint32_t gemv_tc_pack_bytes(int nt) { return tc_layout(nt).pack_bytes; }
int gemv_tc_max_stages() { return kMaxStagesTc; }

template <int NT, int kDecWarps>
static cudaError_t launch_gemv_tc_t(const GemvTcParams& p, const GemvMaps& maps, int grid, cudaStream_t stream) {
  const uint32_t smem = tc_smem_bytes(NT, p.stages);
  const void* kern = (const void*)iq3s_gemv_tc_kernel<NT, kDecWarps>;
  cudaError_t e = ensure_smem_attribute(kern, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(tc_threads(kDecWarps)), smem, stream, p, maps);
}

template <int NT>
static cudaError_t launch_gemv_tc_n(const GemvTcParams& p, int dec_warps, const GemvMaps& maps, int grid,
                                    cudaStream_t stream) {
  switch (dec_warps) {
    case 8: return launch_gemv_tc_t<NT, 8>(p, maps, grid, stream);
    case 12: return launch_gemv_tc_t<NT, 12>(p, maps, grid, stream);
    default: return launch_gemv_tc_t<NT, 16>(p, maps, grid, stream);
  }
}

cudaError_t launch_gemv_tc(const GemvTcParams& p, int nt, int dec_warps, const GemvMaps& maps, int grid,
                           cudaStream_t stream) {
  switch (nt) {
    case 1: return launch_gemv_tc_n<1>(p, dec_warps, maps, grid, stream);
    case 2: return launch_gemv_tc_n<2>(p, dec_warps, maps, grid, stream);
    default: return launch_gemv_tc_n<4>(p, dec_warps, maps, grid, stream);
  }
}

}  // namespace mambo
