// MXFP8 activation quantization (sm_100a).
//
// Restates quantize_fp8_group / quantize_activation_fp8
// (src/python/mambo/kernels/quantize_fp8.py:23-52): per 32 consecutive values
// along K, amax -> e = clamp(ceil(log2(amax/448)), -127, 127) (amax == 0 -> 0),
// q = E4M3(x * 2^-e), scale byte e + 127. The exponent is computed exactly
// from the bits of amax (no log2 approximation).
//
// Layout: each warp quantizes 8 groups per step; 4 lanes own one group of 32
// (8 values each, one 128-bit load for bf16 / two for f32), amax is reduced
// with two quad shuffles, and each lane writes its 8 E4M3 bytes as one 64-bit
// store (a warp writes 256 contiguous bytes).
#include "kernels.cuh"
#include "mxfp8.cuh"

namespace mambo {

__device__ __forceinline__ float e4m3_to_float(uint32_t byte) {
  uint32_t h2;
  const uint16_t in = (uint16_t)(byte & 0xFFu);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(in));
  return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
}

// Round-to-nearest with exact ties resolved toward the smaller magnitude:
// start from the RNE code and step the magnitude down by one code when y sat
// exactly halfway and RNE rounded away from zero. All differences are exact.
__device__ __forceinline__ uint32_t fix_tie_down(uint32_t code, float y) {
  const uint32_t mag = code & 0x7Fu;
  if (mag == 0) return code;
  const float ay = fabsf(y);
  const float up = e4m3_to_float(mag);
  if (!(up > ay)) return code;
  const float down = e4m3_to_float(mag - 1u);
  return (up - ay == ay - down) ? ((code & 0x80u) | (mag - 1u)) : code;
}

template <typename T, bool kVec, int kRounding>
__global__ void __launch_bounds__(256) quantize_mxfp8_kernel(const QuantParams p) {
  const int lane = threadIdx.x & 31;
  const int quad_lane = lane & 3;
  const int64_t groups_per_row = p.k / 32;
  const int64_t total_groups = p.m * groups_per_row;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int64_t warp_id = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const T* x = static_cast<const T*>(p.x);
  // The activations may come from the previous kernel, and the outputs may
  // still be read by it: wait for it, then let the next kernel start early.
  pdl_wait();
  pdl_launch_dependents();

  for (int64_t base = warp_id * 8; base < total_groups; base += warps * 8) {
    const int64_t grp = base + (lane >> 2);
    const bool active = grp < total_groups;
    const int64_t row = active ? grp / groups_per_row : 0;
    const int64_t cg = active ? grp - row * groups_per_row : 0;
    const T* src = x + row * p.ldx + cg * 32 + quad_lane * 8;

    float v[8];
    if (active) {
      if constexpr (sizeof(T) == 2) {
        if constexpr (kVec) {
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src));
          const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
          }
        } else {
          const uint16_t* s16 = reinterpret_cast<const uint16_t*>(src);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = __uint_as_float((uint32_t)__ldg(s16 + i) << 16);
        }
      } else {
        if constexpr (kVec) {
          const float4 a = __ldg(reinterpret_cast<const float4*>(src));
          const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
          v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
          v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
          const float* sf = reinterpret_cast<const float*>(src);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = __ldg(sf + i);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }

    const uint32_t code = mxfp8_scale_code(quad_absmax(v));
    // 2^-e with e = code - 127 (code 0xFF: scale by 2^-127, values become 0 / NaN / +-448).
    const float inv = e8m0_to_float(code == 0xFFu ? 0u : 254u - code);

    uint32_t packed[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float y[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) y[i] = v[4 * h + i] * inv;
      uint32_t lo = cvt_e4m3x2_rn(y[0], y[1]);
      uint32_t hi = cvt_e4m3x2_rn(y[2], y[3]);
      if constexpr (kRounding == MAMBO_ROUND_TIES_DOWN) {
        uint32_t b0 = fix_tie_down(lo & 0xFFu, y[0]), b1 = fix_tie_down(lo >> 8, y[1]);
        uint32_t b2 = fix_tie_down(hi & 0xFFu, y[2]), b3 = fix_tie_down(hi >> 8, y[3]);
        lo = b0 | (b1 << 8);
        hi = b2 | (b3 << 8);
      }
      packed[h] = lo | (hi << 16);
    }

    if (p.sums != nullptr) {
      // The group's quantized values summed: E4M3 values are multiples of 2^-9
      // below 2^9, so a sum of 32 of them needs at most 23 bits and is exact in
      // FP32 in any order; times 2^e (exact). A NaN scale code gives NaN.
      float sum = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t h2;
          const uint16_t two = (uint16_t)(packed[h] >> (16 * j));
          asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(two));
          sum += __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
          sum += __half2float(__ushort_as_half((unsigned short)(h2 >> 16)));
        }
      }
      sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
      sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
      if (active && quad_lane == 0)
        p.sums[row * p.ld_sums + cg] = code == 0xFFu ? __uint_as_float(0x7FC00000u) : sum * e8m0_to_float(code);
    }

    if (active) {
      uint8_t* dst = p.q + row * p.ldq + cg * 32 + quad_lane * 8;
      if constexpr (kVec) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(packed[0], packed[1]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = (uint8_t)(packed[i / 4] >> (8 * (i % 4)));
      }
      if (quad_lane == 0) p.s[row * p.lds + cg] = (uint8_t)code;
    }
  }
}

template <typename T, bool kVec>
static cudaError_t launch_quant_t(const QuantParams& p, int rounding, int grid, cudaStream_t stream) {
  const void* kern = rounding == MAMBO_ROUND_TIES_DOWN
                         ? (const void*)quantize_mxfp8_kernel<T, kVec, MAMBO_ROUND_TIES_DOWN>
                         : (const void*)quantize_mxfp8_kernel<T, kVec, MAMBO_ROUND_NEAREST_EVEN>;
  return launch_pdl(kern, dim3(grid), dim3(256), 0, stream, p);
}

cudaError_t launch_quantize_mxfp8(const QuantParams& p, int x_dtype, int rounding, int num_sms, cudaStream_t stream) {
  const int64_t groups = p.m * (p.k / 32);
  const int64_t warp_steps = (groups + 7) / 8;
  int64_t blocks = (warp_steps + 7) / 8;  // 8 warps per block
  const int64_t cap = (int64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const uintptr_t xa = reinterpret_cast<uintptr_t>(p.x);
  const uintptr_t qa = reinterpret_cast<uintptr_t>(p.q);
  const bool q_vec = (qa % 8 == 0) && (p.ldq % 8 == 0);
  if (x_dtype == MAMBO_BF16) {
    const bool vec = q_vec && (xa % 16 == 0) && (p.ldx % 8 == 0);
    return vec ? launch_quant_t<uint16_t, true>(p, rounding, (int)blocks, stream)
               : launch_quant_t<uint16_t, false>(p, rounding, (int)blocks, stream);
  }
  const bool vec = q_vec && (xa % 16 == 0) && (p.ldx % 4 == 0);
  return vec ? launch_quant_t<float, true>(p, rounding, (int)blocks, stream)
             : launch_quant_t<float, false>(p, rounding, (int)blocks, stream);
}

// Activation tiles of a grouped GEMV launch (GemvGroupPre): one CTA per
// (item, K block), one warp per token. Lane 4g + j takes values 8j .. 8j+7 of
// 32-value group g, so a quad holds a group, as quantize_mxfp8_kernel's lanes
// do, and writes its 8 E4M3 bytes where the GEMV's B tile keeps them (K chunk
// 2g + j/2 of 16 values, token row t); lane 4g writes the scale code into row t
// of scale block g/4, byte g%4.
__global__ void __launch_bounds__(256) group_xtiles_kernel(const __grid_constant__ GroupXtilesParams p) {
  pdl_wait();  // the activations may come from the previous kernel
  pdl_launch_dependents();
  const int tile = blockIdx.x;
  int l = 0;
  while (l + 1 < p.count && p.items[l + 1].xt0 <= tile) ++l;
  const GroupXtilesParams::Item& it = p.items[l];
  const int kb = tile - it.xt0;
  uint8_t* dst = p.tiles + (size_t)tile * (size_t)(288 * p.box);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, j = lane & 3;
  for (int t = warp; t < it.m; t += 8) {
    const uint4 c = __ldg(reinterpret_cast<const uint4*>(it.x + (size_t)t * it.ldx + (size_t)kb * 256 + g * 32 + j * 8));
    uint2 q;
    const uint32_t code = mxfp8_quad_bf16_rne(c, q);
    *reinterpret_cast<uint2*>(dst + ((2 * g + (j >> 1)) * p.box + t) * 16 + (j & 1) * 8) = q;
    if (j == 0) dst[256 * p.box + (g >> 2) * 16 * p.box + t * 16 + (g & 3)] = (uint8_t)code;
    if (it.sums != nullptr) {
      // The group's quantized values summed (exact in FP32 in any order: 32 E4M3 values need at
      // most 23 bits), times 2^e; a NaN scale code gives NaN (as quantize_mxfp8_kernel's sums).
      float sum = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t w = h ? q.y : q.x;
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          uint32_t h2;
          const uint16_t two = (uint16_t)(w >> (16 * b));
          asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(two));
          sum += __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
          sum += __half2float(__ushort_as_half((unsigned short)(h2 >> 16)));
        }
      }
      sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
      sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
      if (j == 0)
        it.sums[(size_t)t * it.ld_sums + (size_t)kb * 8 + g] =
            code == 0xFFu ? __uint_as_float(0x7FC00000u) : sum * e8m0_to_float(code);
    }
  }
}

cudaError_t launch_group_xtiles(const GroupXtilesParams& p, cudaStream_t stream) {
  if (p.total_tiles < 1) return cudaSuccess;
  return launch_pdl((const void*)group_xtiles_kernel, dim3((unsigned)p.total_tiles), dim3(256), 0, stream, p);
}

}  // namespace mambo
