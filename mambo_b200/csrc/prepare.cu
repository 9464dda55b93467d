// IQ3_S weight preparation (AoS GGUF blocks -> SoA fields) and the standalone
// decoder used by the bit-exactness tests.
#include <cuda_fp16.h>

#include "kernels.cuh"

namespace mambo {

// Field sizes and byte offsets inside one 110-byte block
// (src/python/mambo/utils/iq3_s_weight.py:26-33): d 0..1, qs 2..65, qh 66..73,
// signs 74..105, scales 106..109.
__device__ __forceinline__ void field_of_byte(int byte, int& field, int& off, int& size) {
  if (byte < 2) { field = 0; off = 0; size = 2; }
  else if (byte < 66) { field = 1; off = 2; size = 64; }
  else if (byte < 74) { field = 2; off = 66; size = 8; }
  else if (byte < 106) { field = 3; off = 74; size = 32; }
  else { field = 4; off = 106; size = 4; }
}

// One thread per source byte; raw may have any strides and alignment
// (prepare_iq3_s_fields accepts odd-address and strided views, test_iq3_s_fp8.py:118-131).
__global__ void iq3s_prepare_kernel(const PrepareParams p) {
  const int64_t total = p.n_rows * p.n_blocks * 110;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int byte = (int)(i % 110);
    const int64_t nb = i / 110;
    const int64_t b = nb % p.n_blocks;
    const int64_t n = nb / p.n_blocks;
    const uint8_t v = p.raw[n * p.stride_row + b * p.stride_block + byte * p.stride_byte];
    int field, off, size;
    field_of_byte(byte, field, off, size);
    p.dst[field][(b * p.n_rows + n) * size + (byte - off)] = v;
  }
}

cudaError_t launch_iq3s_prepare(const PrepareParams& p, int num_sms, cudaStream_t stream) {
  const int64_t total = p.n_rows * p.n_blocks * 110;
  int64_t blocks = (total + 255) / 256;
  if (blocks > (int64_t)num_sms * 32) blocks = (int64_t)num_sms * 32;
  if (blocks < 1) blocks = 1;
  iq3s_prepare_kernel<<<(int)blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

// One thread per 16-byte chunk of the packed buffer. Record layout (one
// 128-row tile t, one K block b): qs [4 chunks][128 rows][16 B], signs
// [2 chunks][128 rows][16 B], qh [2 columns][128 rows][4 B], d [128] fp16,
// scales [128][4 B]; rows past N are zero (N % 8 == 0, so a chunk never mixes
// valid and padding rows).
// Bit permutations of the packed record (the decoder's shift-and-mask forms):
// a group's sign word, bit 4c+j (weight j of code c) -> bit 8j+7-c, so that
// (w << c) & 0x80808080 puts code c's four signs on bit 7 of each byte;
// a 4-group qh word, bit 8g+4h+j (code 4h+j of group g) -> bit 8j+7-(2g+h),
// so that (w << (2g+h)) & 0x80808080 puts those codes' high index bits there.
__device__ __forceinline__ uint32_t permute_sign_word(uint32_t w) {
  uint32_t o = 0;
#pragma unroll
  for (int c = 0; c < 8; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j) o |= ((w >> (4 * c + j)) & 1u) << (8 * j + 7 - c);
  return o;
}
__device__ __forceinline__ uint32_t permute_qh_word(uint32_t w) {
  uint32_t o = 0;
#pragma unroll
  for (int g = 0; g < 4; ++g)
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int j = 0; j < 4; ++j) o |= ((w >> (8 * g + 4 * h + j)) & 1u) << (8 * j + 7 - (2 * g + h));
  return o;
}

__global__ void iq3s_pack_kernel(const PackWeightParams p) {
  constexpr int kChunks = 14080 / 16;
  const int64_t tiles = (p.n_rows + 127) / 128;
  const int64_t total = tiles * p.n_blocks * kChunks;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rec = i / kChunks;
    const int off = (int)(i - rec * kChunks) * 16;
    const int64_t t = rec / p.n_blocks, b = rec - t * p.n_blocks;
    const int64_t row0 = b * p.n_rows + t * 128;  // SoA index of the tile's first row
    uint4 v = make_uint4(0, 0, 0, 0);
    if (off < 12288) {  // qs or signs: 16 bytes of one row
      const bool is_qs = off < 8192;
      const int o = is_qs ? off : off - 8192, c = o / 2048, r = (o % 2048) / 16;
      if (t * 128 + r < p.n_rows) {
        v = __ldg(reinterpret_cast<const uint4*>((is_qs ? p.qs : p.signs) + (row0 + r) * (is_qs ? 64 : 32) + c * 16));
        if (!is_qs) {
          v.x = permute_sign_word(v.x);
          v.y = permute_sign_word(v.y);
          v.z = permute_sign_word(v.z);
          v.w = permute_sign_word(v.w);
        }
      }
    } else if (off < 13312) {  // qh: 4 bytes of 4 consecutive rows
      const int o = off - 12288, c = o / 512, r = (o % 512) / 4;
      if (t * 128 + r < p.n_rows) {
        const uint8_t* src = p.qh + (row0 + r) * 8 + c * 4;
        v = make_uint4(permute_qh_word(__ldg(reinterpret_cast<const uint32_t*>(src))),
                       permute_qh_word(__ldg(reinterpret_cast<const uint32_t*>(src + 8))),
                       permute_qh_word(__ldg(reinterpret_cast<const uint32_t*>(src + 16))),
                       permute_qh_word(__ldg(reinterpret_cast<const uint32_t*>(src + 24))));
      }
    } else {  // d and scales: rows contiguous
      const bool is_d = off < 13568;
      const int o = is_d ? off - 13312 : off - 13568, bpr = is_d ? 2 : 4, r = o / bpr;
      if (t * 128 + r < p.n_rows) v = __ldg(reinterpret_cast<const uint4*>((is_d ? p.d : p.scales) + row0 * bpr + o));
    }
    reinterpret_cast<uint4*>(p.packed)[i] = v;
  }
}

// The stored 4-bit code of Q4_K value q (0..15): the odd integer v = 2q - 15
// as (v > 0) << 3 | (|v| - 1) / 2, which is q for q >= 8 and 7 - q below.
__device__ __forceinline__ uint32_t q4k_stored_code(uint32_t q) { return q >= 8u ? q : 7u - q; }

// One thread per 16-byte chunk of the Q4_K packed buffer (record layout in kernels.cuh).
__global__ void q4k_pack_kernel(const Q4kPackParams p) {
  constexpr int kChunks = (int)(kQ4kRecordBytes / 16);
  const int64_t tiles = (p.n_rows + 127) / 128;
  const int64_t total = tiles * p.n_blocks * kChunks;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rec = i / kChunks;
    const int off = (int)(i - rec * kChunks) * 16;
    const int64_t t = rec / p.n_blocks, b = rec - t * p.n_blocks;
    uint8_t out[16];
    // Source byte of block (row, b) at in-block offset o.
    auto src = [&](int64_t row, int o) -> uint8_t {
      return row < p.n_rows ? __ldg(p.raw + row * p.stride_row + b * p.stride_block + (int64_t)o * p.stride_byte) : 0;
    };
    if (off < (int)kQ4kRecDm) {  // codes: 16 bytes of one row, re-coded and regrouped per 32-bit word
      const int c = off / 2048, r = (off % 2048) / 16;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t lo = 0, hi = 0;  // the four low nibbles (group 2c'), the four high ones (group 2c'+1)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t byte = src(t * 128 + r, 16 + 16 * c + 4 * w + j);
          lo |= q4k_stored_code(byte & 15u) << (4 * j);
          hi |= q4k_stored_code(byte >> 4) << (4 * j);
        }
        const uint32_t word = lo | (hi << 16);
#pragma unroll
        for (int j = 0; j < 4; ++j) out[4 * w + j] = (uint8_t)(word >> (8 * j));
      }
    } else if (off < (int)kQ4kRecSc) {  // d, dmin: 4 rows x 4 bytes
      const int r0 = (off - (int)kQ4kRecDm) / 4;
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] = src(t * 128 + r0 + j / 4, j % 4);
    } else {  // scales and mins: 12 bytes per row, rows back to back
      const int o0 = off - (int)kQ4kRecSc;
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] = src(t * 128 + (o0 + j) / 12, 4 + (o0 + j) % 12);
    }
    uint4 v;
    v.x = out[0] | (out[1] << 8) | (out[2] << 16) | ((uint32_t)out[3] << 24);
    v.y = out[4] | (out[5] << 8) | (out[6] << 16) | ((uint32_t)out[7] << 24);
    v.z = out[8] | (out[9] << 8) | (out[10] << 16) | ((uint32_t)out[11] << 24);
    v.w = out[12] | (out[13] << 8) | (out[14] << 16) | ((uint32_t)out[15] << 24);
    reinterpret_cast<uint4*>(p.packed)[i] = v;
  }
}

cudaError_t launch_q4k_pack(const Q4kPackParams& p, int num_sms, cudaStream_t stream) {
  const int64_t chunks = (p.n_rows + 127) / 128 * p.n_blocks * (kQ4kRecordBytes / 16);
  int64_t blocks = (chunks + 255) / 256;
  if (blocks > (int64_t)num_sms * 16) blocks = (int64_t)num_sms * 16;
  q4k_pack_kernel<<<(int)blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

// The exponent of each row's largest block scale, floor(log2(max_b |d_b|))
// over the finite d of the row (0 for a row without a finite non-zero d;
// rows past N, up to whole 128-row tiles, also 0): the folded FP16 GEMM
// scales each row's weights by 2^-e so that they stay in FP16's normal range.
// One thread per row.
__global__ void iq3s_row_exp_kernel(const uint16_t* __restrict__ d, int64_t n_rows, int64_t n_blocks, int64_t rows_pad,
                                    int8_t* __restrict__ row_exp) {
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows_pad;
       r += (int64_t)gridDim.x * blockDim.x) {
    uint32_t mag = 0;  // largest finite |d| as fp16 bits (ordered like the values)
    if (r < n_rows)
      for (int64_t b = 0; b < n_blocks; ++b) {
        const uint32_t m = __ldg(d + b * n_rows + r) & 0x7FFFu;
        if (m < 0x7C00u) mag = max(mag, m);  // skip Inf and NaN
      }
    int e = 0;
    if (mag != 0) {
      const float v = __half2float(__ushort_as_half((unsigned short)mag));
      e = (int)((__float_as_uint(v) >> 23) & 0xFFu) - 127;
    }
    row_exp[r] = (int8_t)e;
  }
}

cudaError_t launch_iq3s_row_exp(const uint8_t* d, int64_t n_rows, int64_t n_blocks, int8_t* row_exp,
                                cudaStream_t stream) {
  const int64_t rows_pad = (n_rows + 127) / 128 * 128;
  iq3s_row_exp_kernel<<<(unsigned)((rows_pad + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const uint16_t*>(d), n_rows, n_blocks, rows_pad, row_exp);
  return cudaGetLastError();
}

cudaError_t launch_iq3s_pack(const PackWeightParams& p, int num_sms, cudaStream_t stream) {
  const int64_t total = (p.n_rows + 127) / 128 * p.n_blocks * (14080 / 16);
  int64_t blocks = (total + 255) / 256;
  if (blocks > (int64_t)num_sms * 32) blocks = (int64_t)num_sms * 32;
  if (blocks < 1) blocks = 1;
  iq3s_pack_kernel<<<(int)blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

// One warp per (row, block): lane l decodes codes 2l and 2l+1 (weights 8l..8l+7).
// Mirrors decode_iq3_s_blocks (src/python/mambo/kernels/iq3_s_fp8.py:202-222).
__global__ void iq3s_decode_kernel(const DecodeParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t wb = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; wb < p.n_rows * p.n_blocks;
       wb += warps) {
    const int64_t n = wb / p.n_blocks;
    const int64_t b = wb % p.n_blocks;
    const int64_t blk = b * p.n_rows + n;  // SoA index
    const int g = lane >> 2;               // 32-weight group of this lane's codes
    const uint32_t q0 = p.qs[blk * 64 + 2 * lane];
    const uint32_t q1 = p.qs[blk * 64 + 2 * lane + 1];
    const uint32_t hbyte = p.qh[blk * 8 + g];
    const uint32_t c0 = 2 * (lane & 3), c1 = c0 + 1;  // code index inside the group
    const uint32_t i0 = q0 | (((hbyte >> c0) & 1u) << 8);
    const uint32_t i1 = q1 | (((hbyte >> c1) & 1u) << 8);
    const uint32_t sbyte = p.signs[blk * 32 + lane];  // weights 8l..8l+7
    const uint32_t w0 = __ldg(p.table + i0) | (((sbyte & 0xFu) * 0x10204080u) & 0x80808080u);
    const uint32_t w1 = __ldg(p.table + i1) | (((sbyte >> 4) * 0x10204080u) & 0x80808080u);
    uint2* dst = reinterpret_cast<uint2*>(p.values + n * (p.n_blocks * 256) + b * 256 + 8 * lane);
    *dst = make_uint2(w0, w1);
    if (lane < 8) {
      const uint16_t dh = (uint16_t)(p.d[blk * 2] | (p.d[blk * 2 + 1] << 8));
      const float dv = __half2float(__ushort_as_half(dh));
      const uint32_t nib = (p.scales[blk * 4 + lane / 2] >> (4 * (lane & 1))) & 0xFu;
      p.out_scales[n * (p.n_blocks * 8) + b * 8 + lane] = dv * (float)(1u + 2u * nib);
    }
  }
}

cudaError_t launch_iq3s_decode(const DecodeParams& p, int num_sms, cudaStream_t stream) {
  const int64_t warps = p.n_rows * p.n_blocks;
  int64_t blocks = (warps + 7) / 8;
  if (blocks > (int64_t)num_sms * 16) blocks = (int64_t)num_sms * 16;
  if (blocks < 1) blocks = 1;
  iq3s_decode_kernel<<<(int)blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace mambo
