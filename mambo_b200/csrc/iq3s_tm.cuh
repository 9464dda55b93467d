// Shared pieces of the tcgen05 IQ3_S kernels (GEMV and GEMM): the tile-major
// weight record, the lane-private codebook and the per-group decoder that
// turns IQ3_S codes into E4M3 bytes for the tensor core's A operand.
#pragma once

#include "common.cuh"

namespace mambo {
namespace tm {

// Codebook in shared memory: 512 entries x 32 lanes x 4 bytes, one copy per lane.
constexpr int kTableBytes = 512 * 32 * 4;
// The codebook as read from global memory (uint32[512], E4M3-encoded magnitudes).
constexpr uint32_t kTableStageBytes = 512 * 4;

// One tile-major record: the fields of a (128-row tile, K block) unit, written
// by iq3s_pack_kernel. qs and signs are chunk-major ([16-byte chunk][row][16
// bytes]), qh [4-byte column][row][4 bytes]; then d [row] and scales [row].
// Sign and qh words are bit-permuted (see decode_group_packed).
constexpr int kRecordRows = 128;
constexpr uint32_t kRecQs = 0, kRecSigns = 8192, kRecQh = 12288, kRecD = 13312, kRecScales = 13568;
constexpr uint32_t kRecordBytes = 14080;

// Expands the 8 codes of one 32-weight group into E4M3 bytes (4 per register).
//   q0, q1: the group's 8 qs bytes; hb: its qh byte (bit c = 9th index bit of
//   code c); sg: its 32 sign bits (bit 4c+j = sign of weight j of code c);
//   l4: (lane << 2) in every byte. Codebook entry e of lane l sits at byte
//   (e & 0xFF) << 8 | (e >> 8) << 7 | l << 2, so lanes never share a bank.
//   n * 0x10204080 (n < 16) puts bit j of n on bit 8j+7 (other partial
//   products land elsewhere, without carries, and are masked off);
//   n * 0x01020408 does the same for a nibble held in bits 4-7.
static __device__ __forceinline__ void decode_group(const uint8_t* table, uint32_t q0, uint32_t q1, uint32_t hb,
                                                    uint32_t sg, uint32_t l4, uint32_t* v) {
  const uint32_t h0 = lop3_and_or((hb & 0xFu) * 0x10204080u, 0x80808080u, l4);   // byte j: h_j << 7 | lane << 2
  const uint32_t h1 = lop3_and_or((hb & 0xF0u) * 0x01020408u, 0x80808080u, l4);  // codes 4..7
  const uint32_t q0l = q0 & 0xFFFFu, q0h = q0 >> 16, q1l = q1 & 0xFFFFu, q1h = q1 >> 16;
  const uint32_t m0 = *reinterpret_cast<const uint32_t*>(table + prmt(q0l, h0, 0x3204u));
  const uint32_t m1 = *reinterpret_cast<const uint32_t*>(table + prmt(q0l, h0, 0x3215u));
  const uint32_t m2 = *reinterpret_cast<const uint32_t*>(table + prmt(q0h, h0, 0x3206u));
  const uint32_t m3 = *reinterpret_cast<const uint32_t*>(table + prmt(q0h, h0, 0x3217u));
  const uint32_t m4 = *reinterpret_cast<const uint32_t*>(table + prmt(q1l, h1, 0x3204u));
  const uint32_t m5 = *reinterpret_cast<const uint32_t*>(table + prmt(q1l, h1, 0x3215u));
  const uint32_t m6 = *reinterpret_cast<const uint32_t*>(table + prmt(q1h, h1, 0x3206u));
  const uint32_t m7 = *reinterpret_cast<const uint32_t*>(table + prmt(q1h, h1, 0x3217u));
  const uint32_t s2 = sg >> 8, s4 = sg >> 16, s6 = sg >> 24;
  v[0] = lop3_and_or((sg & 0xFu) * 0x10204080u, 0x80808080u, m0);
  v[1] = lop3_and_or((sg & 0xF0u) * 0x01020408u, 0x80808080u, m1);
  v[2] = lop3_and_or((s2 & 0xFu) * 0x10204080u, 0x80808080u, m2);
  v[3] = lop3_and_or((s2 & 0xF0u) * 0x01020408u, 0x80808080u, m3);
  v[4] = lop3_and_or((s4 & 0xFu) * 0x10204080u, 0x80808080u, m4);
  v[5] = lop3_and_or((s4 & 0xF0u) * 0x01020408u, 0x80808080u, m5);
  v[6] = lop3_and_or((s6 & 0xFu) * 0x10204080u, 0x80808080u, m6);
  v[7] = lop3_and_or((sg >> 28) * 0x10204080u, 0x80808080u, m7);
}

// As decode_group, for the bit-permuted words of a packed record: hw is the
// thread's 4-group qh word with code c's high bit of group g at bit 8j+7-(2g+h)
// (c = 4h+j), hs = 2g for this group; sg is the group's sign word with weight
// j of code c at bit 8j+7-c. Both expand with a shift and one LOP3.
static __device__ __forceinline__ void decode_group_packed(const uint8_t* table, uint32_t q0, uint32_t q1,
                                                           uint32_t hw, uint32_t hs, uint32_t sg, uint32_t l4,
                                                           uint32_t* v) {
  const uint32_t h0 = lop3_and_or(hw << hs, 0x80808080u, l4);         // byte j: h_j << 7 | lane << 2
  const uint32_t h1 = lop3_and_or(hw << (hs + 1u), 0x80808080u, l4);  // codes 4..7
  const uint32_t q0l = q0 & 0xFFFFu, q0h = q0 >> 16, q1l = q1 & 0xFFFFu, q1h = q1 >> 16;
  const uint32_t m0 = *reinterpret_cast<const uint32_t*>(table + prmt(q0l, h0, 0x3204u));
  const uint32_t m1 = *reinterpret_cast<const uint32_t*>(table + prmt(q0l, h0, 0x3215u));
  const uint32_t m2 = *reinterpret_cast<const uint32_t*>(table + prmt(q0h, h0, 0x3206u));
  const uint32_t m3 = *reinterpret_cast<const uint32_t*>(table + prmt(q0h, h0, 0x3217u));
  const uint32_t m4 = *reinterpret_cast<const uint32_t*>(table + prmt(q1l, h1, 0x3204u));
  const uint32_t m5 = *reinterpret_cast<const uint32_t*>(table + prmt(q1l, h1, 0x3215u));
  const uint32_t m6 = *reinterpret_cast<const uint32_t*>(table + prmt(q1h, h1, 0x3206u));
  const uint32_t m7 = *reinterpret_cast<const uint32_t*>(table + prmt(q1h, h1, 0x3217u));
  v[0] = lop3_and_or(sg, 0x80808080u, m0);
  v[1] = lop3_and_or(sg << 1, 0x80808080u, m1);
  v[2] = lop3_and_or(sg << 2, 0x80808080u, m2);
  v[3] = lop3_and_or(sg << 3, 0x80808080u, m3);
  v[4] = lop3_and_or(sg << 4, 0x80808080u, m4);
  v[5] = lop3_and_or(sg << 5, 0x80808080u, m5);
  v[6] = lop3_and_or(sg << 6, 0x80808080u, m6);
  v[7] = lop3_and_or(sg << 7, 0x80808080u, m7);
}

// Builds the lane-private codebook: `tw` holds this thread's share of the
// 2 KB global table (read early to hide its latency), staged in `tstage`.
// All `nthreads` decoder threads (tid 0..nthreads-1) take part; named barrier 1.
template <int kWords>
static __device__ __forceinline__ void build_table(uint8_t* table, uint32_t* tstage, const uint32_t (&tw)[kWords],
                                                   int tid, int nthreads) {
#pragma unroll
  for (int j = 0; j < kWords; ++j) tstage[tid + j * nthreads] = tw[j];
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
  // Four lanes' copies (16 contiguous bytes) per store.
  for (int i = tid; i < 512 * 8; i += nthreads) {
    const uint32_t code = i >> 3, l0 = (i & 7) * 4, e = tstage[code];
    *reinterpret_cast<uint4*>(table + (((code & 0xFFu) << 8) | ((code >> 8) << 7) | (l0 << 2))) =
        make_uint4(e, e, e, e);
  }
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Elects one lane of a converged warp (tcgen05.mma reads its operands from
// uniform registers: issuing from a converged warp keeps them there).
static __device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// Waits (bounded) on an mbarrier phase: a non-blocking try first, then the
// bounded slow path, with the whole warp agreeing on the outcome.
static __device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int site) {
  if (__all_sync(0xFFFFFFFFu, mbar_try_wait(bar, parity))) return true;
  return __all_sync(0xFFFFFFFFu, mbar_wait_bounded(bar, parity, site));
}
// As warp_wait for a barrier that the other CTA of a cluster also arrives on
// (acquire at cluster scope).
static __device__ __forceinline__ bool warp_wait_cluster(uint32_t bar, uint32_t parity, int site) {
  if (__all_sync(0xFFFFFFFFu, mbar_try_wait_cluster(bar, parity))) return true;
  return __all_sync(0xFFFFFFFFu, mbar_wait_cluster_bounded(bar, parity, site));
}

}  // namespace tm
}  // namespace mambo
