// tcgen05 (5th-generation tensor core) helpers for sm_100a: TMEM allocation,
// shared-memory matrix descriptors, MMA issue/commit and TMEM loads.
#pragma once

#include "common.cuh"

namespace mambo {
namespace tc {

// Shared-memory matrix descriptor (tcgen05 format): start address, leading and
// stride byte offsets (all >> 4), descriptor version 1 at bit 46, no swizzle.
// K-major, no-swizzle canonical layout: 8-row x 16-byte core matrices stored as
// 128 contiguous bytes; `lbo` = distance between core matrices along K,
// `sbo` = distance between 8-row groups along M/N.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// Shared-memory matrix descriptor, K-major with the 128-byte swizzle: 8-row x
// 128-byte atoms (1024-byte aligned), `sbo` = distance between 8-row groups.
// Layout type 2 (SWIZZLE_128B) at bits 61-63. A K step inside the 128-byte
// row advances the start address by its byte offset.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;  // leading byte offset: unused for swizzled K-major
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor of kind::f8f6f4: D = F32, A = B = E4M3, both K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] x B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_e4m3(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}

// Instruction descriptor of kind::f16: D = F32, A = B = F16, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A[tmem] x B[smem]^T with FP16 operands (K = 16), issued by one
// thread. A occupies the TMEM lanes of its rows, two FP16 values per column.
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t desc_b, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}

// D[tmem] (+)= A[tmem] x B[smem]^T, issued by one thread. A occupies the TMEM
// lanes of its rows, K packed four E4M3 values per 32-bit column.
__device__ __forceinline__ void mma_e4m3_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t desc_b, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}

// Instruction descriptor of kind::mxf8f6f4 (block-scaled, UE8M0 scales, one
// per 32 K elements): A = B = E4M3, both K-major, D = F32. b_id / a_id pick
// the byte of the 32-bit scale-factor element of TMEM the MMA uses.
__host__ __device__ constexpr uint32_t idesc_mx_e4m3(int m, int n, uint32_t b_id, uint32_t a_id) {
  return (b_id << 4) | ((uint32_t)(n >> 3) << 17) | (1u << 23) | ((uint32_t)(m >> 4) << 24) | (a_id << 29);
}

// D[tmem] (+)= (A[tmem] * 2^sfa) x (B[smem] * 2^sfb)^T, issued by one thread;
// the scale factors of A's rows and B's columns are read from TMEM.
__device__ __forceinline__ void mma_mx_e4m3_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t desc_b, uint32_t idesc,
                                               uint32_t tmem_sfa, uint32_t tmem_sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale.scale_vec::1X [%0], [%1], %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          tmem_d),
      "r"(tmem_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(tmem_sfa), "r"(tmem_sfb));
}

// Copies a 32-row x 16-byte matrix from shared memory (descriptor `sdesc`)
// to 4 consecutive 32-bit columns of TMEM lanes 0-31, repeated in each of the
// four 32-lane quadrants (the layout of MMA scale factors). Ordered before
// later tcgen05.mma of the issuing thread.
__device__ __forceinline__ void cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Each lane writes 4 consecutive 32-bit columns of its TMEM lane (warp-wide).
__device__ __forceinline__ void st_x4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// Each lane writes 8 consecutive 32-bit columns of its TMEM lane (warp-wide).
__device__ __forceinline__ void st_x8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
// Each lane writes N (16 or 32) consecutive 32-bit columns of its TMEM lane.
// No memory clobber: the store touches tensor memory only, so shared-memory
// loads after it may be scheduled ahead of it (tcgen05.wait::st orders it).
template <int N>
__device__ __forceinline__ void st_cols(uint32_t taddr, const uint32_t (&v)[N]) {
  static_assert(N == 16 || N == 32, "16 or 32 columns");
  if constexpr (N == 16) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]));
  } else {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31]));
  }
}

// Loads 8 consecutive 32-bit columns of this lane's TMEM row for each of G
// column offsets, then waits once for all of them.
template <int G>
__device__ __forceinline__ void ld_x8_multi(uint32_t taddr, const uint32_t (&off)[G], float (&v)[G][8]) {
  uint32_t r[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[g][0]), "=r"(r[g][1]), "=r"(r[g][2]), "=r"(r[g][3]), "=r"(r[g][4]), "=r"(r[g][5]),
                   "=r"(r[g][6]), "=r"(r[g][7])
                 : "r"(taddr + off[g]));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  // Tie the registers to the wait: every use below depends on this empty asm.
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      asm volatile("" : "+r"(r[g][i]));
      v[g][i] = __uint_as_float(r[g][i]);
    }
}

// Waits until this thread's earlier tcgen05.st have completed.
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrives (once) on the mbarrier when all MMAs previously issued by this thread complete.
__device__ __forceinline__ void commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Whole-warp TMEM allocation; the TMEM address is written to shared memory at dst.
__device__ __forceinline__ void alloc(uint32_t dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (cta_group::2, a cluster of two CTAs): one MMA spans both CTAs'
// tensor cores. A (M = 256) is rows 0-127 from CTA rank 0's TMEM and rows
// 128-255 from rank 1's, at the same TMEM address; B (N) is columns 0..N/2-1
// from rank 0's shared memory and N/2..N-1 from rank 1's, at the same
// address; D rows land in the TMEM of the CTA that supplied them. Rank 0
// issues the MMAs.
// ---------------------------------------------------------------------------
// Allocation, release and free: one warp of each CTA, the same warp in both,
// the same dst address.
__device__ __forceinline__ void alloc_pair(uint32_t dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// The pair MMA with FP16 operands (K = 16), A from TMEM; issued by one thread of rank 0.
__device__ __forceinline__ void mma_f16_ts_pair(uint32_t tmem_d, uint32_t tmem_a, uint64_t desc_b, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}
// Arrives on the barrier at address bar (a CTA-local offset) in every CTA of
// cta_mask once the issuing thread's earlier pair MMAs have completed.
__device__ __forceinline__ void commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Each lane reads 8 consecutive 32-bit columns of its TMEM lane at two
// addresses, then waits for both loads. The wait names the destination
// registers so that no use of them can be scheduled before it.
__device__ __forceinline__ void ld_x8_pair(uint32_t taddr0, uint32_t taddr1, float (&v0)[8], float (&v1)[8]) {
  uint32_t a[8], b[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7])
               : "r"(taddr0));
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7])
               : "r"(taddr1));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                 "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v0[i] = __uint_as_float(a[i]);
    v1[i] = __uint_as_float(b[i]);
  }
}

}  // namespace tc
}  // namespace mambo
