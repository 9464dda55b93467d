// Parameter blocks and launchers shared between the kernel files and the C ABI.
#pragma once

#include "common.cuh"

namespace mambo {

// Sets a kernel's dynamic shared memory limit once per (kernel, device).
cudaError_t ensure_smem_attribute(const void* kernel, size_t smem_bytes);

// Launches with programmatic stream serialization (and, for cluster > 1, in
// thread-block clusters of `cluster` CTAs along x).
template <typename... Args>
cudaError_t launch_pdl_cluster(const void* kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, int cluster,
                               const Args&... args) {
  void* argv[] = {const_cast<void*>(static_cast<const void*>(&args))...};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    n = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelExC(&cfg, kernel, argv);
}

// Launches with programmatic stream serialization: the kernel may begin while
// the previous kernel in the stream finishes, and must call pdl_wait() before
// touching memory that kernel produces or consumes.
template <typename... Args>
cudaError_t launch_pdl(const void* kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       const Args&... args) {
  return launch_pdl_cluster(kernel, grid, block, smem, stream, 1, args...);
}

struct QuantParams {
  const void* x;
  int64_t m, k, ldx;
  uint8_t* q;
  int64_t ldq;
  uint8_t* s;
  int64_t lds;
  // Optional: per 32-value group, the sum of its quantized values E4M3 * 2^e in
  // FP32 ([m][k/32], row stride ld_sums), summed in a fixed order.
  float* sums;
  int64_t ld_sums;
};
cudaError_t launch_quantize_mxfp8(const QuantParams& p, int x_dtype, int rounding, int num_sms, cudaStream_t stream);

struct PrepareParams {
  const uint8_t* raw;
  int64_t n_rows, n_blocks, stride_row, stride_block, stride_byte;
  uint8_t* dst[5];
};
cudaError_t launch_iq3s_prepare(const PrepareParams& p, int num_sms, cudaStream_t stream);

struct DecodeParams {
  const uint8_t* d;
  const uint8_t* qs;
  const uint8_t* qh;
  const uint8_t* signs;
  const uint8_t* scales;
  int64_t n_rows, n_blocks;
  const uint32_t* table;  // uint32[512], E4M3-encoded magnitudes
  uint8_t* values;        // [N, B*256]
  float* out_scales;      // [N, B*8]
};
cudaError_t launch_iq3s_decode(const DecodeParams& p, int num_sms, cudaStream_t stream);

// SoA fields -> tile-major packed records (see mambo_iq3s_pack).
struct PackWeightParams {
  const uint8_t* d;
  const uint8_t* qs;
  const uint8_t* qh;
  const uint8_t* signs;
  const uint8_t* scales;
  int64_t n_rows, n_blocks;
  uint8_t* packed;
};
cudaError_t launch_iq3s_pack(const PackWeightParams& p, int num_sms, cudaStream_t stream);

// Q4_K (GGUF, 144 bytes per 256 values: fp16 d, fp16 dmin, 12 bytes of 6-bit
// scales and mins, 128 bytes of 4-bit codes q) in tile-major records of
// kQ4kRecordBytes per (128-row tile, K block): the codes chunk-major
// [8 chunks][128 rows][16 bytes], then [128 rows][4 bytes] d and dmin, then
// [128 rows][12 bytes] scales and mins; rows at or past N are zero. Chunk c
// holds code bytes 16c..16c+15 as four 32-bit words; the word of bytes
// b0..b3 carries their low nibbles (group 2(c/2)) in bits 0-15 and their high
// nibbles (group 2(c/2)+1) in bits 16-31, value j of a half in bits 4j..4j+3,
// each re-coded as the odd integer v = 2q - 15: (v > 0) << 3 | (|v| - 1) / 2.
constexpr uint32_t kQ4kRecordBytes = 18432;
constexpr uint32_t kQ4kRecDm = 16384, kQ4kRecSc = 16896;
struct Q4kPackParams {
  const uint8_t* raw;  // [N][B][144] with any byte strides
  int64_t n_rows, n_blocks, stride_row, stride_block, stride_byte;
  uint8_t* packed;
};
cudaError_t launch_q4k_pack(const Q4kPackParams& p, int num_sms, cudaStream_t stream);

struct GemvParams {
  const uint8_t* xq;
  int64_t ldxq;
  const uint8_t* xs;
  int64_t ldxs;
  int m;
  int n_rows;
  int n_blocks;
  // SoA weight fields (the TMA loader reads them through the tensor maps)
  const uint8_t* d;
  const uint8_t* qs;
  const uint8_t* qh;
  const uint8_t* signs;
  const uint8_t* scales;
  const uint32_t* table;
  void* out;
  int out_bf16;
  int64_t ldo;
  float* partials;  // [grid][2][rows][8*NT]
  int* counters;    // [row_tiles][warps], zero between launches
  int warps;        // consumer warps (16 weight rows each)
  int stages;
  int row_tiles;
  int total_units;
  int x_bulk;  // xq base and row stride 16-byte aligned: activation rows arrive by bulk copies
};

struct GemvMaps {
  CUtensorMap qs, signs, qh, d, scales;
};

bool make_gemv_maps(const GemvParams& p, GemvMaps* maps);
cudaError_t launch_gemv(const GemvParams& p, int nt, bool use_tma, const GemvMaps& maps, int grid,
                        cudaStream_t stream);
uint32_t gemv_smem_bytes_host(int rows, int nt, int stages, int n_blocks);

// tcgen05 GEMV with the decoded weight operand in tensor memory.
struct GemvTmParams {
  int m;  // tokens of this launch (<= 8*NT)
  int n_rows;
  int n_blocks;
  // SoA weight fields: for one K block, the fields of 128 consecutive rows are
  // contiguous, so a work unit arrives as five 1D bulk copies.
  const uint8_t* d;
  const uint8_t* qs;
  const uint8_t* qh;
  const uint8_t* signs;
  const uint8_t* scales;
  const uint8_t* packed;  // tile-major records (one copy per unit), or null: five copies from the fields
  const uint32_t* table;  // uint32[512], E4M3-encoded magnitudes
  void* out;
  int out_bf16;
  int64_t ldo;
  float* partials;  // [grid][2][128][8*NT]
  int* counters;    // [row_tiles][4], zero between launches
  int stages;
  int prefetch;  // units prefetched into L2 beyond the stage ring
  int kparts;    // > 0: row tile t is split into kparts K ranges, CTA t*kparts+k in a cluster of kparts; 0: stream-K
  int row_tiles;
  int total_units;
  // Tokens per activation TMA box (the maps' box rows; 1..8*NT, 0 = 8*NT):
  // boxes of the launch's own rows only, no out-of-bounds rows to fill.
  int box_rows;
  // Fused activation quantization: bf16 activations [m][ldx] (16-byte aligned
  // rows) quantized to MXFP8 in the kernel instead of read as xq/xs; null: TMA.
  const uint16_t* x_bf16;
  int64_t ldx;
  // Optional MXFP8 quantization of the output for the next linear (null q_out:
  // none; needs n_rows % 32 == 0): q_out [m][ldq] E4M3 and s_out [m][lds] UE8M0
  // of the values as stored in out, round to nearest even.
  uint8_t* q_out;
  int64_t ldq;
  uint8_t* s_out;
  int64_t lds;
  // Q4_K launches: the activations' group sums [m][K/32] (row stride ldsum, 16-byte aligned rows).
  const float* xsum;
  int64_t ldsum;
};

struct GemvTmMaps {
  CUtensorMap x;                         // activations [K/16 chunks][m tokens][16 bytes], box 16 x 8*NT x 16
  CUtensorMap xs;                        // activation scales [m tokens][K/32 groups], box 16 x 8*NT
  CUtensorMap xb;                        // bf16 activations [m tokens][K], box 256 x 8*NT (fused quantization)
};

// One linear of a grouped GEMV launch: independent linears (no output feeds
// another's input) with bf16 activations quantized in the kernel and
// tile-major packed weights. Units and row tiles are numbered across the
// group in item order.
struct GemvItem {
  const uint8_t* packed;
  const uint16_t* x;  // bf16 [m][ldx]
  void* out;          // [m][ldo], f32 or bf16
  int64_t ldx;
  int64_t ldo;
  int n_rows;
  int n_blocks;
  int m;
  int out_bf16;
  int unit0;  // first unit of this item in the launch's numbering
  int tile0;  // first row tile of this item in the launch's numbering
  int xt0;    // GemvGroupPre: first activation tile of this item (one per K block)
  const float* xsum;  // Q4_K groups: the activations' group sums [m][ldsum] (made by the pre-pass)
  int64_t ldsum;
  uint8_t* q_out;  // optional MXFP8 quantization of out (as GemvTmParams::q_out)
  int64_t ldq;
  uint8_t* s_out;
  int64_t lds;
};
constexpr int kGemvMaxItems = 32;
constexpr int kGemvMaxGrid = 256;  // CTAs of a grouped launch (one per SM)
struct GemvGroup {
  CUtensorMap xb[kGemvMaxItems];  // bf16 activation map of each item (box 256 x 8*NT)
  GemvItem items[kGemvMaxItems];
  int count;
  // First unit of each CTA's stream-K range (cta_start[grid] = all units):
  // ranges of about equal estimated time, not equal unit counts, since a
  // unit's cost grows with its item's token count. Strictly increasing.
  int cta_start[kGemvMaxGrid + 1];
};
// A grouped launch whose activations a pre-pass quantized (launch_group_xtiles):
// per item and K block one tile at xtiles + (items[l].xt0 + kb) * gemv_xtile_bytes(NT),
// laid out as the GEMV's activation slot needs it; the GEMV's activation warps
// only copy tiles (three bulk copies per unit) instead of quantizing every
// K block once per row tile.
struct GemvGroupPre : GemvGroup {
  const uint8_t* xtiles;
};
// Bytes of one activation tile: the B tile [16 K chunks][8*NT tokens][16 bytes]
// (E4M3), then the rows of the two scale blocks ([8*NT tokens][16 bytes] each,
// groups 0-3 / 4-7 of the K block in bytes 0-3).
__host__ __device__ constexpr uint32_t gemv_xtile_bytes(int nt) { return 288u * 8u * (uint32_t)nt; }
// The pre-pass: bf16 rows of every item -> its activation tiles, the standalone
// quantizer's arithmetic (round to nearest even). Rows past an item's M are
// left as they are (their products are never read).
struct GroupXtilesParams {
  struct Item {
    const uint16_t* x;
    int64_t ldx;
    int m;
    int n_blocks;
    int xt0;
    float* sums;  // optional (Q4_K): each 32-value group's sum of quantized values [m][ld_sums]
    int64_t ld_sums;
  } items[kGemvMaxItems];
  int count;
  int total_tiles;
  int box;  // token rows of a tile (8*NT)
  uint8_t* tiles;
};
cudaError_t launch_group_xtiles(const GroupXtilesParams& p, cudaStream_t stream);

// The single-linear launch's stand-in for GemvGroup.
struct GemvNoGroup {
  int count;
};
// Row-split tensor-parallel linear with its all-reduce in the same launch (the
// third policy type of the GEMV, in place of GemvGroup / GemvNoGroup). Every
// rank's exchange buffer, mapped into this process (base[rank] is this rank's
// own): [2 launch parities][world source ranks][max_rows][tokens] 8-byte words
// {FP32 partial, launch tag}, then at ctl_offset {epoch, CTAs done}.
constexpr int kGemvArMaxRanks = 8;
struct GemvAr {
  uint8_t* base[kGemvArMaxRanks];
  int world, rank;
  int max_rows;  // rows of a source rank's partial slot (a multiple of 128)
  uint32_t ctl_offset;
};
// Byte size of one rank's exchange slots (up to 32 tokens).
__host__ __device__ inline size_t gemv_ar_slot_bytes(int world, int max_rows) {
  return (size_t)2 * world * max_rows * 32 * 8;
}
cudaError_t launch_gemv_tm_ar(const GemvTmParams& p, const GemvAr& ar, int nt, const GemvTmMaps& maps, int grid,
                              cudaStream_t stream);
// Grouped launch (stream-K over the concatenated units of every item).
cudaError_t launch_gemv_tm_group(const GemvTmParams& p, const GemvGroup& g, int nt, int dec_warps, int grid,
                                 cudaStream_t stream);
cudaError_t launch_gemv_tm_group_pre(const GemvTmParams& p, const GemvGroupPre& g, int nt, int grid,
                                     cudaStream_t stream, bool q4k = false);

// Activation map for the tcgen05 GEMV; false when xq is not 16-byte aligned
// with a row stride that is a multiple of 16.
bool make_gemv_x_map(const uint8_t* xq, int64_t ldxq, int m, int n_blocks, int box_tokens, CUtensorMap* map);
// Scale map for the tcgen05 GEMV; false unless xs is 16-byte aligned with a row stride that is a multiple of 16.
bool make_gemv_xs_map(const uint8_t* xs, int64_t ldxs, int m, int n_blocks, int box_tokens, CUtensorMap* map);
cudaError_t launch_gemv_tm(const GemvTmParams& p, int nt, int dec_warps, const GemvTmMaps& maps, int grid,
                           cudaStream_t stream, bool q4k = false);
// Shared memory of the Q4_K GEMV (no codebook, 18,432-byte records).
uint32_t q4k_gemv_smem_bytes(int nt, int stages, int kparts);
uint32_t gemv_tm_smem_bytes(int nt, int stages, int kparts, bool fused = false, bool q4k = false);
// bf16 activation map for the GEMV's fused quantization; false unless x is
// 16-byte aligned with a row stride (elements) that is a multiple of 8.
bool make_gemv_xb_map(const uint16_t* x, int64_t ldx, int m, int64_t k, int box_tokens, CUtensorMap* map);
// Clusters of `kparts` CTAs of this configuration that can be resident at once (0 if none / on error).
int gemv_tm_max_clusters(int nt, int dec_warps, int stages, int kparts, bool q4k = false);
int gemv_tm_max_stages();

// tcgen05 GEMM for prefill-sized M (128 weight rows x 128 tokens per tile).
struct GemmTmParams {
  int m;  // tokens
  int n_rows;
  int n_blocks;
  const uint8_t* packed;    // tile-major weight records (iq3s_pack_kernel)
  const uint8_t* xs_atoms;  // activation scales as scale-factor atoms (launch_xs_atoms)
  const uint32_t* table;    // uint32[512], E4M3-encoded magnitudes
  void* out;
  int out_bf16;
  int64_t ldo;
  int wstages;  // weight stages
  int row_tiles;
  int tok_tiles;
};
struct GemmTmMaps {
  CUtensorMap x;  // activations [m tokens][K bytes], box 128 bytes x 128 tokens, 128-byte swizzle
};
bool make_gemm_x8_map(const uint8_t* xq, int64_t ldxq, int m, int64_t k, CUtensorMap* map);
cudaError_t launch_gemm_tm(const GemmTmParams& p, const GemmTmMaps& maps, int grid, cudaStream_t stream);
uint32_t gemm_tm_smem_bytes(int wstages);
int gemm_tm_max_wstages();
int gemm_tm_tile_tokens();
// FP16-operand GEMM (A = sign*grid*(1+2*nibble) exact in FP16, one accumulator
// per K block): activations converted to FP16 relative to a per-token power of two.
struct GemmF16Params {
  int m;
  int n_rows;
  int n_blocks;
  const uint8_t* packed;       // tile-major weight records
  const float* tok_scale;      // [m]: 2^(largest scale exponent of the token)
  const uint32_t* table;       // uint32[512], E4M3-encoded magnitudes
  void* out;
  int out_bf16;
  int64_t ldo;
  int wstages;
  int row_tiles;
  int tok_tiles;
  int out_tma;  // 1: bf16 output tiles staged in shared memory and written by a TMA store
  // K split (single CTAs only): each (row tile, token tile) is split into
  // ksplit contiguous K ranges taken by different CTAs. Each epilogue warp
  // publishes its FP32 partial [ksplit][32 token quads][128 rows][4] per tile
  // and counts in on split_counters[tile * 8 + warp] (zero between launches);
  // the last of the ksplit contributors sums them in K order and stores.
  int ksplit;                  // 1 = no split
  float* partials;             // [out tiles][ksplit][128 x 128] FP32
  int* split_counters;         // [out tiles][8], zero on entry and left zero
  // Folded kernel (MAMBO_KERNEL_GEMM_F16_FOLD): per-row exponents e (rows of
  // whole tiles); the weight operand is fp16(d * 2^-e * (1+2*nibble)) * grid,
  // one accumulator covers the whole K range, out = D * 2^e * tok_scale.
  const int8_t* row_exp;
};
// Per-row exponents for the folded FP16 GEMM (the tail of the packed buffer):
// row_exp[r] = floor(log2(max_b |d_b|)) over row r's finite block scales.
cudaError_t launch_iq3s_row_exp(const uint8_t* d, int64_t n_rows, int64_t n_blocks, int8_t* row_exp,
                                cudaStream_t stream);
struct GemmF16Maps {
  CUtensorMap x16;  // FP16 activations [m tokens][K], box 64 halves x 128 tokens, 128-byte swizzle
  CUtensorMap out;  // bf16 output [m][ldo] (with out_tma), box 128 rows x 128 tokens
};
cudaError_t launch_gemm_f16(const GemmF16Params& p, const GemmF16Maps& maps, int grid, cudaStream_t stream,
                            bool fold = false);
uint32_t gemm_f16_smem_bytes(int wstages, bool out_stage = false);
// bf16 output map for the FP16 GEMM's TMA stores; false unless out is 16-byte aligned with ldo % 8 == 0.
bool make_gemm_out_map(void* out, int64_t ldo, int n_rows, int m, CUtensorMap* map);
int gemm_f16_max_wstages();
// MXFP8 activations -> FP16 x16[m][k] (row stride ld halves) = E4M3 * 2^(e_group - e_max(token)),
// tok_scale[m] = 2^(e_max - 127). Exact while a group's exponent is within 12 of the token's largest.
cudaError_t launch_x16(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int m, int64_t k,
                       uint16_t* x16, int64_t ld, float* tok_scale, cudaStream_t stream);
// bf16 / f32 activations [m][k] (row stride ldx elements, 16-byte aligned rows) -> MXFP8 codes
// (round to nearest even, as mambo_quantize_mxfp8) -> the x16 / tok_scale launch_x16 forms, in one launch.
cudaError_t launch_x16_quant(const void* x, int x_dtype, int64_t ldx, int m, int64_t k, uint16_t* x16, int64_t ld,
                             float* tok_scale, cudaStream_t stream);
size_t x16_quant_smem_bytes(int64_t k);
bool make_gemm_x16_map(const uint16_t* x16, int64_t ld, int m, int64_t k, int box_tokens, CUtensorMap* map);
// CTA pairs of the FP16 GEMM that fit on the device at once, and their launch.
int gemm_f16_pair_max_clusters(int wstages, bool out_stage);
// wide: the 256 x 256-token tiles of MAMBO_KERNEL_GEMM_F16_WIDE (block scale folded).
cudaError_t launch_gemm_f16_pair(const GemmF16Params& p, const GemmF16Maps& maps, int clusters, cudaStream_t stream,
                                 bool wide = false);

// Activation scales [m][K/32] -> atoms [ceil(m/128)][K/128][32][16] (bytes: m_pad * K / 32).
cudaError_t launch_xs_atoms(const uint8_t* xs, int64_t ldxs, int m, int n_blocks, uint8_t* atoms, cudaStream_t stream);

cudaError_t launch_wait_selftest(unsigned long long limit_ns, cudaStream_t stream);
cudaError_t probe_kernel_image();

}  // namespace mambo
