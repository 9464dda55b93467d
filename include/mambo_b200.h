/*
 * mambo_b200 -- C ABI of the B200 (sm_100a) IQ3_S x MXFP8 quantized-linear path.
 *
 * Every entry point is asynchronous on the given CUDA stream, takes plain
 * device pointers and sizes, returns an int status (MAMBO_OK on success) and
 * never throws or aborts. On failure a message is kept per host thread and
 * can be read with mambo_last_error().
 *
 * Each declaration cites the reference interface it replaces (paths relative
 * to the Menooker/Mambo tree). The reference launches cuTile kernels from
 * Python through CuPy; these functions are what its launch wrappers
 * (the modules in src/python/mambo/kernels) bind to in this build.
 */
#ifndef MAMBO_B200_H
#define MAMBO_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MAMBO_API __attribute__((visibility("default")))
#else
#define MAMBO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* mambo_stream_t; /* a cudaStream_t; NULL = legacy default stream */

/* Status codes. */
enum {
  MAMBO_OK = 0,
  MAMBO_EINVAL = 1,         /* bad shape, dtype, stride or pointer (reference: ValueError / TypeError) */
  MAMBO_ENOTSUPPORTED = 2,  /* device is not sm_100 (reference: RuntimeError "no tuned config") */
  MAMBO_ECUDA = 3,          /* a CUDA runtime call failed */
  MAMBO_ETIMEOUT = 4,       /* a bounded device-side wait gave up (see mambo_device_status) */
  MAMBO_EWORKSPACE = 5      /* workspace missing or too small */
};

/* Element types of activations / outputs. */
enum { MAMBO_F32 = 0, MAMBO_BF16 = 1 };

/* Rounding of activation values to E4M3. */
enum {
  MAMBO_ROUND_NEAREST_EVEN = 0, /* cvt.rn (cuTile astype in quantize_fp8.py:37) */
  MAMBO_ROUND_TIES_DOWN = 1     /* exact ties to the smaller magnitude (fp8_reference.py:81-83) */
};

/*
 * Prepared IQ3_S weight: the byte-preserving structure-of-arrays split of
 * GGUF blocks [N, B, 110] (B = K/256), fields laid out [B, N, ...] and
 * C-contiguous. Mirrors IQ3SFields (src/python/mambo/utils/iq3_s_weight.py:10-22).
 */
typedef struct MamboIQ3SWeight {
  const void* d;      /* float16 [B, N]       block base scale           */
  const void* qs;     /* uint8   [B, N, 64]   low 8 bits of 9-bit codes  */
  const void* qh;     /* uint8   [B, N, 8]    high code bits             */
  const void* signs;  /* uint8   [B, N, 32]   one sign bit per weight    */
  const void* scales; /* uint8   [B, N, 4]    8 packed 4-bit group scales */
  int64_t n_rows;     /* N */
  int64_t n_blocks;   /* B */
  const void* packed; /* optional tile-major copy made by mambo_iq3s_pack (NULL = none): the
                         tcgen05 GEMV then fetches a work unit with one copy instead of five */
} MamboIQ3SWeight;
/* With `packed` set, qs, qh and signs may be NULL (the packed copy holds their bytes; d and
 * scales stay required): every linear entry point runs on such a weight, while
 * mambo_iq3s_decode, mambo_iq3s_pack and MAMBO_KERNEL_GEMV_SYNC return MAMBO_EINVAL. */

/* Rows per tile of the packed layout and bytes per (tile, K block) record. */
#define MAMBO_IQ3S_TILE_ROWS 128
#define MAMBO_IQ3S_RECORD_BYTES 14080

/* Launch configuration of the linear kernels (NULL = tuned default for the shape). */
typedef struct MamboLinearConfig {
  int kernel;        /* MAMBO_KERNEL_* */
  int warps;         /* GEMV: decoder warps (8, 16); GEMV_SYNC: compute warps (16 weight rows each); GEMM: 8 */
  int stages;        /* shared-memory pipeline depth (GEMV, GEMM: weight stages) */
  int ctas_per_sm;   /* GEMV_SYNC: persistent grid = SMs * ctas_per_sm (0 = 1); GEMV: 0 or 1 */
  int split;         /* GEMV: 0 = stream-K over all SMs, 1 = one CTA per row tile, 2 = K split in clusters */
  int loader;        /* GEMV_SYNC weight staging: 0 = TMA when the layout allows it, 1 = plain loads */
  int prefetch;      /* GEMV: work units whose weights are prefetched into L2 beyond the stage ring */
  int reserved;
} MamboLinearConfig;

/* Kernel kinds: GEMV = weight-streaming decode kernel on tcgen05 tensor cores
 * (the default below 32 tokens); GEMM = tcgen05 kernel over 128-row x
 * 128-token tiles (the default from 32 tokens; needs the packed weight copy
 * and 16-byte aligned activation rows); GEMV_SYNC = the weight-streaming
 * kernel on legacy mma.sync FP8 instructions, kept as a measured baseline (on
 * sm_100 its FP8 fragments go through conversions). AUTO = pick by M as the
 * reference does with LARGE_TOKEN_THRESHOLD (iq3_s_fp8.py:384-399).
 * GEMM_F16 = the large-M tcgen05 kernel with FP16 operands: the group scale
 * (1+2*nibble) folded exactly into the weight operand and one FP32 accumulator
 * per 256-wide K block; activations enter as FP16 relative to each token's
 * largest scale (exact unless a group's scale is more than 2^12 below it).
 * MAMBO_KERNEL_GEMM_F16_PAIR: the same arithmetic on clusters of two CTAs
 * whose tensor cores share each activation tile (256 weight rows per tile).
 * MAMBO_KERNEL_GEMM_F16_FOLD: the FP16 GEMM with the block scale d folded too,
 * rounded, into the weight operand (fp16(d * 2^-e * (1+2*nibble)) * grid, e a
 * per-row exponent stored with the packed copy): one accumulator covers the
 * whole K range, so no per-block epilogue; about 2^-12 relative rounding per
 * weight, within the 1e-3 relative Frobenius bound of the linear.
 * MAMBO_KERNEL_GEMM_F16_WIDE: the folded arithmetic on CTA pairs with tiles of
 * 256 weight rows x 256 tokens: each decoded weight block feeds twice the
 * tensor work of a 128-token tile (the GEMM_F16 kernels are paced by their
 * weight decoders), and each activation tile serves 256 weight rows. */
enum {
  MAMBO_KERNEL_AUTO = 0,
  MAMBO_KERNEL_GEMV = 1,
  MAMBO_KERNEL_GEMM = 2,
  MAMBO_KERNEL_GEMV_SYNC = 3,
  MAMBO_KERNEL_GEMM_F16 = 4,
  MAMBO_KERNEL_GEMM_F16_PAIR = 5,
  MAMBO_KERNEL_GEMM_F16_FOLD = 6,
  MAMBO_KERNEL_GEMM_F16_WIDE = 7
};

/* Library version string. */
MAMBO_API const char* mambo_version(void);

/* Copies the calling thread's last error message into buf (NUL-terminated). Returns its status code. */
MAMBO_API int mambo_last_error(char* buf, size_t len);

/* MAMBO_OK when the current device is sm_100 and the library's kernels load on it. */
MAMBO_API int mambo_device_check(void);

/*
 * Splits GGUF IQ3_S blocks into the SoA weight fields on the GPU.
 * raw: byte tensor [N, B, 110] with arbitrary byte strides (element stride of
 * the last dim may be > 1; any address alignment). Outputs must be
 * C-contiguous buffers of the MamboIQ3SWeight field sizes.
 * Replaces prepare_iq3_s_fields (src/python/mambo/utils/iq3_s_weight.py:25-54).
 */
MAMBO_API int mambo_iq3s_prepare(const uint8_t* raw, int64_t n_rows, int64_t n_blocks, int64_t stride_row, int64_t stride_block,
                       int64_t stride_byte, void* d, void* qs, void* qh, void* signs, void* scales,
                       mambo_stream_t stream);

/*
 * Packed weight layout (no counterpart in the reference; an addition for the
 * tcgen05 GEMV). Records of MAMBO_IQ3S_RECORD_BYTES, one per (128-row tile t,
 * K block b), at ((t * B) + b) * MAMBO_IQ3S_RECORD_BYTES, each holding the
 * tile's fields back to back, chunk-major so that consecutive rows' bytes are
 * adjacent: qs [4][128][16 B] (16-byte chunk, row), signs [2][128][16 B],
 * qh [2][128][4 B], d [128] fp16, scales [128][4 B]; rows at or past N are zero. A run of work
 * units (consecutive K blocks of one tile, then the next tile) is one
 * contiguous range. After the records, at byte tiles * B * RECORD_BYTES, one
 * int8 per row of whole tiles: floor(log2(max_b |d_b|)) over the row's finite
 * block scales (0 without one), used by MAMBO_KERNEL_GEMM_F16_FOLD.
 * mambo_iq3s_packed_bytes gives the size of the buffer and
 * mambo_iq3s_pack fills it from prepared SoA fields (N % 8 == 0; 16-byte
 * aligned fields and buffer). The SoA fields stay valid and unchanged.
 */
MAMBO_API size_t mambo_iq3s_packed_bytes(int64_t n_rows, int64_t n_blocks);
MAMBO_API int mambo_iq3s_pack(const MamboIQ3SWeight* w, void* packed, mambo_stream_t stream);

/*
 * Standalone decoder: values u8 [N, B*256] signed E4M3 bytes, scales f32 [N, B*8] = d*(1+2*nibble).
 * fp8_table: device uint32[512], the codebook with magnitudes as E4M3 bytes.
 * Replaces decode_iq3_s_blocks / launch_dequant_iq3_s (src/python/mambo/kernels/iq3_s_fp8.py:202-222,341-351).
 */
MAMBO_API int mambo_iq3s_decode(const MamboIQ3SWeight* w, const uint32_t* fp8_table, uint8_t* values, float* scales,
                      mambo_stream_t stream);

/*
 * MXFP8 activation quantization: x [M, K] (f32 or bf16, row stride ldx elements,
 * K % 32 == 0) -> q u8 [M, K] E4M3 (row stride ldq) and s u8 [M, K/32] UE8M0
 * (row stride lds). Scale exponent e = clamp(ceil(log2(amax/448)), -127, 127),
 * amax == 0 -> e = 0; q = E4M3(x * 2^-e) with the given rounding.
 * Replaces quantize_activation_fp8 / launch_quantize_fp8 (src/python/mambo/kernels/quantize_fp8.py:23-52,67-84).
 */
MAMBO_API int mambo_quantize_mxfp8(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, uint8_t* q, int64_t ldq,
                         uint8_t* s, int64_t lds, int rounding, mambo_stream_t stream);

/*
 * IQ3_S x MXFP8 linear: out[M, N] = decode_mxfp8(xq, xs) @ dequant(w).T, FP32
 * accumulation, each 32-weight group's partial product scaled by d*(1+2*nibble)
 * in FP32. xq u8 [M, K] (row stride ldxq), xs u8 [M, K/32] (row stride ldxs),
 * out f32 or bf16 [M, N] (row stride ldo). workspace: device scratch of
 * mambo_iq3s_linear_workspace_bytes() bytes, zero-filled once when it is
 * allocated (the kernels leave it zeroed again). Calls that share a workspace
 * must not overlap on the GPU.
 * Replaces iq3_s_fp8_matmul / iq3_s_fp8_matmul_medium / launch_iq3_s_fp8_matmul
 * (src/python/mambo/kernels/iq3_s_fp8.py:225-333,364-399).
 */
MAMBO_API int mambo_iq3s_linear(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int64_t m,
                      const MamboIQ3SWeight* w, const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo,
                      const MamboLinearConfig* cfg, void* workspace, size_t workspace_bytes, mambo_stream_t stream);

/*
 * Quantization + linear in one call: x bf16 or f32 [M, K] (row stride ldx)
 * -> MXFP8 (round to nearest even) -> the IQ3_S x MXFP8 linear -> out.
 * Below 32 tokens, with bf16 rows 16-byte aligned, the tcgen05 GEMV quantizes
 * the activations itself (one launch, no xq/xs round trip; the same
 * arithmetic as mambo_quantize_mxfp8, bit-identical results); otherwise the
 * quantizer runs into the workspace first. workspace:
 * mambo_iq3s_linear_fused_workspace_bytes() bytes, zero-filled once.
 * Replaces launch_quantize_fp8 + launch_iq3_s_fp8_matmul
 * (src/python/mambo/kernels/quantize_fp8.py:67-84, iq3_s_fp8.py:364-399).
 */
MAMBO_API int mambo_iq3s_linear_fused(const void* x, int x_dtype, int64_t ldx, int64_t m, const MamboIQ3SWeight* w,
                                      const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo,
                                      const MamboLinearConfig* cfg, void* workspace, size_t workspace_bytes,
                                      mambo_stream_t stream);

/* Workspace bytes mambo_iq3s_linear_fused needs for this shape and configuration. */
MAMBO_API size_t mambo_iq3s_linear_fused_workspace_bytes(int64_t m, int64_t n_rows, int64_t n_blocks,
                                                         const MamboLinearConfig* cfg);

/* One linear of a group: x [m, K] (row stride ldx, f32 or bf16) times w into
 * out [m, N] (row stride ldo, f32 or bf16). */
typedef struct MamboLinearItem {
  const void* x;
  int x_dtype;
  int64_t ldx;
  int64_t m;
  const MamboIQ3SWeight* w;
  void* out;
  int out_dtype;
  int64_t ldo;
} MamboLinearItem;

#define MAMBO_MAX_GROUP 32

/*
 * Several independent linears (no item's out overlaps another item's x or
 * weights), each as mambo_iq3s_linear_fused computes it (MXFP8 activations,
 * round to nearest even). With up to MAMBO_MAX_GROUP items, all with bf16
 * activations in 16-byte aligned rows, M < 32 and w->packed set, this is ONE
 * persistent GEMV launch over the units of every item (stream-K): the weights
 * of the next linear stream in while the previous one finishes, and the
 * per-launch set-up is paid once. Otherwise the items run one after another.
 * workspace: mambo_iq3s_linear_group_workspace_bytes() bytes, zero-filled once.
 * No reference counterpart (the reference launches one linear per call,
 * iq3_s_fp8.py:364-399).
 */
MAMBO_API int mambo_iq3s_linear_group(const MamboLinearItem* items, int count, const uint32_t* fp8_table,
                                      void* workspace, size_t workspace_bytes, mambo_stream_t stream);

/* Workspace bytes mambo_iq3s_linear_group needs for these items. */
MAMBO_API size_t mambo_iq3s_linear_group_workspace_bytes(const MamboLinearItem* items, int count);

/*
 * The linear's output quantized to MXFP8 for the next linear, as
 * mambo_quantize_mxfp8(out, round to nearest even) would give it: q E4M3
 * [M, N] (row stride ldq), s UE8M0 [M, N/32] (row stride lds). N % 32 == 0.
 */
typedef struct MamboQuantOut {
  uint8_t* q;
  int64_t ldq;
  uint8_t* s;
  int64_t lds;
} MamboQuantOut;

/*
 * mambo_iq3s_linear, mambo_iq3s_linear_fused and mambo_iq3s_linear_group that
 * also write the output's MXFP8 quantization (qout; NULL, or an entry whose q
 * is NULL, writes none). On the tcgen05 GEMV (M < 32, packed weights) the
 * epilogue forms it where each output value is final -- a warp owns 32
 * consecutive output features, one MXFP8 group per token -- so the next
 * linear takes MXFP8 activations without a quantization pass; the codes are
 * bit-identical to quantizing the stored output (bf16 or f32) separately.
 * Elsewhere the quantizer runs on out after the linear. The workspace is that
 * of the call without qout. qouts of the group: count entries.
 * Replaces the launch_quantize_fp8 call on a linear's output that the next
 * linear needs (src/python/mambo/kernels/quantize_fp8.py:42-52,67-84).
 */
MAMBO_API int mambo_iq3s_linear_q(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int64_t m,
                                  const MamboIQ3SWeight* w, const uint32_t* fp8_table, void* out, int out_dtype,
                                  int64_t ldo, const MamboQuantOut* qout, const MamboLinearConfig* cfg,
                                  void* workspace, size_t workspace_bytes, mambo_stream_t stream);
MAMBO_API int mambo_iq3s_linear_fused_q(const void* x, int x_dtype, int64_t ldx, int64_t m, const MamboIQ3SWeight* w,
                                        const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo,
                                        const MamboQuantOut* qout, const MamboLinearConfig* cfg, void* workspace,
                                        size_t workspace_bytes, mambo_stream_t stream);
MAMBO_API int mambo_iq3s_linear_group_q(const MamboLinearItem* items, const MamboQuantOut* qouts, int count,
                                        const uint32_t* fp8_table, void* workspace, size_t workspace_bytes,
                                        mambo_stream_t stream);

/* Workspace bytes mambo_iq3s_linear needs for this shape and configuration. */
MAMBO_API size_t mambo_iq3s_linear_workspace_bytes(int64_t m, int64_t n_rows, int64_t n_blocks, const MamboLinearConfig* cfg);

/* Size of the library-held scratch of mambo_iq3s_linear_noalloc (3 MiB per GPU). */
#define MAMBO_STATIC_SCRATCH_BYTES (3u * 1024u * 1024u)

/*
 * mambo_iq3s_linear for callers that cannot allocate device memory. It has no
 * counterpart in the reference, whose Python wrappers allocate freely.
 *
 * Who needs it: a plugin loaded into a host whose memory pool owns the device
 * memory (a serving engine that reserves nearly all HBM up front for its KV
 * cache, so a private cudaMalloc fails or eats into that reserve), and code that
 * has no handle to the host's allocator. Such callers cannot provide the
 * workspace that mambo_iq3s_linear takes.
 *
 * What it does instead: the split-K counters, FP32 partials and packed
 * activations live in a file-scope static device array of
 * MAMBO_STATIC_SCRATCH_BYTES. Every GPU on which the library's kernels are
 * loaded holds that array until the process exits. Nothing is allocated:
 * no cudaMalloc, no cudaFree, no allocating library routine.
 *
 * Arguments and results: the same as mambo_iq3s_linear without the workspace.
 * It runs the tcgen05 GEMV only (cfg NULL or kernel MAMBO_KERNEL_GEMV or AUTO;
 * N % 8 == 0; 16-byte aligned weight fields) and processes M in chunks of
 * 8 tokens.
 *
 * Limits: N <= 524288 and K <= 98304 (K/256 <= 384). Larger shapes return
 * MAMBO_EINVAL, and mambo_last_error names the limit.
 *
 * Set-up: the first call on each device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current). Make that first call
 * before any stream capture: a first call made while `stream` is capturing
 * returns MAMBO_EINVAL and launches nothing.
 *
 * Zeroing: each call clears the split-K counters it uses, with
 * cudaMemsetAsync on `stream`, before launching its kernels.
 *
 * Concurrency: all calls on one device share the array. Calls that overlap on
 * the GPU (different streams, or graphs replayed concurrently) race and give
 * wrong results; order them on one stream.
 */
MAMBO_API int mambo_iq3s_linear_noalloc(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int64_t m,
                              const MamboIQ3SWeight* w, const uint32_t* fp8_table, void* out, int out_dtype,
                              int64_t ldo, const MamboLinearConfig* cfg, mambo_stream_t stream);

/*
 * Q4_K x MXFP8 linear (GGUF type Q4_K; no counterpart kernel in the reference,
 * which lists the type in its tensor-type table,
 * src/python/mambo/utils/gguf_manifest.py:30-42, and decodes it only through
 * gguf-py). A Q4_K block holds 256 weights in 144 bytes: fp16 d, fp16 dmin, 12
 * bytes of eight 6-bit scales s_g and mins m_g, 128 bytes of 4-bit codes q;
 * weight = d*s_g*q - dmin*m_g = (d*s_g/2)*(2q - 15) + (7.5*d*s_g - dmin*m_g).
 * The odd integers 2q - 15 (-15..15) are exact E4M3 operands of the tensor
 * cores; per 32-weight group g the FP32 epilogue adds d*s_g/2 times the
 * group's partial product and the constant term times the token's sum of the
 * group's (quantized) activations.
 *
 * Packed layout: one record of MAMBO_Q4K_RECORD_BYTES per (128-row tile t,
 * K block b) at ((t * B) + b) * MAMBO_Q4K_RECORD_BYTES: codes [8 chunks][128
 * rows][16 B], then [128 rows][4 B] d and dmin, then [128 rows][12 B] scales
 * and mins; rows at or past N are zero. Chunk c holds code bytes 16c..16c+15
 * of the row's block as four 32-bit words: the word of bytes b0..b3 carries
 * their low nibbles in bits 0-15 and their high nibbles in bits 16-31 (value j
 * of a half in bits 4j..4j+3), each re-coded as (q >= 8 ? q : 7 - q), the sign
 * and magnitude index of 2q - 15. mambo_q4k_pack fills it from raw blocks [N, B, 144] with any
 * byte strides (any alignment); the packed buffer must be 16-byte aligned.
 */
#define MAMBO_Q4K_BLOCK_BYTES 144
#define MAMBO_Q4K_RECORD_BYTES 18432
MAMBO_API size_t mambo_q4k_packed_bytes(int64_t n_rows, int64_t n_blocks);
MAMBO_API int mambo_q4k_pack(const uint8_t* raw, int64_t n_rows, int64_t n_blocks, int64_t stride_row,
                             int64_t stride_block, int64_t stride_byte, void* packed, mambo_stream_t stream);

/*
 * mambo_quantize_mxfp8 that also writes, per 32-value group, the sum of its
 * quantized values E4M3(q) * 2^e as FP32 (sums [M, K/32], row stride ld_sums):
 * exact, since 32 E4M3 values sum to at most 23 significant bits. A group with
 * scale code 0xFF (NaN or infinity among its values) gets a NaN sum.
 */
MAMBO_API int mambo_quantize_mxfp8_sums(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, uint8_t* q,
                                        int64_t ldq, uint8_t* s, int64_t lds, float* sums, int64_t ld_sums,
                                        int rounding, mambo_stream_t stream);

/*
 * out[M, N] = decode_mxfp8(xq, xs) @ dequant_q4k(w).T with FP32 accumulation.
 * xq, xs as for mambo_iq3s_linear; xsum: the group sums of the same quantized
 * activations (mambo_quantize_mxfp8_sums), 16-byte aligned, row stride ldsum a
 * multiple of 4. packed: the mambo_q4k_pack buffer of an [N, K] weight (B =
 * K/256 blocks per row). cfg: NULL, or MAMBO_KERNEL_GEMV / AUTO with warps 0
 * or 8, split 0 (stream-K); stages and prefetch are tunable. The tcgen05 GEMV
 * runs in chunks of 32 tokens. workspace: mambo_q4k_linear_workspace_bytes()
 * bytes, zero-filled once (the kernels leave it zeroed again).
 */
MAMBO_API size_t mambo_q4k_linear_workspace_bytes(int64_t m, int64_t n_rows, int64_t n_blocks,
                                                  const MamboLinearConfig* cfg);
MAMBO_API int mambo_q4k_linear(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, const float* xsum,
                               int64_t ldsum, int64_t m, const void* packed, int64_t n_rows, int64_t n_blocks,
                               void* out, int out_dtype, int64_t ldo, const MamboLinearConfig* cfg, void* workspace,
                               size_t workspace_bytes, mambo_stream_t stream);
/* Quantization (round to nearest even, with group sums) into the workspace, then mambo_q4k_linear. */
MAMBO_API size_t mambo_q4k_linear_fused_workspace_bytes(int64_t m, int64_t n_rows, int64_t n_blocks,
                                                        const MamboLinearConfig* cfg);
MAMBO_API int mambo_q4k_linear_fused(const void* x, int x_dtype, int64_t ldx, int64_t m, const void* packed,
                                     int64_t n_rows, int64_t n_blocks, void* out, int out_dtype, int64_t ldo,
                                     const MamboLinearConfig* cfg, void* workspace, size_t workspace_bytes,
                                     mambo_stream_t stream);

/*
 * Several independent Q4_K linears in one call (no counterpart in the reference, whose linears
 * run one per call): out_i[M_i, N_i] = linear(x_i, packed_i) as mambo_q4k_linear_fused computes
 * it. When every item has bf16 activations in 16-byte aligned rows, 1 <= M < 32 and N % 8 == 0,
 * a pre-pass quantizes all items' activations once (MXFP8 codes and group sums) and one
 * persistent GEMV launch streams all items' packed records; otherwise the items run one after
 * another through mambo_q4k_linear_fused. workspace: mambo_q4k_linear_group_workspace_bytes(),
 * zero-filled once. No output may overlap another item's input.
 */
typedef struct MamboQ4KItem {
  const void* x;      /* activations [m, K], bf16 or f32 (x_dtype), row stride ldx */
  int x_dtype;
  int64_t ldx;
  int64_t m;
  const void* packed; /* mambo_q4k_pack buffer of the [n_rows, K] weight, K = 256 * n_blocks */
  int64_t n_rows;
  int64_t n_blocks;
  void* out;          /* [m, n_rows], out_dtype, row stride ldo */
  int out_dtype;
  int64_t ldo;
} MamboQ4KItem;
MAMBO_API size_t mambo_q4k_linear_group_workspace_bytes(const MamboQ4KItem* items, int count);
MAMBO_API int mambo_q4k_linear_group(const MamboQ4KItem* items, int count, void* workspace, size_t workspace_bytes,
                                     mambo_stream_t stream);

/* Number of tunable configurations of a kernel kind, and the i-th one (for the autotuner).
 * Replaces the search spaces of make_benchmark_cases (src/python/mambo/kernels/iq3_s_fp8.py:402-465). */
MAMBO_API int mambo_num_configs(int kernel);
MAMBO_API int mambo_config_at(int kernel, int index, MamboLinearConfig* cfg);

/* Tuned default configuration for a shape (what NULL cfg resolves to). */
MAMBO_API int mambo_default_config(int64_t m, int64_t n_rows, int64_t n_blocks, MamboLinearConfig* cfg);

/*
 * Device-side failure channel (no counterpart in the reference, whose kernels
 * have no waits). Every wait of the pipelined kernels is bounded: when one
 * gives up it records MAMBO_ETIMEOUT with a site id and returns instead of
 * hanging. mambo_device_status reads (and with reset != 0 clears) that record;
 * it synchronizes with the device.
 */
MAMBO_API int mambo_device_status(int reset, int* code, int* where, int* block);
/* Wall-clock limit of one bounded device wait (default 1 s). */
MAMBO_API int mambo_set_wait_limit_ns(unsigned long long ns);
/* Launches a kernel whose bounded wait on a barrier nothing completes gives up
 * after limit_ns; afterwards mambo_device_status reports MAMBO_ETIMEOUT. */
MAMBO_API int mambo_selftest_wait_timeout(unsigned long long limit_ns, mambo_stream_t stream);

/*
 * Tensor-parallel row split with its all-reduce in the same launch (no
 * counterpart in the reference, which runs every linear on one GPU). Each of
 * `world` ranks (one process per GPU, up to 8) holds a K slice of the weight;
 * the GEMV that multiplies it writes each row tile's partial straight into
 * every rank's exchange buffer over NVLink (plain peer stores, no multicast;
 * each value shares an 8-byte word with the call's tag, so no fence or flag is
 * needed), waits (bounded, MAMBO_ETIMEOUT) for every rank's partial of the
 * same rows and sums them in rank order: every rank gets the identical [m, N]
 * result, with no separate collective launch. This replaces
 * the GEMV + NCCL all-reduce pair of a row split (the O and down projections
 * of a tensor-parallel layer) at decode sizes.
 *
 * mambo_ar_comm_create allocates this rank's exchange buffer on the current
 * device (slots for up to max_rows output rows, a multiple of 128 up to 2^18,
 * and 32 tokens: 512 * world * max_rows bytes) and writes its CUDA IPC handle
 * (MAMBO_AR_HANDLE_BYTES bytes) to ipc_handle. The caller exchanges the
 * handles between the ranks (e.g. an all-gather over its process group) and
 * passes all of them, in rank order, to mambo_ar_comm_connect. Every rank
 * must then make the same sequence of mambo_iq3s_linear_fused_ar calls on a
 * communicator (same M, N and configuration): each call's epoch pairs it with
 * the peers' matching call. Calls on one communicator must not overlap on the
 * GPU (issue them on one stream).
 */
typedef struct MamboArComm MamboArComm;
#define MAMBO_AR_HANDLE_BYTES 64
MAMBO_API int mambo_ar_comm_create(int world, int rank, int64_t max_rows, MamboArComm** comm, void* ipc_handle);
MAMBO_API int mambo_ar_comm_connect(MamboArComm* comm, const void* ipc_handles);
MAMBO_API int mambo_ar_comm_destroy(MamboArComm* comm);
/* This rank's slice: x [m, K/world] (bf16, 16-byte aligned rows, m < 32) times
 * its weight shard w [N, K/world] -> out [m, N] (f32 or bf16), the sum over
 * all ranks. workspace: mambo_iq3s_linear_fused_workspace_bytes() bytes. */
MAMBO_API int mambo_iq3s_linear_fused_ar(const void* x, int x_dtype, int64_t ldx, int64_t m, const MamboIQ3SWeight* w,
                                         const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo,
                                         MamboArComm* comm, const MamboLinearConfig* cfg, void* workspace,
                                         size_t workspace_bytes, mambo_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MAMBO_B200_H */
