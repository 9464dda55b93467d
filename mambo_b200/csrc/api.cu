// C ABI of libmambo_b200 (declared in include/mambo_b200.h).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <string>

#include "kernels.cuh"

namespace mambo {

__device__ DeviceStatus g_device_status = {0, 0, 0, 0};
__device__ unsigned long long g_wait_limit_ns = 1000000000ull;  // 1 s

cudaError_t ensure_smem_attribute(const void* kernel, size_t smem_bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(kernel, dev);
  auto it = done.find(key);
  if (it != done.end() && it->second >= smem_bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes);
  if (e == cudaSuccess) done[key] = smem_bytes;
  return e;
}

// Trivial kernel: its attributes tell whether this library's sm_100a image loads on the device.
__global__ void probe_kernel() {}
cudaError_t probe_kernel_image() {
  cudaFuncAttributes attr;
  return cudaFuncGetAttributes(&attr, probe_kernel);
}

// Waits on an mbarrier that nothing arrives at: the bounded wait must give up
// after limit_ns, record MAMBO_ETIMEOUT in the device status and return.
__global__ void wait_selftest_kernel(unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t addr = smem_u32(&bar);
    const unsigned long long t0 = globaltimer_ns();
    bool done = false;
    for (uint32_t i = 1; !done; ++i) {
      done = mbar_try_wait(addr, 0);
      if (!done && (i & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) {
        record_timeout(kSiteSelfTest);
        break;
      }
    }
    // Complete the phase ourselves so the barrier is not left pending.
    mbar_arrive(addr);
  }
}

cudaError_t launch_wait_selftest(unsigned long long limit_ns, cudaStream_t stream) {
  wait_selftest_kernel<<<1, 32, 0, stream>>>(limit_ns);
  return cudaGetLastError();
}

}  // namespace mambo

using namespace mambo;

namespace {

thread_local std::string g_last_error;
thread_local int g_last_code = MAMBO_OK;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  g_last_code = code;
  return code;
}

int ok() {
  g_last_code = MAMBO_OK;
  return MAMBO_OK;
}

int cuda_fail(cudaError_t e, const char* what) {
  if (e == cudaErrorNoKernelImageForDevice || e == cudaErrorInvalidDeviceFunction)
    return fail(MAMBO_ENOTSUPPORTED, "%s: %s (this library is built for sm_100a only)", what, cudaGetErrorString(e));
  return fail(MAMBO_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct DeviceInfo {
  int sms = 0;
  int major = 0, minor = 0;
  int max_smem_optin = 0;
  int smem_per_sm = 0;
};

DeviceInfo device_info(int* status) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  static bool have[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    *status = cuda_fail(e == cudaSuccess ? cudaErrorInvalidDevice : e, "cudaGetDevice");
    return DeviceInfo{};
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!have[dev]) {
    DeviceInfo d;
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cache[dev] = d;
    have[dev] = true;
  }
  *status = MAMBO_OK;
  return cache[dev];
}

int require_sm100(DeviceInfo* info) {
  int st;
  *info = device_info(&st);
  if (st != MAMBO_OK) return st;
  if (info->major != 10 || info->minor != 0)
    return fail(MAMBO_ENOTSUPPORTED, "IQ3_S FP8 kernels have no build for sm%d%d (this library targets sm_100a)",
                info->major, info->minor);
  return MAMBO_OK;
}

// --- configurations ---------------------------------------------------------
// tcgen05 GEMV (MAMBO_KERNEL_GEMV): {decoder warps, stages, prefetch}, each with split 0 and 1.
struct TcChoice {
  int warps, stages, prefetch;
};
const TcChoice kTcChoices[] = {
    {8, 3, 0}, {8, 4, 0}, {8, 4, 4}, {8, 6, 0}, {8, 6, 4}, {8, 8, 4},
    {16, 3, 0}, {16, 4, 0}, {16, 4, 4}, {16, 6, 0}, {16, 6, 4}, {16, 8, 4},
};
// split 0 (stream-K), 1 (row tile per CTA) and 2 (cluster K split) for each choice.
constexpr int kNumTcConfigs = 3 * (int)(sizeof(kTcChoices) / sizeof(kTcChoices[0]));
// mma.sync GEMV (MAMBO_KERNEL_GEMV_SYNC): warps x stages x split.
const int kSyncWarps[] = {4, 8, 12, 16};
const int kSyncStages[] = {3, 4, 6, 8};
constexpr int kNumSyncConfigs = 4 * 4 * 2;

int gemv_nt_for(int64_t m) { return m <= 8 ? 1 : (m <= 16 ? 2 : 4); }

// Shared memory an SM offers one CTA (B200: 227 KB); used when no device is visible.
constexpr int kSmemOptinDefault = 232448;

int kernel_of(const MamboLinearConfig& c) { return c.kernel == MAMBO_KERNEL_AUTO ? MAMBO_KERNEL_GEMV : c.kernel; }
// All five SoA fields are present.
bool has_soa(const MamboIQ3SWeight* w) { return w->d && w->qs && w->qh && w->signs && w->scales; }
// A weight the linears can use: d and scales, and either the packed copy (the
// tcgen05 kernels read only it) or the remaining SoA fields.
bool weight_fields_ok(const MamboIQ3SWeight* w) {
  return w->d && w->scales && (w->packed || (w->qs && w->qh && w->signs));
}
// The FP16-operand GEMM, on single CTAs or on CTA pairs.
bool is_gemm_f16(int kind) {
  return kind == MAMBO_KERNEL_GEMM_F16 || kind == MAMBO_KERNEL_GEMM_F16_PAIR || kind == MAMBO_KERNEL_GEMM_F16_FOLD ||
         kind == MAMBO_KERNEL_GEMM_F16_WIDE;
}
// FP16 GEMM kinds that run on single CTAs and take a K split.
bool is_gemm_f16_single(int kind) { return kind == MAMBO_KERNEL_GEMM_F16 || kind == MAMBO_KERNEL_GEMM_F16_FOLD; }
bool is_gemm(int kind) { return kind == MAMBO_KERNEL_GEMM || is_gemm_f16(kind); }

// Shared memory of a configuration (for MAMBO_KERNEL_GEMV without the cluster
// partials, which the plan sizes to what is left).
uint32_t config_smem(const MamboLinearConfig& c, int nt, int64_t b) {
  if (kernel_of(c) == MAMBO_KERNEL_GEMV_SYNC) return gemv_smem_bytes_host(c.warps * 16, nt, c.stages, (int)b);
  if (kernel_of(c) == MAMBO_KERNEL_GEMM) return gemm_tm_smem_bytes(c.stages);
  if (is_gemm_f16(kernel_of(c))) return gemm_f16_smem_bytes(c.stages);
  return gemv_tm_smem_bytes(nt, c.stages, 1);
}

// Prefill-sized M (the reference's large-token path, LARGE_TOKEN_THRESHOLD):
// the tcgen05 GEMM over 128 x 128 tiles.
constexpr int64_t kGemmMinTokens = 32;
// Weight stages of the GEMM configurations, and the FP16 GEMM's K splits
// (its search space is stages x splits; the other GEMMs search stages only).
const int kGemmStages[] = {2, 3, 4};
constexpr int kNumGemmConfigs = (int)(sizeof(kGemmStages) / sizeof(kGemmStages[0]));
const int kGemmSplits[] = {1, 2, 3, 4, 6, 8};
constexpr int kNumGemmF16Configs = kNumGemmConfigs * (int)(sizeof(kGemmSplits) / sizeof(kGemmSplits[0]));

// Split-K counters live at the start of every workspace: 64 Ki ints, zero
// between calls, a fixed region so that a call never finds another shape's
// partials there. Shapes needing more are rejected.
constexpr size_t kCounterBytes = 256 * 1024;
// The first half holds the GEMVs' counters (4 per 128-row tile), the second
// the FP16 GEMM's K-split counters (8 per output tile).
constexpr size_t kGemvCounterBytes = 128 * 1024;
constexpr size_t kGemmSplitCounterOffset = kGemvCounterBytes;
constexpr size_t kGemmSplitCounterBytes = kCounterBytes - kGemmSplitCounterOffset;
constexpr int kGemmMaxSplit = 8;

int gemm_f16_default_split(int64_t m, int64_t n, int64_t b, int sms);
int gemm_f16_clamp_split(int split, int64_t m, int64_t n, int64_t b);

void default_config(int64_t m, int64_t n, int64_t b, MamboLinearConfig* cfg, int smem_optin, int sms) {
  std::memset(cfg, 0, sizeof(*cfg));
  if (m >= kGemmMinTokens) {
    cfg->kernel = MAMBO_KERNEL_GEMM_F16;
    cfg->warps = 8;
    cfg->ctas_per_sm = 1;
    cfg->stages = 4;
    cfg->split = gemm_f16_default_split(m, n, b, sms > 0 ? sms : 148);
    while (cfg->stages > 2 && (int)config_smem(*cfg, 4, b) > smem_optin) --cfg->stages;
    return;
  }
  cfg->kernel = MAMBO_KERNEL_GEMV;
  cfg->warps = 8;
  cfg->ctas_per_sm = 1;
  // Cluster K-split while every row tile gets its own CTAs; stream-K beyond that.
  cfg->split = (n + 127) / 128 <= (sms > 0 ? sms : 148) ? 2 : 0;
  cfg->prefetch = 4;
  // Deepest weight-stage ring (up to 8) that fits next to the codebook.
  const int nt = gemv_nt_for(m < 32 ? m : 32);
  cfg->stages = 8;
  while (cfg->stages > 2 && (int)config_smem(*cfg, nt, b) > smem_optin) --cfg->stages;
}

// AUTO resolved for a shape: the kernel by M, and unset fields from the
// tuned default (a GEMM also takes the default K split when split is 0).
void resolve_auto(MamboLinearConfig* c, int64_t m, int64_t n, int64_t b, int smem_optin, int sms) {
  if (c->kernel != MAMBO_KERNEL_AUTO) return;
  MamboLinearConfig a;
  default_config(m, n, b, &a, smem_optin, sms);
  c->kernel = a.kernel;
  if (c->stages == 0) c->stages = a.stages;
  if (is_gemm(a.kernel) && c->split == 0) c->split = a.split;
}

int validate_config(const MamboLinearConfig* cfg, int64_t m, int64_t b, const DeviceInfo& info) {
  const int kind = kernel_of(*cfg);
  if (kind != MAMBO_KERNEL_GEMV && kind != MAMBO_KERNEL_GEMV_SYNC && !is_gemm(kind))
    return fail(MAMBO_EINVAL, "unknown kernel kind %d", cfg->kernel);
  if (is_gemm(kind)) {
    const int smax = kind == MAMBO_KERNEL_GEMM ? gemm_tm_max_wstages() : gemm_f16_max_wstages();
    if (cfg->stages < 2 || cfg->stages > smax) return fail(MAMBO_EINVAL, "stages must be in [2, %d]", smax);
    const int smax_split = is_gemm_f16_single(kind) ? kGemmMaxSplit : 1;
    if (cfg->split < 0 || cfg->split > smax_split)
      return fail(MAMBO_EINVAL, "split (K parts) must be in [0, %d] for this kernel", smax_split);
  } else if (kind == MAMBO_KERNEL_GEMV_SYNC) {
    if (cfg->warps != 4 && cfg->warps != 8 && cfg->warps != 12 && cfg->warps != 16)
      return fail(MAMBO_EINVAL, "warps must be 4, 8, 12 or 16");
    if (cfg->stages < 2 || cfg->stages > 12) return fail(MAMBO_EINVAL, "stages must be in [2, 12]");
  } else {
    if (cfg->stages < 2 || cfg->stages > gemv_tm_max_stages())
      return fail(MAMBO_EINVAL, "stages must be in [2, %d]", gemv_tm_max_stages());
    if (cfg->warps != 8 && cfg->warps != 16) return fail(MAMBO_EINVAL, "decoder warps must be 8 or 16");
    if (cfg->ctas_per_sm < 0 || cfg->ctas_per_sm > 1) return fail(MAMBO_EINVAL, "ctas_per_sm must be 0 or 1");
    if (cfg->prefetch < 0 || cfg->prefetch > 64) return fail(MAMBO_EINVAL, "prefetch must be in [0, 64]");
    if (cfg->split < 0 || cfg->split > 2) return fail(MAMBO_EINVAL, "split must be 0 (stream-K), 1 (row tile per CTA) or 2 (cluster K-split)");
  }
  const uint32_t smem = config_smem(*cfg, gemv_nt_for(m), b);
  if ((int)smem > info.max_smem_optin)
    return fail(MAMBO_EINVAL, "configuration needs %u bytes of shared memory (device allows %d)", smem,
                info.max_smem_optin);
  return MAMBO_OK;
}


struct GemvPlan {
  int nt, rows, row_tiles, units, grid, counter_slots, kparts;
  size_t counters_bytes, partial_bytes, xcopy_bytes, xscopy_bytes;
};

size_t align256(size_t v) { return (v + 255) / 256 * 256; }
// Row stride of activation scales copied for the TMA (a multiple of 16 bytes).
int64_t xs_copy_stride(int64_t n_blocks) { return (n_blocks * 8 + 15) / 16 * 16; }

// K parts per row tile for the cluster K-split: as many as leave every row
// tile its own cluster on the SMs (at most 8, the portable cluster size, and
// one K block each), within shared memory, and with every cluster resident at
// once.
// q4k: the Q4_K variant of the kernel (its own shared-memory size).
int cluster_kparts(int row_tiles, int64_t b, const MamboLinearConfig& cfg, int nt, int sms, int smem_optin,
                   bool q4k = false) {
  int kp = row_tiles > 0 ? sms / row_tiles : 1;
  kp = kp < 1 ? 1 : kp > 8 ? 8 : kp;
  if (kp > b) kp = (int)b;
  auto smem = [&](int k) { return q4k ? q4k_gemv_smem_bytes(nt, cfg.stages, k) : gemv_tm_smem_bytes(nt, cfg.stages, k); };
  while (kp > 1 && (int)smem(kp) > smem_optin) --kp;
  while (kp > 1 && gemv_tm_max_clusters(nt, cfg.warps, cfg.stages, kp, q4k) < row_tiles) --kp;
  return kp;
}

// The GEMM's activation scales in scale-factor atom layout, 1 KB per
// (128-token tile, K block), after the split-K counters: those must stay zero
// for the GEMV calls that share the workspace.
size_t gemm_workspace_bytes(int64_t m, int64_t b) {
  const int64_t tok = gemm_tm_tile_tokens();
  return kCounterBytes + align256((size_t)((m + tok - 1) / tok) * (size_t)b * 1024);
}

// Output tiles of the FP16 GEMM, and the K split it can take: at most
// kGemmMaxSplit parts, every part at least 4 K blocks, counters for every tile.
int64_t gemm_f16_out_tiles(int64_t m, int64_t n) { return ((n + 127) / 128) * ((m + 127) / 128); }
int gemm_f16_clamp_split(int split, int64_t m, int64_t n, int64_t b) {
  int ks = split < 1 ? 1 : split > kGemmMaxSplit ? kGemmMaxSplit : split;
  while (ks > 1 && b / ks < 4) --ks;
  if (ks > 1 && (size_t)gemm_f16_out_tiles(m, n) * 8 * sizeof(int) > kGemmSplitCounterBytes) ks = 1;
  return ks;
}

// The K split the FP16 GEMM takes by default: only when the output tiles
// leave SMs idle, the most parts (up to 4, at least 8 K blocks each) that
// still run as one wave of work items. Measured on B200: splitting a launch
// that already fills the SMs costs more in partials and per-item pipeline
// fill than it gains in balance (Llama-3-8B down at 2048 tokens, 512 tiles:
// 308 -> 349 us with two parts), while 64 tiles at 64 tokens gain (Llama-3-70B
// O: 52 -> 41 us with two parts). The autotuner searches up to 8 parts.
int gemm_f16_default_split(int64_t m, int64_t n, int64_t b, int sms) {
  const int64_t tiles = gemm_f16_out_tiles(m, n);
  int ks = 1;
  for (int k = 2; k <= 4; ++k)
    if (tiles * k <= sms && b / k >= 8 && gemm_f16_clamp_split(k, m, n, b) == k) ks = k;
  return ks;
}

// The FP16 GEMM's workspace: the counter region (the GEMVs' counters left
// zero, the K-split counters), the FP16 activations [m][K], the tokens'
// scales (padded to whole 256-token tiles: the epilogue reads them 16 at a
// time, the wide GEMM's tiles are 256 tokens) and, with a K split, the FP32
// partials of every output tile.
size_t gemm_f16_tok_scale_bytes(int64_t m) { return align256((size_t)((m + 255) / 256 * 256) * 4); }
size_t gemm_f16_partial_bytes(int64_t m, int64_t n, int ks) {
  return ks > 1 ? align256((size_t)gemm_f16_out_tiles(m, n) * ks * 128 * 128 * sizeof(float)) : 0;
}
size_t gemm_f16_workspace_bytes(int64_t m, int64_t n, int64_t b, int ks) {
  return kCounterBytes + align256((size_t)m * (size_t)b * 256 * 2) + gemm_f16_tok_scale_bytes(m) +
         gemm_f16_partial_bytes(m, n, ks);
}

// The GEMM reads activations through a TMA map (16-byte aligned rows) and
// weights from the tile-major packed copy.
bool gemm_usable(const MamboIQ3SWeight* w, const uint8_t* xq, int64_t ldxq, int64_t m) {
  return w->packed != nullptr && w->n_rows % 8 == 0 && (uintptr_t)xq % 16 == 0 && ldxq % 16 == 0 &&
         m <= (int64_t)1 << 30;
}

GemvPlan plan_gemv(int64_t m_chunk, int64_t n, int64_t b, const MamboLinearConfig& cfg, int sms, int smem_optin,
                   bool q4k = false) {
  GemvPlan P{};
  const bool tc = kernel_of(cfg) == MAMBO_KERNEL_GEMV;
  P.nt = gemv_nt_for(m_chunk);
  P.rows = tc ? 128 : cfg.warps * 16;
  P.row_tiles = (int)((n + P.rows - 1) / P.rows);
  P.units = (int)(P.row_tiles * b);
  P.counter_slots = P.row_tiles * (tc ? 4 : cfg.warps);
  P.counters_bytes = kCounterBytes;
  if (tc && cfg.split != 0) {
    // Whole row tiles (split 1) or row tiles split over the CTAs of a cluster (split 2).
    P.kparts = cfg.split == 2 ? cluster_kparts(P.row_tiles, b, cfg, P.nt, sms, smem_optin, q4k) : 1;
    P.grid = P.row_tiles * P.kparts;
  } else {
    int ctas = sms * (!tc && cfg.ctas_per_sm > 0 ? cfg.ctas_per_sm : 1);
    if (cfg.split == 1) ctas = P.row_tiles;  // one CTA per row tile, no split-K
    P.grid = P.units < ctas ? P.units : ctas;
    if (P.grid < 1) P.grid = 1;
    P.partial_bytes = align256((size_t)P.grid * 2 * P.rows * 8 * P.nt * sizeof(float));
  }
  // Activations whose rows are not 16-byte aligned are copied here for the TMA.
  P.xcopy_bytes = tc ? align256((size_t)m_chunk * b * 256) : 0;
  P.xscopy_bytes = tc ? align256((size_t)m_chunk * xs_copy_stride(b)) : 0;
  return P;
}

// The tcgen05 GEMM: activation scales to scale-factor atoms (workspace), then
// one persistent launch over all (128-row, 128-token) tiles.
int launch_gemm(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int64_t m, const MamboIQ3SWeight* w,
                const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo, const MamboLinearConfig& c,
                const DeviceInfo& info, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  const size_t need = gemm_workspace_bytes(m, w->n_blocks);
  if (!workspace || workspace_bytes < need)
    return fail(MAMBO_EWORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if ((uintptr_t)workspace % 256) return fail(MAMBO_EINVAL, "workspace must be 256-byte aligned");
  if ((int)gemm_tm_smem_bytes(c.stages) > info.max_smem_optin)
    return fail(MAMBO_EINVAL, "configuration needs %u bytes of shared memory (device allows %d)",
                gemm_tm_smem_bytes(c.stages), info.max_smem_optin);
  uint8_t* atoms = (uint8_t*)workspace + kCounterBytes;
  cudaError_t e = launch_xs_atoms(xs, ldxs, (int)m, (int)w->n_blocks, atoms, stream);
  if (e != cudaSuccess) return cuda_fail(e, "iq3s_xs_atoms");
  GemmTmMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  if (!make_gemm_x8_map(xq, ldxq, (int)m, w->n_blocks * 256, &maps.x))
    return fail(MAMBO_ECUDA, "could not encode the activation tensor map");
  GemmTmParams p{};
  p.m = (int)m;
  p.n_rows = (int)w->n_rows;
  p.n_blocks = (int)w->n_blocks;
  p.packed = (const uint8_t*)w->packed;
  p.xs_atoms = atoms;
  p.table = fp8_table;
  p.out = out;
  p.out_bf16 = out_dtype == MAMBO_BF16;
  p.ldo = ldo;
  p.wstages = c.stages;
  p.row_tiles = (int)((w->n_rows + 127) / 128);
  p.tok_tiles = (int)((m + gemm_tm_tile_tokens() - 1) / gemm_tm_tile_tokens());
  const int64_t tiles = (int64_t)p.row_tiles * p.tok_tiles;
  const int grid = (int)(tiles < info.sms ? tiles : info.sms);
  e = launch_gemm_tm(p, maps, grid, stream);
  if (e != cudaSuccess) return cuda_fail(e, "iq3s_gemm_tm");
  return ok();
}

// Where the FP16 GEMM's activation operand comes from: MXFP8 codes (xq, xs),
// or bf16 / f32 rows quantized on the way (x, x_dtype, ldx).
struct GemmF16Source {
  const uint8_t* xq;
  int64_t ldxq;
  const uint8_t* xs;
  int64_t ldxs;
  const void* x;
  int x_dtype;
  int64_t ldx;
};

// The FP16-operand GEMM: activations to FP16 with per-token scales
// (workspace; from bf16 / f32 rows the quantization is part of that pass),
// then one persistent launch over all tiles.
int launch_gemm_f16_path(const GemmF16Source& src, int64_t m, const MamboIQ3SWeight* w, const uint32_t* fp8_table,
                         void* out, int out_dtype, int64_t ldo, const MamboLinearConfig& c, const DeviceInfo& info,
                         void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  const bool wide = c.kernel == MAMBO_KERNEL_GEMM_F16_WIDE;
  const bool pair = c.kernel == MAMBO_KERNEL_GEMM_F16_PAIR || wide;
  const bool fold = c.kernel == MAMBO_KERNEL_GEMM_F16_FOLD || wide;
  const int ks = pair ? 1 : gemm_f16_clamp_split(c.split, m, w->n_rows, w->n_blocks);
  const size_t need = gemm_f16_workspace_bytes(m, w->n_rows, w->n_blocks, ks);
  if (!workspace || workspace_bytes < need)
    return fail(MAMBO_EWORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if ((uintptr_t)workspace % 256) return fail(MAMBO_EINVAL, "workspace must be 256-byte aligned");
  if ((int)gemm_f16_smem_bytes(c.stages) > info.max_smem_optin)
    return fail(MAMBO_EINVAL, "configuration needs %u bytes of shared memory (device allows %d)",
                gemm_f16_smem_bytes(c.stages), info.max_smem_optin);
  const int64_t k = w->n_blocks * 256;
  uint16_t* x16 = (uint16_t*)((uint8_t*)workspace + kCounterBytes);
  float* tok_scale = (float*)((uint8_t*)x16 + align256((size_t)m * k * 2));
  cudaError_t e = src.x ? launch_x16_quant(src.x, src.x_dtype, src.ldx, (int)m, k, x16, k, tok_scale, stream)
                        : launch_x16(src.xq, src.ldxq, src.xs, src.ldxs, (int)m, k, x16, k, tok_scale, stream);
  if (e != cudaSuccess) return cuda_fail(e, src.x ? "iq3s_x16_quant" : "iq3s_x16");
  GemmF16Maps maps;
  std::memset(&maps, 0, sizeof(maps));
  // A CTA of a pair loads 64 of the tile's 128 tokens (wide: 128 of 256).
  if (!make_gemm_x16_map(x16, k, (int)m, k, pair && !wide ? 64 : 128, &maps.x16))
    return fail(MAMBO_ECUDA, "could not encode the FP16 activation tensor map");
  GemmF16Params p{};
  p.m = (int)m;
  p.n_rows = (int)w->n_rows;
  p.n_blocks = (int)w->n_blocks;
  p.packed = (const uint8_t*)w->packed;
  p.tok_scale = tok_scale;
  p.table = fp8_table;
  p.out = out;
  p.out_bf16 = out_dtype == MAMBO_BF16;
  p.ldo = ldo;
  p.wstages = c.stages;
  p.row_tiles = (int)((w->n_rows + 127) / 128);
  p.tok_tiles = (int)(wide ? (m + 255) / 256 : (m + 127) / 128);
  p.ksplit = ks;
  if (fold)  // the row exponents after the packed records
    p.row_exp = (const int8_t*)w->packed + (size_t)p.row_tiles * (size_t)w->n_blocks * MAMBO_IQ3S_RECORD_BYTES;
  if (ks > 1) {
    // Partials after the token scales; counters in the counter region's second half.
    p.partials = (float*)((uint8_t*)tok_scale + gemm_f16_tok_scale_bytes(m));
    p.split_counters = (int*)((uint8_t*)workspace + kGemmSplitCounterOffset);
  }
  // bf16 output in 16-byte aligned rows: tiles leave through shared memory and
  // a TMA store, with the weight stages it needs room for (not with a K split:
  // there each epilogue warp of a tile's last contributor stores its part).
  if (ks == 1 && out_dtype == MAMBO_BF16 && make_gemm_out_map(out, ldo, (int)w->n_rows, (int)m, &maps.out)) {
    int st = c.stages;
    while (st > 2 && (int)gemm_f16_smem_bytes(st, true) > info.max_smem_optin) --st;
    if ((int)gemm_f16_smem_bytes(st, true) <= info.max_smem_optin) {
      p.out_tma = 1;
      p.wstages = st;
    }
  }
  if (pair) {
    const int64_t tiles = (int64_t)((p.row_tiles + 1) / 2) * p.tok_tiles;
    int clusters = gemm_f16_pair_max_clusters(p.wstages, p.out_tma != 0);
    if (clusters < 1) return fail(MAMBO_EINVAL, "no CTA pair of this configuration fits on the device");
    if (tiles < clusters) clusters = (int)tiles;
    e = launch_gemm_f16_pair(p, maps, clusters, stream, wide);
    if (e != cudaSuccess) return cuda_fail(e, wide ? "iq3s_gemm_f16 (wide pairs)" : "iq3s_gemm_f16 (pairs)");
    return ok();
  }
  const int64_t tiles = (int64_t)p.row_tiles * p.tok_tiles * ks;
  const int grid = (int)(tiles < info.sms ? tiles : info.sms);
  e = launch_gemm_f16(p, maps, grid, stream, fold);
  if (e != cudaSuccess) return cuda_fail(e, fold ? "iq3s_gemm_f16 (folded)" : "iq3s_gemm_f16");
  return ok();
}

// The GEMV's activation tensor maps (MXFP8 codes and scales of tokens [0, mc));
// rows that are not 16-byte aligned are copied to xcopy / xscopy first.
int gemv_activation_maps(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int64_t mc, int64_t b,
                         int box, uint8_t* xcopy, uint8_t* xscopy, GemvTmMaps* maps, cudaStream_t stream) {
  const int64_t k = b * 256;
  if (!make_gemv_x_map(xq, ldxq, (int)mc, (int)b, box, &maps->x)) {
    if (!xcopy) return fail(MAMBO_EINVAL, "x_values rows must be 16-byte aligned");
    cudaError_t e = cudaMemcpy2DAsync(xcopy, (size_t)k, xq, (size_t)ldxq, (size_t)k, (size_t)mc,
                                      cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return cuda_fail(e, "copy of unaligned x_values");
    if (!make_gemv_x_map(xcopy, k, (int)mc, (int)b, box, &maps->x))
      return fail(MAMBO_ECUDA, "activation tensor map could not be encoded");
  }
  if (!make_gemv_xs_map(xs, ldxs, (int)mc, (int)b, box, &maps->xs)) {
    if (!xscopy) return fail(MAMBO_EINVAL, "x_scales rows must be 16-byte aligned");
    const int64_t ld = xs_copy_stride(b);
    cudaError_t e = cudaMemcpy2DAsync(xscopy, (size_t)ld, xs, (size_t)ldxs, (size_t)(b * 8), (size_t)mc,
                                      cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return cuda_fail(e, "copy of unaligned x_scales");
    if (!make_gemv_xs_map(xscopy, ld, (int)mc, (int)b, box, &maps->xs))
      return fail(MAMBO_ECUDA, "activation-scale tensor map could not be encoded");
  }
  return MAMBO_OK;
}

// Launches the tcgen05 GEMV for tokens [0, mc) of xq/xs (already offset to the chunk).
int launch_tc_chunk(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int64_t mc,
                    const MamboIQ3SWeight* w, const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo,
                    const MamboLinearConfig& c, const GemvPlan& P, const DeviceInfo& info, int* counters,
                    float* partials, uint8_t* xcopy, uint8_t* xscopy, cudaStream_t stream,
                    const uint16_t* x_bf16 = nullptr, int64_t ldx = 0, const MamboQuantOut* qo = nullptr) {
  GemvTmMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  const uintptr_t fields[5] = {(uintptr_t)w->d, (uintptr_t)w->qs, (uintptr_t)w->qh, (uintptr_t)w->signs,
                               (uintptr_t)w->scales};
  for (uintptr_t f : fields)
    if (f % 16 != 0 || w->n_rows % 8 != 0)
      return fail(MAMBO_EINVAL,
                  "the tcgen05 GEMV needs N %% 8 == 0 and 16-byte aligned weight fields (use MAMBO_KERNEL_GEMV_SYNC)");
  const int box = 8 * P.nt;
  if (x_bf16) {
    // Fused quantization: the kernel loads the bf16 rows itself.
    if (!make_gemv_xb_map(x_bf16, ldx, (int)mc, w->n_blocks * 256, box, &maps.xb))
      return fail(MAMBO_EINVAL, "bf16 activations need 16-byte aligned rows");
  } else {
    // TMA boxes of the chunk's own rows (mc <= box).
    const int st = gemv_activation_maps(xq, ldxq, xs, ldxs, mc, w->n_blocks, (int)mc, xcopy, xscopy, &maps, stream);
    if (st != MAMBO_OK) return st;
  }
  GemvTmParams p{};
  p.m = (int)mc;
  p.n_rows = (int)w->n_rows;
  p.n_blocks = (int)w->n_blocks;
  p.d = (const uint8_t*)w->d;
  p.qs = (const uint8_t*)w->qs;
  p.qh = (const uint8_t*)w->qh;
  p.signs = (const uint8_t*)w->signs;
  p.scales = (const uint8_t*)w->scales;
  p.packed = (const uint8_t*)w->packed;
  if ((uintptr_t)w->packed % 16) return fail(MAMBO_EINVAL, "the packed weight buffer must be 16-byte aligned");
  p.table = fp8_table;
  p.out = out;
  p.out_bf16 = out_dtype == MAMBO_BF16;
  p.ldo = ldo;
  p.partials = partials;
  p.counters = counters;
  p.stages = c.stages;
  p.prefetch = c.prefetch;
  p.kparts = P.kparts;
  p.row_tiles = P.row_tiles;
  p.total_units = P.units;
  p.x_bf16 = x_bf16;
  p.ldx = ldx;
  p.box_rows = x_bf16 ? 0 : (int)mc;
  if (qo && qo->q) {  // quantized output for the next linear, written by the epilogue
    p.q_out = qo->q;
    p.ldq = qo->ldq;
    p.s_out = qo->s;
    p.lds = qo->lds;
  }
  cudaError_t e = launch_gemv_tm(p, P.nt, c.warps, maps, P.grid, stream);
  if (e != cudaSuccess) return cuda_fail(e, "iq3s_gemv_tm");
  return MAMBO_OK;
}

bool want_qout(const MamboQuantOut* qo) { return qo != nullptr && qo->q != nullptr; }

int check_qout(const MamboQuantOut* qo, int64_t n, int64_t m) {
  if (!want_qout(qo)) return MAMBO_OK;
  if (!qo->s) return fail(MAMBO_EINVAL, "quantized output: null scale pointer");
  if (n % 32) return fail(MAMBO_EINVAL, "quantized output needs N %% 32 == 0 (N=%lld)", (long long)n);
  if (qo->ldq < n || qo->lds < n / 32) return fail(MAMBO_EINVAL, "quantized output row stride is smaller than the row");
  (void)m;
  return MAMBO_OK;
}

// The quantized output chunk of tokens [m0, ...).
MamboQuantOut qout_rows(const MamboQuantOut* qo, int64_t m0) {
  MamboQuantOut r{};
  if (want_qout(qo)) r = MamboQuantOut{qo->q + m0 * qo->ldq, qo->ldq, qo->s + m0 * qo->lds, qo->lds};
  return r;
}

int linear_impl(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int64_t m, const MamboIQ3SWeight* w,
                const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo, const MamboQuantOut* qo,
                const MamboLinearConfig* cfg, void* workspace, size_t workspace_bytes, cudaStream_t stream);
int fused_impl(const void* x, int x_dtype, int64_t ldx, int64_t m, const MamboIQ3SWeight* w, const uint32_t* fp8_table,
               void* out, int out_dtype, int64_t ldo, const MamboQuantOut* qo, const MamboLinearConfig* cfg,
               void* workspace, size_t workspace_bytes, cudaStream_t stream);

}  // namespace

extern "C" {

const char* mambo_version(void) { return "mambo_b200 0.1.0 (sm_100a)"; }

int mambo_last_error(char* buf, size_t len) {
  if (buf && len) {
    std::strncpy(buf, g_last_error.c_str(), len - 1);
    buf[len - 1] = '\0';
  }
  return g_last_code;
}

int mambo_device_check(void) {
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  cudaError_t e = probe_kernel_image();
  if (e != cudaSuccess) return cuda_fail(e, "loading the sm_100a kernel image");
  return ok();
}

int mambo_device_status(int reset, int* code, int* where, int* block) {
  DeviceStatus st{};
  cudaError_t e = cudaMemcpyFromSymbol(&st, g_device_status, sizeof(st));
  if (e != cudaSuccess) return cuda_fail(e, "reading the device status");
  if (code) *code = st.code;
  if (where) *where = st.where;
  if (block) *block = st.block;
  if (reset) {
    DeviceStatus zero{};
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_fail(e, "resetting the device status");
  }
  return ok();
}

int mambo_set_wait_limit_ns(unsigned long long ns) {
  cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns));
  if (e != cudaSuccess) return cuda_fail(e, "setting the wait limit");
  return ok();
}

int mambo_selftest_wait_timeout(unsigned long long limit_ns, mambo_stream_t stream) {
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  cudaError_t e = launch_wait_selftest(limit_ns, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "launching the wait self-test");
  return ok();
}

int mambo_iq3s_prepare(const uint8_t* raw, int64_t n_rows, int64_t n_blocks, int64_t stride_row,
                       int64_t stride_block, int64_t stride_byte, void* d, void* qs, void* qh, void* signs,
                       void* scales, mambo_stream_t stream) {
  if (!raw || !d || !qs || !qh || !signs || !scales) return fail(MAMBO_EINVAL, "null pointer");
  if (n_rows < 1 || n_blocks < 1) return fail(MAMBO_EINVAL, "IQ3_S weight must have positive N and K");
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  PrepareParams p{raw, n_rows, n_blocks, stride_row, stride_block, stride_byte,
                  {(uint8_t*)d, (uint8_t*)qs, (uint8_t*)qh, (uint8_t*)signs, (uint8_t*)scales}};
  cudaError_t e = launch_iq3s_prepare(p, info.sms, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "iq3s_prepare");
  return ok();
}

size_t mambo_iq3s_packed_bytes(int64_t n_rows, int64_t n_blocks) {
  if (n_rows < 1 || n_blocks < 1) return 0;
  const size_t tiles = (size_t)((n_rows + MAMBO_IQ3S_TILE_ROWS - 1) / MAMBO_IQ3S_TILE_ROWS);
  // The records, then one row exponent per row of whole tiles (16-byte padded).
  return tiles * (size_t)n_blocks * MAMBO_IQ3S_RECORD_BYTES + (tiles * MAMBO_IQ3S_TILE_ROWS + 15) / 16 * 16;
}

int mambo_iq3s_pack(const MamboIQ3SWeight* w, void* packed, mambo_stream_t stream) {
  if (!w || !packed) return fail(MAMBO_EINVAL, "null pointer");
  if (!w->d || !w->qs || !w->qh || !w->signs || !w->scales) return fail(MAMBO_EINVAL, "null weight field");
  if (w->n_rows < 1 || w->n_blocks < 1) return fail(MAMBO_EINVAL, "IQ3_S weight must have positive N and K");
  if (w->n_rows % 8 != 0) return fail(MAMBO_EINVAL, "the packed layout needs N %% 8 == 0");
  const uintptr_t ptrs[6] = {(uintptr_t)w->d, (uintptr_t)w->qs, (uintptr_t)w->qh, (uintptr_t)w->signs,
                             (uintptr_t)w->scales, (uintptr_t)packed};
  for (uintptr_t a : ptrs)
    if (a % 16) return fail(MAMBO_EINVAL, "weight fields and the packed buffer must be 16-byte aligned");
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  PackWeightParams p{(const uint8_t*)w->d, (const uint8_t*)w->qs, (const uint8_t*)w->qh, (const uint8_t*)w->signs,
                     (const uint8_t*)w->scales, w->n_rows, w->n_blocks, (uint8_t*)packed};
  cudaError_t e = launch_iq3s_pack(p, info.sms, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "iq3s_pack");
  const size_t records = (size_t)((w->n_rows + 127) / 128) * (size_t)w->n_blocks * MAMBO_IQ3S_RECORD_BYTES;
  e = launch_iq3s_row_exp((const uint8_t*)w->d, w->n_rows, w->n_blocks, (int8_t*)packed + records,
                          (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "iq3s_row_exp");
  return ok();
}

int mambo_iq3s_decode(const MamboIQ3SWeight* w, const uint32_t* fp8_table, uint8_t* values, float* scales,
                      mambo_stream_t stream) {
  if (!w || !fp8_table || !values || !scales) return fail(MAMBO_EINVAL, "null pointer");
  if (!has_soa(w)) return fail(MAMBO_EINVAL, "the decoder reads the SoA weight fields, which this weight does not carry");
  if (w->n_rows < 1 || w->n_blocks < 1) return fail(MAMBO_EINVAL, "IQ3_S weight must have positive N and K");
  if ((uintptr_t)values % 8) return fail(MAMBO_EINVAL, "values must be 8-byte aligned");
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  DecodeParams p{(const uint8_t*)w->d, (const uint8_t*)w->qs, (const uint8_t*)w->qh, (const uint8_t*)w->signs,
                 (const uint8_t*)w->scales, w->n_rows, w->n_blocks, fp8_table, values, scales};
  cudaError_t e = launch_iq3s_decode(p, info.sms, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "iq3s_decode");
  return ok();
}

int mambo_quantize_mxfp8(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, uint8_t* q, int64_t ldq,
                         uint8_t* s, int64_t lds, int rounding, mambo_stream_t stream) {
  if (!x || !q || !s) return fail(MAMBO_EINVAL, "null pointer");
  if (x_dtype != MAMBO_F32 && x_dtype != MAMBO_BF16) return fail(MAMBO_EINVAL, "activation must be f32 or bf16");
  if (m < 1 || k < 32 || k % 32) return fail(MAMBO_EINVAL, "activation must be [M,K] with K divisible by 32");
  if (ldx < k || ldq < k || lds < k / 32) return fail(MAMBO_EINVAL, "row stride smaller than the row");
  if (rounding != MAMBO_ROUND_NEAREST_EVEN && rounding != MAMBO_ROUND_TIES_DOWN)
    return fail(MAMBO_EINVAL, "unknown rounding mode %d", rounding);
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  QuantParams p{x, m, k, ldx, q, ldq, s, lds};
  cudaError_t e = launch_quantize_mxfp8(p, x_dtype, rounding, info.sms, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "quantize_mxfp8");
  return ok();
}

int mambo_default_config(int64_t m, int64_t n_rows, int64_t n_blocks, MamboLinearConfig* cfg) {
  if (!cfg) return fail(MAMBO_EINVAL, "null config");
  int st;
  DeviceInfo info = device_info(&st);
  default_config(m, n_rows, n_blocks, cfg, (st == MAMBO_OK && info.max_smem_optin > 0) ? info.max_smem_optin
                                                                                        : kSmemOptinDefault,
                 st == MAMBO_OK ? info.sms : 148);
  return ok();
}

int mambo_num_configs(int kernel) {
  if (kernel == MAMBO_KERNEL_GEMV || kernel == MAMBO_KERNEL_AUTO) return kNumTcConfigs;
  if (is_gemm_f16_single(kernel)) return kNumGemmF16Configs;
  if (is_gemm(kernel)) return kNumGemmConfigs;
  if (kernel == MAMBO_KERNEL_GEMV_SYNC) return kNumSyncConfigs;
  return 0;
}

int mambo_config_at(int kernel, int index, MamboLinearConfig* cfg) {
  if (!cfg) return fail(MAMBO_EINVAL, "null config");
  if (kernel == MAMBO_KERNEL_AUTO) kernel = MAMBO_KERNEL_GEMV;
  const int n = mambo_num_configs(kernel);
  if (n == 0 || index < 0 || index >= n) return fail(MAMBO_EINVAL, "no configuration %d for kernel %d", index, kernel);
  std::memset(cfg, 0, sizeof(*cfg));
  cfg->kernel = kernel;
  cfg->ctas_per_sm = 1;
  cfg->split = index % 2;
  if (is_gemm(kernel)) {
    cfg->split = 0;
    cfg->warps = 8;
    if (is_gemm_f16_single(kernel)) {
      cfg->stages = kGemmStages[index % kNumGemmConfigs];
      cfg->split = kGemmSplits[index / kNumGemmConfigs];
    } else {
      cfg->stages = kGemmStages[index];
    }
  } else if (kernel == MAMBO_KERNEL_GEMV) {
    cfg->split = index % 3;
    const TcChoice& t = kTcChoices[index / 3];
    cfg->warps = t.warps;
    cfg->stages = t.stages;
    cfg->prefetch = t.prefetch;
  } else {
    cfg->warps = kSyncWarps[index / 8];
    cfg->stages = kSyncStages[(index / 2) % 4];
  }
  return ok();
}

size_t mambo_iq3s_linear_workspace_bytes(int64_t m, int64_t n_rows, int64_t n_blocks, const MamboLinearConfig* cfg) {
  int st;
  DeviceInfo info = device_info(&st);
  MamboLinearConfig c;
  if (cfg) c = *cfg;
  else default_config(m, n_rows, n_blocks, &c, (st == MAMBO_OK && info.max_smem_optin > 0) ? info.max_smem_optin
                                                                                          : kSmemOptinDefault,
                      st == MAMBO_OK ? info.sms : 148);
  const int sms = (st == MAMBO_OK && info.sms > 0) ? info.sms : 148;
  const int smem_optin = (st == MAMBO_OK && info.max_smem_optin > 0) ? info.max_smem_optin : kSmemOptinDefault;
  resolve_auto(&c, m, n_rows, n_blocks, smem_optin, sms);  // as mambo_iq3s_linear resolves it
  // A GEMM call may fall back to the GEMV (unaligned activations, no packed
  // weight copy): room for both.
  MamboLinearConfig cv = c;
  if (is_gemm(kernel_of(c)))
    default_config(m < 32 ? m : 31, n_rows, n_blocks, &cv, smem_optin, sms);
  const int64_t m_chunk = m < 32 ? m : 32;
  GemvPlan P = plan_gemv(m_chunk, n_rows, n_blocks, cv, sms, smem_optin);
  const size_t gemv = P.counters_bytes + P.partial_bytes + P.xcopy_bytes + P.xscopy_bytes;
  const size_t gemm = kernel_of(c) == MAMBO_KERNEL_GEMM       ? gemm_workspace_bytes(m, n_blocks)
                     : is_gemm_f16(kernel_of(c))
                         ? gemm_f16_workspace_bytes(m, n_rows, n_blocks,
                                                    is_gemm_f16_single(c.kernel)
                                                        ? gemm_f16_clamp_split(c.split, m, n_rows, n_blocks)
                                                        : 1)
                                                             : 0;
  return gemv > gemm ? gemv : gemm;
}

int mambo_iq3s_linear(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int64_t m,
                      const MamboIQ3SWeight* w, const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo,
                      const MamboLinearConfig* cfg, void* workspace, size_t workspace_bytes, mambo_stream_t stream) {
  return linear_impl(xq, ldxq, xs, ldxs, m, w, fp8_table, out, out_dtype, ldo, nullptr, cfg, workspace,
                     workspace_bytes, (cudaStream_t)stream);
}

int mambo_iq3s_linear_q(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int64_t m,
                        const MamboIQ3SWeight* w, const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo,
                        const MamboQuantOut* qout, const MamboLinearConfig* cfg, void* workspace,
                        size_t workspace_bytes, mambo_stream_t stream) {
  return linear_impl(xq, ldxq, xs, ldxs, m, w, fp8_table, out, out_dtype, ldo, qout, cfg, workspace, workspace_bytes,
                     (cudaStream_t)stream);
}

}  // extern "C"

namespace {

// Runs the quantizer on a finished linear's output when the caller asked for
// its MXFP8 quantization and the kernel did not form it in its epilogue.
int quantize_output_after(int st, const MamboQuantOut* qo, const void* out, int out_dtype, int64_t m, int64_t n,
                          int64_t ldo, cudaStream_t stream) {
  if (st != MAMBO_OK || !want_qout(qo)) return st;
  return mambo_quantize_mxfp8(out, out_dtype, m, n, ldo, qo->q, qo->ldq, qo->s, qo->lds, MAMBO_ROUND_NEAREST_EVEN,
                              stream);
}

int linear_impl(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int64_t m, const MamboIQ3SWeight* w,
                const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo, const MamboQuantOut* qo,
                const MamboLinearConfig* cfg, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!xq || !xs || !w || !fp8_table || !out) return fail(MAMBO_EINVAL, "null pointer");
  if (!weight_fields_ok(w)) return fail(MAMBO_EINVAL, "null weight field");
  if (w->n_rows < 1 || w->n_blocks < 1) return fail(MAMBO_EINVAL, "IQ3_S weight must have positive N and K");
  if (w->n_rows > (1 << 30) || w->n_blocks > (1 << 20)) return fail(MAMBO_EINVAL, "weight too large");
  const int64_t k = w->n_blocks * 256;
  if (m < 1) return fail(MAMBO_EINVAL, "x_values must be uint8 [M,K] with M >= 1");
  if (ldxq < k) return fail(MAMBO_EINVAL, "x_values row stride %lld is smaller than K=%lld", (long long)ldxq,
                            (long long)k);
  if (ldxs < k / 32) return fail(MAMBO_EINVAL, "x_scales row stride is smaller than K/32");
  if (out_dtype != MAMBO_F32 && out_dtype != MAMBO_BF16) return fail(MAMBO_EINVAL, "out must be f32 or bf16");
  if (ldo < w->n_rows) return fail(MAMBO_EINVAL, "out row stride is smaller than N");
  if (check_qout(qo, w->n_rows, m) != MAMBO_OK) return g_last_code;
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  MamboLinearConfig c;
  if (cfg) c = *cfg; else default_config(m, w->n_rows, w->n_blocks, &c, info.max_smem_optin, info.sms);
  resolve_auto(&c, m, w->n_rows, w->n_blocks, info.max_smem_optin, info.sms);
  if (is_gemm(c.kernel)) {
    if (gemm_usable(w, xq, ldxq, m)) {
      st = validate_config(&c, 32, w->n_blocks, info);
      if (st != MAMBO_OK) return st;
      if (is_gemm_f16(c.kernel))
        st = launch_gemm_f16_path(GemmF16Source{xq, ldxq, xs, ldxs, nullptr, 0, 0}, m, w, fp8_table, out, out_dtype,
                                  ldo, c, info, workspace, workspace_bytes, stream);
      else
        st = launch_gemm(xq, ldxq, xs, ldxs, m, w, fp8_table, out, out_dtype, ldo, c, info, workspace,
                         workspace_bytes, stream);
      return quantize_output_after(st, qo, out, out_dtype, m, w->n_rows, ldo, stream);
    }
    if (cfg && is_gemm(cfg->kernel))
      return fail(MAMBO_EINVAL,
                  "the GEMM needs the tile-major packed weight copy (N %% 8 == 0) and 16-byte aligned activation rows");
    // Otherwise the GEMV in 32-token chunks.
    default_config(31, w->n_rows, w->n_blocks, &c, info.max_smem_optin, info.sms);
  }
  if (c.kernel == MAMBO_KERNEL_GEMV && (w->n_rows % 8 != 0 || c.loader != 0)) {
    // The legacy mma.sync GEMV: the deepest of the given stages that fits.
    c.kernel = MAMBO_KERNEL_GEMV_SYNC;
    if (c.stages > 12) c.stages = 12;
    while (c.stages > 2 &&
           (int)config_smem(c, gemv_nt_for(m < 32 ? m : 32), w->n_blocks) > info.max_smem_optin)
      --c.stages;
  }
  if (c.kernel == MAMBO_KERNEL_GEMV_SYNC && c.warps == 0) c.warps = 8;
  if (c.kernel == MAMBO_KERNEL_GEMV_SYNC && c.stages > 12) c.stages = 4;
  st = validate_config(&c, m < 32 ? m : 32, w->n_blocks, info);
  if (st != MAMBO_OK) return st;

  const int64_t m_chunk_max = 32;
  const bool tc = kernel_of(c) == MAMBO_KERNEL_GEMV;
  for (int64_t m0 = 0; m0 < m; m0 += m_chunk_max) {
    const int64_t mc = (m - m0) < m_chunk_max ? (m - m0) : m_chunk_max;
    GemvPlan P = plan_gemv(mc, w->n_rows, w->n_blocks, c, info.sms, info.max_smem_optin);
    if ((size_t)P.counter_slots * sizeof(int) > kGemvCounterBytes)
      return fail(MAMBO_EINVAL, "N=%lld needs more split-K counters than the workspace holds", (long long)w->n_rows);
    const size_t need = P.counters_bytes + P.partial_bytes + P.xcopy_bytes + P.xscopy_bytes;
    if (!workspace || workspace_bytes < need)
      return fail(MAMBO_EWORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    if ((uintptr_t)workspace % 256) return fail(MAMBO_EINVAL, "workspace must be 256-byte aligned");
    const size_t esz = out_dtype == MAMBO_BF16 ? 2 : 4;
    int* counters = (int*)workspace;
    float* partials = (float*)((uint8_t*)workspace + P.counters_bytes);
    uint8_t* xcopy = (uint8_t*)workspace + P.counters_bytes + P.partial_bytes;
    uint8_t* xscopy = xcopy + P.xcopy_bytes;

    if (tc) {
      const MamboQuantOut qc = qout_rows(qo, m0);  // the epilogue quantizes this chunk's outputs
      st = launch_tc_chunk(xq + m0 * ldxq, ldxq, xs + m0 * ldxs, ldxs, mc, w, fp8_table,
                           (uint8_t*)out + m0 * ldo * esz, out_dtype, ldo, c, P, info, counters, partials, xcopy,
                           xscopy, stream, nullptr, 0, &qc);
      if (st != MAMBO_OK) return st;
      continue;
    }
    if (!has_soa(w))
      return fail(MAMBO_EINVAL, "MAMBO_KERNEL_GEMV_SYNC reads the SoA weight fields, which this weight does not carry");
    GemvParams mp{};
    mp.n_rows = (int)w->n_rows;
    mp.n_blocks = (int)w->n_blocks;
    mp.d = (const uint8_t*)w->d;
    mp.qs = (const uint8_t*)w->qs;
    mp.qh = (const uint8_t*)w->qh;
    mp.signs = (const uint8_t*)w->signs;
    mp.scales = (const uint8_t*)w->scales;
    mp.warps = c.warps;
    GemvMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    const bool have_maps = (c.loader == 0) && make_gemv_maps(mp, &maps);
    cudaError_t e;
    {
      GemvParams p = mp;
      p.xq = xq + m0 * ldxq;
      p.ldxq = ldxq;
      p.xs = xs + m0 * ldxs;
      p.ldxs = ldxs;
      p.m = (int)mc;
      p.table = fp8_table;
      p.out = (uint8_t*)out + m0 * ldo * esz;
      p.out_bf16 = out_dtype == MAMBO_BF16;
      p.ldo = ldo;
      p.counters = counters;
      p.partials = partials;
      p.stages = c.stages;
      p.row_tiles = P.row_tiles;
      p.total_units = P.units;
      p.x_bulk = ((uintptr_t)p.xq % 16 == 0) && (ldxq % 16 == 0);
      e = launch_gemv(p, P.nt, have_maps, maps, P.grid, stream);
      if (e != cudaSuccess) return cuda_fail(e, "iq3s_gemv_sync");
    }
  }
  // The legacy GEMV has no quantizing epilogue.
  st = tc ? MAMBO_OK : quantize_output_after(MAMBO_OK, qo, out, out_dtype, m, w->n_rows, ldo, stream);
  return st == MAMBO_OK ? ok() : st;
}

}  // namespace

extern "C" {

size_t mambo_iq3s_linear_fused_workspace_bytes(int64_t m, int64_t n_rows, int64_t n_blocks,
                                               const MamboLinearConfig* cfg) {
  const int64_t k = n_blocks * 256;
  return align256(mambo_iq3s_linear_workspace_bytes(m, n_rows, n_blocks, cfg)) + align256((size_t)(m * k)) +
         align256((size_t)(m * (k / 32)));
}

int mambo_iq3s_linear_fused(const void* x, int x_dtype, int64_t ldx, int64_t m, const MamboIQ3SWeight* w,
                            const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo,
                            const MamboLinearConfig* cfg, void* workspace, size_t workspace_bytes,
                            mambo_stream_t stream) {
  return fused_impl(x, x_dtype, ldx, m, w, fp8_table, out, out_dtype, ldo, nullptr, cfg, workspace, workspace_bytes,
                    (cudaStream_t)stream);
}

int mambo_iq3s_linear_fused_q(const void* x, int x_dtype, int64_t ldx, int64_t m, const MamboIQ3SWeight* w,
                              const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo,
                              const MamboQuantOut* qout, const MamboLinearConfig* cfg, void* workspace,
                              size_t workspace_bytes, mambo_stream_t stream) {
  return fused_impl(x, x_dtype, ldx, m, w, fp8_table, out, out_dtype, ldo, qout, cfg, workspace, workspace_bytes,
                    (cudaStream_t)stream);
}

}  // extern "C"

namespace {

int fused_impl(const void* x, int x_dtype, int64_t ldx, int64_t m, const MamboIQ3SWeight* w, const uint32_t* fp8_table,
               void* out, int out_dtype, int64_t ldo, const MamboQuantOut* qo, const MamboLinearConfig* cfg,
               void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!x || !w || !fp8_table || !out) return fail(MAMBO_EINVAL, "null pointer");
  if (!weight_fields_ok(w)) return fail(MAMBO_EINVAL, "null weight field");
  if (w->n_rows < 1 || w->n_blocks < 1) return fail(MAMBO_EINVAL, "IQ3_S weight must have positive N and K");
  if (w->n_rows > (1 << 30) || w->n_blocks > (1 << 20)) return fail(MAMBO_EINVAL, "weight too large");
  if (x_dtype != MAMBO_F32 && x_dtype != MAMBO_BF16) return fail(MAMBO_EINVAL, "activation must be f32 or bf16");
  const int64_t k = w->n_blocks * 256;
  if (m < 1) return fail(MAMBO_EINVAL, "activation must be [M,K] with M >= 1");
  if (ldx < k) return fail(MAMBO_EINVAL, "activation row stride is smaller than K");
  if (out_dtype != MAMBO_F32 && out_dtype != MAMBO_BF16) return fail(MAMBO_EINVAL, "out must be f32 or bf16");
  if (ldo < w->n_rows) return fail(MAMBO_EINVAL, "out row stride is smaller than N");
  if (check_qout(qo, w->n_rows, m) != MAMBO_OK) return g_last_code;
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  MamboLinearConfig c;
  if (cfg) c = *cfg; else default_config(m, w->n_rows, w->n_blocks, &c, info.max_smem_optin, info.sms);
  resolve_auto(&c, m, w->n_rows, w->n_blocks, info.max_smem_optin, info.sms);
  const uintptr_t fields[6] = {(uintptr_t)w->d, (uintptr_t)w->qs, (uintptr_t)w->qh, (uintptr_t)w->signs,
                               (uintptr_t)w->scales, (uintptr_t)w->packed};
  bool aligned = w->n_rows % 8 == 0;
  for (uintptr_t f : fields) aligned = aligned && f % 16 == 0;
  // Decode-sized M on the tcgen05 GEMV: the kernel quantizes the bf16 rows itself.
  if (x_dtype == MAMBO_BF16 && m < kGemmMinTokens && c.kernel == MAMBO_KERNEL_GEMV && c.loader == 0 && aligned &&
      (uintptr_t)x % 16 == 0 && ldx % 8 == 0) {
    st = validate_config(&c, m, w->n_blocks, info);
    if (st != MAMBO_OK) return st;
    // The bf16 box ring takes the room of one or two weight stages: the
    // deepest pipeline that fits it under the same plan (fewer stages keep
    // the cluster K split valid, so the summation order, and the result, is
    // the two-step path's); without room at all, two steps.
    const GemvPlan P = plan_gemv(m, w->n_rows, w->n_blocks, c, info.sms, info.max_smem_optin);
    while (c.stages > 2 && (int)gemv_tm_smem_bytes(P.nt, c.stages, P.kparts, true) > info.max_smem_optin)
      --c.stages;
    if ((size_t)P.counter_slots * sizeof(int) > kGemvCounterBytes)
      return fail(MAMBO_EINVAL, "N=%lld needs more split-K counters than the workspace holds", (long long)w->n_rows);
    if ((int)gemv_tm_smem_bytes(P.nt, c.stages, P.kparts, true) <= info.max_smem_optin) {
      const size_t need = P.counters_bytes + P.partial_bytes;
      if (!workspace || workspace_bytes < need)
        return fail(MAMBO_EWORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
      if ((uintptr_t)workspace % 256) return fail(MAMBO_EINVAL, "workspace must be 256-byte aligned");
      int* counters = (int*)workspace;
      float* partials = (float*)((uint8_t*)workspace + P.counters_bytes);
      st = launch_tc_chunk(nullptr, 0, nullptr, 0, m, w, fp8_table, out, out_dtype, ldo, c, P, info, counters,
                           partials, nullptr, nullptr, stream, (const uint16_t*)x, ldx, qo);
      return st == MAMBO_OK ? ok() : st;
    }
  }
  // Prefill-sized M on the FP16 GEMM: the quantization is part of the pass
  // that writes the GEMM's FP16 activations (one launch instead of two, no
  // MXFP8 round trip through memory); the same codes, the same results.
  const int elt = x_dtype == MAMBO_BF16 ? 2 : 4;
  if (m >= kGemmMinTokens && is_gemm_f16(c.kernel) && w->packed && aligned && (uintptr_t)x % 16 == 0 &&
      (ldx * elt) % 16 == 0 && m <= (int64_t)1 << 30 && x16_quant_smem_bytes(k) <= (size_t)info.max_smem_optin) {
    st = validate_config(&c, 32, w->n_blocks, info);
    if (st != MAMBO_OK) return st;
    st = launch_gemm_f16_path(GemmF16Source{nullptr, 0, nullptr, 0, x, x_dtype, ldx}, m, w, fp8_table, out,
                              out_dtype, ldo, c, info, workspace, workspace_bytes, stream);
    st = quantize_output_after(st, qo, out, out_dtype, m, w->n_rows, ldo, stream);
    return st == MAMBO_OK ? ok() : st;
  }
  // Otherwise: quantize into the workspace, then the linear.
  const size_t lin = align256(mambo_iq3s_linear_workspace_bytes(m, w->n_rows, w->n_blocks, cfg));
  const size_t need = mambo_iq3s_linear_fused_workspace_bytes(m, w->n_rows, w->n_blocks, cfg);
  if (!workspace || workspace_bytes < need)
    return fail(MAMBO_EWORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  uint8_t* xq = (uint8_t*)workspace + lin;
  uint8_t* xs = xq + align256((size_t)(m * k));
  st = mambo_quantize_mxfp8(x, x_dtype, m, k, ldx, xq, k, xs, k / 32, MAMBO_ROUND_NEAREST_EVEN, stream);
  if (st != MAMBO_OK) return st;
  return linear_impl(xq, k, xs, k / 32, m, w, fp8_table, out, out_dtype, ldo, qo, cfg, workspace, lin, stream);
}

}  // namespace

extern "C" {


}  // extern "C"

// --------------------------------------------------------------------------
// Grouped linears: one persistent launch over independent linears.
// --------------------------------------------------------------------------
namespace {

constexpr int kGroupDecWarps = 8;
// Cost of a grouped launch's unit per activation pass (thousandths of a one-token unit).
constexpr int64_t kGroupCostPerPass = 200;
static_assert(MAMBO_MAX_GROUP == kGemvMaxItems, "group size limit of the C ABI and of the kernel");

// Whether the items qualify for one grouped launch (bf16 activations with
// 16-byte aligned rows, packed weights, M < 32, counters for every row tile).
bool group_fusable(const MamboLinearItem* items, int count) {
  if (count < 1 || count > kGemvMaxItems) return false;
  int64_t tiles = 0, units = 0;
  for (int i = 0; i < count; ++i) {
    const MamboLinearItem& it = items[i];
    const MamboIQ3SWeight* w = it.w;
    if (it.x_dtype != MAMBO_BF16 || it.m < 1 || it.m >= kGemmMinTokens) return false;
    if ((uintptr_t)it.x % 16 || it.ldx % 8) return false;
    if (!w->packed || (uintptr_t)w->packed % 16 || w->n_rows % 8) return false;
    const int64_t rt = (w->n_rows + 127) / 128;
    tiles += rt;
    units += rt * w->n_blocks;
  }
  return (size_t)tiles * 4 * sizeof(int) <= kGemvCounterBytes && units < (int64_t)1 << 30;
}

int group_nt(const MamboLinearItem* items, int count) {
  int64_t m = 1;
  for (int i = 0; i < count; ++i) m = items[i].m > m ? items[i].m : m;
  return gemv_nt_for(m);
}

size_t group_partial_bytes(int nt, int sms) { return align256((size_t)sms * 2 * 128 * 8 * nt * sizeof(float)); }

// A grouped launch quantizes its activations in a pre-pass (launch_group_xtiles)
// when an item has two or more tokens: the GEMV's activation warps would
// otherwise quantize every K block once per row tile, and from two tokens that
// work paces the pipeline (grouped launches of 8 tokens took 1.23 times as long
// per unit as those of one). One-token groups keep the quantization in the GEMV.
bool group_prequantize(const MamboLinearItem* items, int count) {
  for (int i = 0; i < count; ++i)
    if (items[i].m >= 2) return true;
  return false;
}
// The pre-pass's activation tiles: one per item and K block.
size_t group_xtiles_bytes(const MamboLinearItem* items, int count) {
  if (!group_prequantize(items, count)) return 0;
  size_t tiles = 0;
  for (int i = 0; i < count; ++i) tiles += (size_t)items[i].w->n_blocks;
  return align256(tiles * gemv_xtile_bytes(group_nt(items, count)));
}

// Estimated time of one (128-row tile, K block) unit of a grouped launch
// item with m tokens, in thousandths of a one-token unit. It grows with the
// activation warps' passes over the unit's bf16 block (from two tokens a lane
// quantizes one 32-value group of four tokens a pass). Measured on B200 with
// Llama-3-8B decode shapes: grouped launches of 1, 2, 4 and 8 tokens take
// 1.00, 1.03, 1.03 and 1.23 times as long per unit.
int64_t group_unit_cost(int m) { return m <= 1 ? 1000 : 830 + kGroupCostPerPass * (int64_t)((m + 3) / 4); }

int64_t group_item_units(const GemvItem& gi) { return (int64_t)((gi.n_rows + 127) / 128) * gi.n_blocks; }

// First unit of each CTA of a grouped launch (start[grid] = units): contiguous
// ranges of about equal estimated time, at least one unit each (grid <= units).
// uniform: every unit costs the same (the activations were quantized beforehand).
void split_group_units(const GemvGroup& g, int units, int grid, int* start, bool uniform) {
  auto cost = [uniform](int m) -> int64_t { return uniform ? 1000 : group_unit_cost(m); };
  int64_t total = 0;
  for (int i = 0; i < g.count; ++i) total += group_item_units(g.items[i]) * cost(g.items[i].m);
  start[0] = 0;
  int item = 0;
  int64_t before = 0;  // cost of the units of the items ahead of `item`
  for (int c = 1; c < grid; ++c) {
    const int64_t target = total * c / grid;
    while (item + 1 < g.count &&
           before + group_item_units(g.items[item]) * cost(g.items[item].m) <= target) {
      before += group_item_units(g.items[item]) * cost(g.items[item].m);
      ++item;
    }
    const int64_t cu = cost(g.items[item].m);
    // Rounded down, as a single linear's even split is: a group of one splits the same way.
    const int64_t u = g.items[item].unit0 + (target - before) / cu;
    const int64_t lo = start[c - 1] + 1, hi = units - (grid - c);
    start[c] = (int)(u < lo ? lo : u > hi ? hi : u);
  }
  start[grid] = units;
}

}  // namespace

extern "C" {

size_t mambo_iq3s_linear_group_workspace_bytes(const MamboLinearItem* items, int count) {
  if (!items || count < 1) return 0;
  int st;
  DeviceInfo info = device_info(&st);
  const int sms = (st == MAMBO_OK && info.sms > 0) ? info.sms : 148;
  size_t need = kCounterBytes + group_partial_bytes(group_nt(items, count), sms);
  bool have_w = true;
  for (int i = 0; i < count; ++i) have_w = have_w && items[i].w != nullptr;
  if (have_w && group_fusable(items, count)) need += group_xtiles_bytes(items, count);
  for (int i = 0; i < count; ++i) {  // the per-item path, when the group does not qualify
    if (!items[i].w) continue;
    const size_t b = mambo_iq3s_linear_fused_workspace_bytes(items[i].m, items[i].w->n_rows, items[i].w->n_blocks,
                                                             nullptr);
    need = b > need ? b : need;
  }
  return need;
}

int mambo_iq3s_linear_group(const MamboLinearItem* items, int count, const uint32_t* fp8_table, void* workspace,
                            size_t workspace_bytes, mambo_stream_t stream) {
  return mambo_iq3s_linear_group_q(items, nullptr, count, fp8_table, workspace, workspace_bytes, stream);
}

int mambo_iq3s_linear_group_q(const MamboLinearItem* items, const MamboQuantOut* qouts, int count,
                              const uint32_t* fp8_table, void* workspace, size_t workspace_bytes,
                              mambo_stream_t stream) {
  if (!items || !fp8_table) return fail(MAMBO_EINVAL, "null pointer");
  if (count < 1) return fail(MAMBO_EINVAL, "a group needs at least one linear");
  for (int i = 0; i < count; ++i) {
    const MamboLinearItem& it = items[i];
    const MamboIQ3SWeight* w = it.w;
    if (!it.x || !w || !it.out) return fail(MAMBO_EINVAL, "item %d: null pointer", i);
    if (!weight_fields_ok(w)) return fail(MAMBO_EINVAL, "item %d: null weight field", i);
    if (w->n_rows < 1 || w->n_blocks < 1 || w->n_rows > (1 << 30) || w->n_blocks > (1 << 20))
      return fail(MAMBO_EINVAL, "item %d: IQ3_S weight must have positive N and K", i);
    if (it.x_dtype != MAMBO_F32 && it.x_dtype != MAMBO_BF16)
      return fail(MAMBO_EINVAL, "item %d: activation must be f32 or bf16", i);
    if (it.m < 1 || it.ldx < w->n_blocks * 256) return fail(MAMBO_EINVAL, "item %d: activation must be [M,K]", i);
    if (it.out_dtype != MAMBO_F32 && it.out_dtype != MAMBO_BF16)
      return fail(MAMBO_EINVAL, "item %d: out must be f32 or bf16", i);
    if (it.ldo < w->n_rows) return fail(MAMBO_EINVAL, "item %d: out row stride is smaller than N", i);
    if (qouts && check_qout(&qouts[i], w->n_rows, it.m) != MAMBO_OK) return g_last_code;
  }
  if (!workspace || (uintptr_t)workspace % 256) return fail(MAMBO_EINVAL, "workspace must be 256-byte aligned");
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  if (!group_fusable(items, count)) {
    // One call per item, in order, on the stream (they share the workspace).
    for (int i = 0; i < count; ++i) {
      const MamboLinearItem& it = items[i];
      st = fused_impl(it.x, it.x_dtype, it.ldx, it.m, it.w, fp8_table, it.out, it.out_dtype, it.ldo,
                      qouts ? &qouts[i] : nullptr, nullptr, workspace, workspace_bytes, (cudaStream_t)stream);
      if (st != MAMBO_OK) return st;
    }
    return ok();
  }
  const int nt = group_nt(items, count);
  const bool pre = group_prequantize(items, count);
  const size_t need = kCounterBytes + group_partial_bytes(nt, info.sms) + group_xtiles_bytes(items, count);
  if (workspace_bytes < need)
    return fail(MAMBO_EWORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  GemvGroup g;
  std::memset(&g, 0, sizeof(g));
  g.count = count;
  int units = 0, tiles = 0, box = 8 * nt, xtiles = 0;
  for (int i = 0; i < count; ++i) {
    const MamboLinearItem& it = items[i];
    const MamboIQ3SWeight* w = it.w;
    const int rt = (int)((w->n_rows + 127) / 128);
    GemvItem& gi = g.items[i];
    gi.packed = (const uint8_t*)w->packed;
    gi.x = (const uint16_t*)it.x;
    gi.out = it.out;
    gi.ldx = it.ldx;
    gi.ldo = it.ldo;
    gi.n_rows = (int)w->n_rows;
    gi.n_blocks = (int)w->n_blocks;
    gi.m = (int)it.m;
    gi.out_bf16 = it.out_dtype == MAMBO_BF16;
    gi.unit0 = units;
    gi.tile0 = tiles;
    gi.xt0 = xtiles;
    xtiles += gi.n_blocks;
    if (qouts && want_qout(&qouts[i])) {  // N % 32 == 0 was checked: the epilogue quantizes the output
      gi.q_out = qouts[i].q;
      gi.ldq = qouts[i].ldq;
      gi.s_out = qouts[i].s;
      gi.lds = qouts[i].lds;
    }
    if (!make_gemv_xb_map(gi.x, it.ldx, gi.m, w->n_blocks * 256, box, &g.xb[i]))
      return fail(MAMBO_EINVAL, "item %d: bf16 activations need 16-byte aligned rows", i);
    units += rt * gi.n_blocks;
    tiles += rt;
  }
  GemvTmParams p;
  std::memset(&p, 0, sizeof(p));
  p.m = box;
  p.n_rows = 0;
  p.n_blocks = 1;  // per item in the group
  p.packed = g.items[0].packed;
  p.table = fp8_table;
  p.counters = (int*)workspace;
  p.partials = (float*)((uint8_t*)workspace + kCounterBytes);
  p.stages = 8;
  while (p.stages > 2 && (int)gemv_tm_smem_bytes(nt, p.stages, 0, true) > info.max_smem_optin) --p.stages;
  if ((int)gemv_tm_smem_bytes(nt, p.stages, 0, true) > info.max_smem_optin)
    return fail(MAMBO_EINVAL, "the grouped GEMV does not fit in shared memory");
  p.prefetch = 0;
  p.kparts = 0;
  p.row_tiles = tiles;
  p.total_units = units;
  int grid = units < info.sms ? units : info.sms;
  if (grid > kGemvMaxGrid) grid = kGemvMaxGrid;
  split_group_units(g, units, grid, g.cta_start, pre);
  if (pre) {
    // The pre-pass writes every item's activation tiles after the partials;
    // the GEMV (launched with programmatic serialization) starts its weight
    // stream while the pre-pass runs and reads the tiles after it.
    uint8_t* xt = (uint8_t*)workspace + kCounterBytes + group_partial_bytes(nt, info.sms);
    GroupXtilesParams xp;
    std::memset(&xp, 0, sizeof(xp));
    xp.count = count;
    xp.total_tiles = xtiles;
    xp.box = box;
    xp.tiles = xt;
    for (int i = 0; i < count; ++i)
      xp.items[i] = GroupXtilesParams::Item{g.items[i].x, g.items[i].ldx, g.items[i].m, g.items[i].n_blocks,
                                            g.items[i].xt0};
    cudaError_t e = launch_group_xtiles(xp, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "group_xtiles_kernel");
    GemvGroupPre gp;
    std::memset(&gp, 0, sizeof(gp));
    static_cast<GemvGroup&>(gp) = g;
    gp.xtiles = xt;
    e = launch_gemv_tm_group_pre(p, gp, nt, grid, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "iq3s_gemv_tm_kernel (group, quantized beforehand)");
    return ok();
  }
  cudaError_t e = launch_gemv_tm_group(p, g, nt, kGroupDecWarps, grid, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "iq3s_gemv_tm_kernel (group)");
  return ok();
}

}  // extern "C"

// --------------------------------------------------------------------------
// mambo_iq3s_linear_noalloc: the tcgen05 GEMV with library-held scratch, for
// callers that cannot allocate device memory (see include/mambo_b200.h).
// --------------------------------------------------------------------------

// Every GPU on which this module is loaded holds this array until the process
// exits. Layout: split-K counters | FP32 partials | activation rows copied for alignment.
static __device__ __align__(256) uint8_t g_linear_scratch[MAMBO_STATIC_SCRATCH_BYTES];

namespace {

constexpr size_t kStaticCounterBytes = 64 * 1024;  // 4 counters per 128-row tile: N <= 524288
constexpr int kStaticMaxCtas = 160;                // persistent grid cap (B200: 148 SMs)
constexpr int64_t kStaticChunk = 8;                // tokens per launch (one 8-token tile)
// Every chunk, the shorter last one included, is launched with the plan made
// for a full chunk: that holds while all chunk sizes share one token tile.
static_assert(kStaticChunk <= 8, "chunks of 1..kStaticChunk tokens must all use the 8-token tile (gemv_nt_for == 1)");
constexpr size_t kStaticPartialBytes = (size_t)kStaticMaxCtas * 2 * 128 * 8 * sizeof(float);
constexpr size_t kStaticXcopyOffset = kStaticCounterBytes + kStaticPartialBytes;
constexpr int64_t kStaticMaxK = 98304;  // activation rows copied for alignment: kStaticChunk x K bytes
static_assert(kStaticXcopyOffset % 256 == 0, "scratch regions must stay 256-byte aligned");
static_assert(kStaticXcopyOffset + kStaticChunk * kStaticMaxK + kStaticChunk * (kStaticMaxK / 32) <= MAMBO_STATIC_SCRATCH_BYTES,
              "static scratch too small");

// Device address of g_linear_scratch on the current device, looked up once per
// device (with that device current) and cached. The look-up is not allowed
// while `stream` is being captured into a CUDA graph: the first call on a
// device must come before any capture.
int static_scratch_address(uint8_t** out, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(MAMBO_ENOTSUPPORTED, "device ordinal %d out of range", dev);
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(stream, &cap);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
    if (cap != cudaStreamCaptureStatusNone)
      return fail(MAMBO_EINVAL,
                  "the first mambo_iq3s_linear_noalloc call on device %d is inside a stream capture; make one call "
                  "on this device before capturing",
                  dev);
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_linear_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
    if (!p || (uintptr_t)p % 256) return fail(MAMBO_ECUDA, "static scratch is not 256-byte aligned");
    addr[dev] = p;
  }
  *out = (uint8_t*)addr[dev];
  return MAMBO_OK;
}

}  // namespace

extern "C" int mambo_iq3s_linear_noalloc(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, int64_t m,
                                         const MamboIQ3SWeight* w, const uint32_t* fp8_table, void* out,
                                         int out_dtype, int64_t ldo, const MamboLinearConfig* cfg,
                                         mambo_stream_t stream) {
  if (!xq || !xs || !w || !fp8_table || !out) return fail(MAMBO_EINVAL, "null pointer");
  if (!weight_fields_ok(w)) return fail(MAMBO_EINVAL, "null weight field");
  if (w->n_rows < 1 || w->n_blocks < 1) return fail(MAMBO_EINVAL, "IQ3_S weight must have positive N and K");
  const int64_t k = w->n_blocks * 256;
  if (m < 1) return fail(MAMBO_EINVAL, "x_values must be uint8 [M,K] with M >= 1");
  if (ldxq < k) return fail(MAMBO_EINVAL, "x_values row stride %lld is smaller than K=%lld", (long long)ldxq,
                            (long long)k);
  if (ldxs < k / 32) return fail(MAMBO_EINVAL, "x_scales row stride is smaller than K/32");
  if (out_dtype != MAMBO_F32 && out_dtype != MAMBO_BF16) return fail(MAMBO_EINVAL, "out must be f32 or bf16");
  if (ldo < w->n_rows) return fail(MAMBO_EINVAL, "out row stride is smaller than N");
  if (w->n_rows % 8 != 0) return fail(MAMBO_EINVAL, "mambo_iq3s_linear_noalloc needs N %% 8 == 0");
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  const int64_t m_chunk = m < kStaticChunk ? m : kStaticChunk;
  MamboLinearConfig c;
  if (cfg) c = *cfg; else default_config(m_chunk, w->n_rows, w->n_blocks, &c, info.max_smem_optin, info.sms);
  if (c.kernel == MAMBO_KERNEL_AUTO) c.kernel = MAMBO_KERNEL_GEMV;
  if (c.kernel != MAMBO_KERNEL_GEMV || c.loader != 0)
    return fail(MAMBO_EINVAL, "mambo_iq3s_linear_noalloc runs the tcgen05 GEMV (MAMBO_KERNEL_GEMV, loader 0) only");
  st = validate_config(&c, m_chunk, w->n_blocks, info);
  if (st != MAMBO_OK) return st;

  const int sms = info.sms < kStaticMaxCtas ? info.sms : kStaticMaxCtas;
  const GemvPlan P = plan_gemv(m_chunk, w->n_rows, w->n_blocks, c, sms, info.max_smem_optin);
  const size_t counter_bytes = (size_t)P.counter_slots * sizeof(int);
  if (counter_bytes > kStaticCounterBytes)
    return fail(MAMBO_EINVAL, "N=%lld exceeds the static-scratch limit of mambo_iq3s_linear_noalloc (N <= %zu)",
                (long long)w->n_rows, kStaticCounterBytes / sizeof(int) / 4 * 128);
  if (k > kStaticMaxK)
    return fail(MAMBO_EINVAL, "K=%lld exceeds the static-scratch limit of mambo_iq3s_linear_noalloc (K <= %lld)",
                (long long)k, (long long)kStaticMaxK);
  if (P.partial_bytes > kStaticPartialBytes)
    return fail(MAMBO_EINVAL, "grid of %d CTAs exceeds the static scratch", P.grid);

  uint8_t* scratch = nullptr;
  st = static_scratch_address(&scratch, (cudaStream_t)stream);
  if (st != MAMBO_OK) return st;
  int* counters = (int*)scratch;
  float* partials = (float*)(scratch + kStaticCounterBytes);
  uint8_t* xcopy = scratch + kStaticXcopyOffset;

  // The counters must start at zero; a call that gave up on a bounded wait may
  // have left some behind, so every call clears the ones it uses.
  cudaError_t e = cudaMemsetAsync(counters, 0, counter_bytes, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(static scratch counters)");

  const size_t esz = out_dtype == MAMBO_BF16 ? 2 : 4;
  for (int64_t m0 = 0; m0 < m; m0 += kStaticChunk) {
    const int64_t mc = (m - m0) < kStaticChunk ? (m - m0) : kStaticChunk;
    st = launch_tc_chunk(xq + m0 * ldxq, ldxq, xs + m0 * ldxs, ldxs, mc, w, fp8_table,
                         (uint8_t*)out + m0 * ldo * esz, out_dtype, ldo, c, P, info, counters, partials, xcopy,
                         xcopy + kStaticChunk * kStaticMaxK, (cudaStream_t)stream);
    if (st != MAMBO_OK) return st;
  }
  return ok();
}

// ---------------------------------------------------------------------------
// Q4_K x MXFP8 linear on the tcgen05 GEMV (GGUF type Q4_K; the reference lists
// the type in src/python/mambo/utils/gguf_manifest.py:30-42 and has no kernel
// for it). Stream-K over (128-row tile, K block) units, 32-token chunks.
namespace {

// The Q4_K GEMV configuration: tcgen05 GEMV, 8 decoder warps. Default (from
// B200 measurements of the Llama-3-8B decode shapes with weights rotated past
// the L2): 4 weight stages, no L2 prefetch; the cluster K-split for long K
// (32 blocks or more) when every row tile gets at least two CTAs, stream-K
// otherwise.
int q4k_config(const MamboLinearConfig* cfg, int64_t mc, int64_t n, int64_t b, const DeviceInfo& info,
               MamboLinearConfig* c) {
  MamboLinearConfig d{};
  d.kernel = MAMBO_KERNEL_GEMV;
  d.warps = 8;
  d.ctas_per_sm = 1;
  d.split = (b >= 32 && (n + 127) / 128 * 2 <= info.sms) ? 2 : 0;
  d.prefetch = 0;
  d.stages = 4;
  if (cfg && cfg->kernel != MAMBO_KERNEL_AUTO) {
    if (cfg->kernel != MAMBO_KERNEL_GEMV)
      return fail(MAMBO_EINVAL, "Q4_K runs on the tcgen05 GEMV (MAMBO_KERNEL_GEMV) only");
    if (cfg->warps != 0 && cfg->warps != 8) return fail(MAMBO_EINVAL, "Q4_K decodes with 8 decoder warps");
    if (cfg->loader != 0) return fail(MAMBO_EINVAL, "Q4_K streams the packed records (loader 0)");
    if (cfg->split < 0 || cfg->split > 2)
      return fail(MAMBO_EINVAL, "split must be 0 (stream-K), 1 (row tile per CTA) or 2 (cluster K-split)");
    if (cfg->stages != 0) d.stages = cfg->stages;
    d.split = cfg->split;
    d.prefetch = cfg->prefetch;
  }
  if (d.stages < 2 || d.stages > gemv_tm_max_stages())
    return fail(MAMBO_EINVAL, "stages must be in [2, %d]", gemv_tm_max_stages());
  if (d.prefetch < 0 || d.prefetch > 64) return fail(MAMBO_EINVAL, "prefetch must be in [0, 64]");
  const uint32_t smem = q4k_gemv_smem_bytes(gemv_nt_for(mc), d.stages, d.split == 2 ? 2 : 0);
  if ((int)smem > info.max_smem_optin)
    return fail(MAMBO_EINVAL, "configuration needs %u bytes of shared memory (device allows %d)", smem,
                info.max_smem_optin);
  *c = d;
  return MAMBO_OK;
}

size_t q4k_gemv_workspace(const GemvPlan& P) {
  return P.counters_bytes + P.partial_bytes + P.xcopy_bytes + P.xscopy_bytes;
}

size_t q4k_plan_bytes(int64_t m, int64_t n_rows, int64_t n_blocks, const MamboLinearConfig* cfg) {
  int st;
  DeviceInfo info = device_info(&st);
  if (st != MAMBO_OK || info.sms <= 0) {
    info.sms = 148;
    info.max_smem_optin = kSmemOptinDefault;
  }
  MamboLinearConfig c;
  const int64_t mc = m < 32 ? m : 32;
  if (q4k_config(cfg, mc, n_rows, n_blocks, info, &c) != MAMBO_OK) return 0;
  return q4k_gemv_workspace(plan_gemv(mc, n_rows, n_blocks, c, info.sms, info.max_smem_optin, true));
}

int q4k_linear_impl(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, const float* xsum,
                    int64_t ldsum, int64_t m, const void* packed, int64_t n_rows, int64_t n_blocks, void* out,
                    int out_dtype, int64_t ldo, const MamboLinearConfig* cfg, void* workspace, size_t workspace_bytes,
                    cudaStream_t stream) {
  if (!xq || !xs || !xsum || !packed || !out) return fail(MAMBO_EINVAL, "null pointer");
  if (n_rows < 1 || n_blocks < 1) return fail(MAMBO_EINVAL, "Q4_K weight must have positive N and K");
  if (n_rows > (int64_t)1 << 24 || n_blocks > 4096) return fail(MAMBO_EINVAL, "Q4_K weight too large");
  const int64_t k = n_blocks * 256;
  if (m < 1) return fail(MAMBO_EINVAL, "x_values must be uint8 [M,K] with M >= 1");
  if (ldxq < k || ldxs < k / 32 || ldsum < k / 32) return fail(MAMBO_EINVAL, "activation row stride smaller than the row");
  if ((uintptr_t)xsum % 16 || ldsum % 4)
    return fail(MAMBO_EINVAL, "x_sums must be 16-byte aligned with a row stride that is a multiple of 4");
  if ((uintptr_t)packed % 16) return fail(MAMBO_EINVAL, "the packed weight buffer must be 16-byte aligned");
  if (out_dtype != MAMBO_F32 && out_dtype != MAMBO_BF16) return fail(MAMBO_EINVAL, "out must be f32 or bf16");
  if (ldo < n_rows) return fail(MAMBO_EINVAL, "out row stride is smaller than N");
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  const int64_t m_chunk_max = 32;
  const size_t esz = out_dtype == MAMBO_BF16 ? 2 : 4;
  for (int64_t m0 = 0; m0 < m; m0 += m_chunk_max) {
    const int64_t mc = (m - m0) < m_chunk_max ? (m - m0) : m_chunk_max;
    MamboLinearConfig c;
    st = q4k_config(cfg, mc, n_rows, n_blocks, info, &c);
    if (st != MAMBO_OK) return st;
    const GemvPlan P = plan_gemv(mc, n_rows, n_blocks, c, info.sms, info.max_smem_optin, true);
    if ((size_t)P.counter_slots * sizeof(int) > kGemvCounterBytes)
      return fail(MAMBO_EINVAL, "N=%lld needs more split-K counters than the workspace holds", (long long)n_rows);
    const size_t need = q4k_gemv_workspace(P);
    if (!workspace || workspace_bytes < need)
      return fail(MAMBO_EWORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    if ((uintptr_t)workspace % 256) return fail(MAMBO_EINVAL, "workspace must be 256-byte aligned");
    uint8_t* xcopy = (uint8_t*)workspace + P.counters_bytes + P.partial_bytes;
    GemvTmMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    st = gemv_activation_maps(xq + m0 * ldxq, ldxq, xs + m0 * ldxs, ldxs, mc, n_blocks, (int)mc, xcopy,
                              xcopy + P.xcopy_bytes, &maps, stream);
    if (st != MAMBO_OK) return st;
    GemvTmParams p{};
    p.m = (int)mc;
    p.n_rows = (int)n_rows;
    p.n_blocks = (int)n_blocks;
    p.packed = (const uint8_t*)packed;
    p.out = (uint8_t*)out + m0 * ldo * esz;
    p.out_bf16 = out_dtype == MAMBO_BF16;
    p.ldo = ldo;
    p.partials = (float*)((uint8_t*)workspace + P.counters_bytes);
    p.counters = (int*)workspace;
    p.stages = c.stages;
    p.prefetch = c.prefetch;
    p.kparts = P.kparts;
    p.row_tiles = P.row_tiles;
    p.total_units = P.units;
    p.xsum = xsum + m0 * ldsum;
    p.ldsum = ldsum;
    p.box_rows = (int)mc;
    cudaError_t e = launch_gemv_tm(p, P.nt, 8, maps, P.grid, stream, true);
    if (e != cudaSuccess) return cuda_fail(e, "q4k_gemv_tm");
  }
  return ok();
}

}  // namespace

extern "C" {

size_t mambo_q4k_packed_bytes(int64_t n_rows, int64_t n_blocks) {
  if (n_rows < 1 || n_blocks < 1) return 0;
  return (size_t)((n_rows + 127) / 128) * (size_t)n_blocks * kQ4kRecordBytes;
}

int mambo_q4k_pack(const uint8_t* raw, int64_t n_rows, int64_t n_blocks, int64_t stride_row, int64_t stride_block,
                   int64_t stride_byte, void* packed, mambo_stream_t stream) {
  if (!raw || !packed) return fail(MAMBO_EINVAL, "null pointer");
  if (n_rows < 1 || n_blocks < 1) return fail(MAMBO_EINVAL, "Q4_K weight must have positive N and K");
  if ((uintptr_t)packed % 16) return fail(MAMBO_EINVAL, "the packed buffer must be 16-byte aligned");
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  Q4kPackParams p{raw, n_rows, n_blocks, stride_row, stride_block, stride_byte, (uint8_t*)packed};
  cudaError_t e = launch_q4k_pack(p, info.sms, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "q4k_pack");
  return ok();
}

int mambo_quantize_mxfp8_sums(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, uint8_t* q, int64_t ldq,
                              uint8_t* s, int64_t lds, float* sums, int64_t ld_sums, int rounding,
                              mambo_stream_t stream) {
  if (!x || !q || !s || !sums) return fail(MAMBO_EINVAL, "null pointer");
  if (x_dtype != MAMBO_F32 && x_dtype != MAMBO_BF16) return fail(MAMBO_EINVAL, "activation must be f32 or bf16");
  if (m < 1 || k < 32 || k % 32) return fail(MAMBO_EINVAL, "activation must be [M,K] with K divisible by 32");
  if (ldx < k || ldq < k || lds < k / 32 || ld_sums < k / 32)
    return fail(MAMBO_EINVAL, "row stride smaller than the row");
  if (rounding != MAMBO_ROUND_NEAREST_EVEN && rounding != MAMBO_ROUND_TIES_DOWN)
    return fail(MAMBO_EINVAL, "unknown rounding mode %d", rounding);
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  QuantParams p{x, m, k, ldx, q, ldq, s, lds, sums, ld_sums};
  cudaError_t e = launch_quantize_mxfp8(p, x_dtype, rounding, info.sms, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "quantize_mxfp8 (sums)");
  return ok();
}

size_t mambo_q4k_linear_workspace_bytes(int64_t m, int64_t n_rows, int64_t n_blocks, const MamboLinearConfig* cfg) {
  if (m < 1 || n_rows < 1 || n_blocks < 1) return 0;
  return q4k_plan_bytes(m, n_rows, n_blocks, cfg);
}

int mambo_q4k_linear(const uint8_t* xq, int64_t ldxq, const uint8_t* xs, int64_t ldxs, const float* xsum,
                     int64_t ldsum, int64_t m, const void* packed, int64_t n_rows, int64_t n_blocks, void* out,
                     int out_dtype, int64_t ldo, const MamboLinearConfig* cfg, void* workspace,
                     size_t workspace_bytes, mambo_stream_t stream) {
  return q4k_linear_impl(xq, ldxq, xs, ldxs, xsum, ldsum, m, packed, n_rows, n_blocks, out, out_dtype, ldo, cfg,
                         workspace, workspace_bytes, (cudaStream_t)stream);
}

size_t mambo_q4k_linear_fused_workspace_bytes(int64_t m, int64_t n_rows, int64_t n_blocks,
                                              const MamboLinearConfig* cfg) {
  if (m < 1 || n_rows < 1 || n_blocks < 1) return 0;
  const int64_t k = n_blocks * 256;
  return align256(q4k_plan_bytes(m, n_rows, n_blocks, cfg)) + align256((size_t)(m * k)) +
         align256((size_t)(m * xs_copy_stride(n_blocks))) + align256((size_t)(m * (k / 32)) * sizeof(float));
}

int mambo_q4k_linear_fused(const void* x, int x_dtype, int64_t ldx, int64_t m, const void* packed, int64_t n_rows,
                           int64_t n_blocks, void* out, int out_dtype, int64_t ldo, const MamboLinearConfig* cfg,
                           void* workspace, size_t workspace_bytes, mambo_stream_t stream) {
  if (!x || !packed || !out) return fail(MAMBO_EINVAL, "null pointer");
  if (m < 1 || n_rows < 1 || n_blocks < 1) return fail(MAMBO_EINVAL, "shapes must be positive");
  const size_t need = mambo_q4k_linear_fused_workspace_bytes(m, n_rows, n_blocks, cfg);
  if (!workspace || workspace_bytes < need)
    return fail(MAMBO_EWORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if ((uintptr_t)workspace % 256) return fail(MAMBO_EINVAL, "workspace must be 256-byte aligned");
  const int64_t k = n_blocks * 256, lds = xs_copy_stride(n_blocks);
  const size_t gemv_bytes = align256(q4k_plan_bytes(m, n_rows, n_blocks, cfg));
  uint8_t* xq = (uint8_t*)workspace + gemv_bytes;
  uint8_t* xs = xq + align256((size_t)(m * k));
  float* xsum = (float*)(xs + align256((size_t)(m * lds)));
  int st = mambo_quantize_mxfp8_sums(x, x_dtype, m, k, ldx, xq, k, xs, lds, xsum, k / 32, MAMBO_ROUND_NEAREST_EVEN,
                                     stream);
  if (st != MAMBO_OK) return st;
  return q4k_linear_impl(xq, k, xs, lds, xsum, k / 32, m, packed, n_rows, n_blocks, out, out_dtype, ldo, cfg,
                         workspace, gemv_bytes, (cudaStream_t)stream);
}

}  // extern "C"
static_assert(MAMBO_Q4K_RECORD_BYTES == kQ4kRecordBytes, "Q4_K record size of the C ABI and of the kernel");

// ---- Grouped Q4_K linears (a quantization pre-pass with group sums, then one grouped GEMV launch)

namespace {

bool q4k_group_fusable(const MamboQ4KItem* items, int count) {
  if (count < 1 || count > kGemvMaxItems) return false;
  int64_t tiles = 0, units = 0;
  for (int i = 0; i < count; ++i) {
    const MamboQ4KItem& it = items[i];
    if (it.x_dtype != MAMBO_BF16 || it.m < 1 || it.m >= kGemmMinTokens) return false;
    if ((uintptr_t)it.x % 16 || it.ldx % 8 || (uintptr_t)it.packed % 16 || it.n_rows % 8) return false;
    const int64_t rt = (it.n_rows + 127) / 128;
    tiles += rt;
    units += rt * it.n_blocks;
  }
  return (size_t)tiles * 4 * sizeof(int) <= kGemvCounterBytes && units < (int64_t)1 << 30;
}

int q4k_group_nt(const MamboQ4KItem* items, int count) {
  int64_t m = 1;
  for (int i = 0; i < count; ++i) m = items[i].m > m ? items[i].m : m;
  return gemv_nt_for(m);
}

// Workspace of the grouped launch: counters, stream-K partials, the pre-pass's activation tiles
// (one per item and K block), then each item's group sums [m][K/32] (256-byte aligned per item).
size_t q4k_group_bytes(const MamboQ4KItem* items, int count, int sms, size_t* tiles_off, size_t* sums_off) {
  const int nt = q4k_group_nt(items, count);
  size_t tiles = 0, sums = 0;
  for (int i = 0; i < count; ++i) {
    tiles += (size_t)items[i].n_blocks;
    sums += align256((size_t)items[i].m * (size_t)items[i].n_blocks * 8 * sizeof(float));
  }
  const size_t t0 = kCounterBytes + group_partial_bytes(nt, sms);
  const size_t s0 = t0 + align256(tiles * gemv_xtile_bytes(nt));
  if (tiles_off) *tiles_off = t0;
  if (sums_off) *sums_off = s0;
  return s0 + sums;
}

}  // namespace

extern "C" {

size_t mambo_q4k_linear_group_workspace_bytes(const MamboQ4KItem* items, int count) {
  if (!items || count < 1) return 0;
  int st;
  DeviceInfo info = device_info(&st);
  const int sms = (st == MAMBO_OK && info.sms > 0) ? info.sms : 148;
  size_t need = 0;
  for (int i = 0; i < count; ++i) {
    if (items[i].m < 1 || items[i].n_rows < 1 || items[i].n_blocks < 1) return 0;
    const size_t b = mambo_q4k_linear_fused_workspace_bytes(items[i].m, items[i].n_rows, items[i].n_blocks, nullptr);
    need = b > need ? b : need;  // the per-item path, when the group does not qualify
  }
  if (q4k_group_fusable(items, count)) {
    const size_t g = q4k_group_bytes(items, count, sms, nullptr, nullptr);
    need = g > need ? g : need;
  }
  return need;
}

int mambo_q4k_linear_group(const MamboQ4KItem* items, int count, void* workspace, size_t workspace_bytes,
                           mambo_stream_t stream) {
  if (!items) return fail(MAMBO_EINVAL, "null pointer");
  if (count < 1) return fail(MAMBO_EINVAL, "a group needs at least one linear");
  for (int i = 0; i < count; ++i) {
    const MamboQ4KItem& it = items[i];
    if (!it.x || !it.packed || !it.out) return fail(MAMBO_EINVAL, "item %d: null pointer", i);
    if (it.m < 1 || it.n_rows < 1 || it.n_blocks < 1) return fail(MAMBO_EINVAL, "item %d: shapes must be positive", i);
    if (it.n_rows > (int64_t)1 << 24 || it.n_blocks > 4096) return fail(MAMBO_EINVAL, "item %d: weight too large", i);
    if (it.x_dtype != MAMBO_F32 && it.x_dtype != MAMBO_BF16)
      return fail(MAMBO_EINVAL, "item %d: activation must be f32 or bf16", i);
    if (it.ldx < it.n_blocks * 256) return fail(MAMBO_EINVAL, "item %d: activation must be [M,K]", i);
    if (it.out_dtype != MAMBO_F32 && it.out_dtype != MAMBO_BF16)
      return fail(MAMBO_EINVAL, "item %d: out must be f32 or bf16", i);
    if (it.ldo < it.n_rows) return fail(MAMBO_EINVAL, "item %d: out row stride is smaller than N", i);
  }
  if (!workspace || (uintptr_t)workspace % 256) return fail(MAMBO_EINVAL, "workspace must be 256-byte aligned");
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  if (!q4k_group_fusable(items, count)) {
    for (int i = 0; i < count; ++i) {
      const MamboQ4KItem& it = items[i];
      st = mambo_q4k_linear_fused(it.x, it.x_dtype, it.ldx, it.m, it.packed, it.n_rows, it.n_blocks, it.out,
                                  it.out_dtype, it.ldo, nullptr, workspace, workspace_bytes, stream);
      if (st != MAMBO_OK) return st;
    }
    return ok();
  }
  const int nt = q4k_group_nt(items, count);
  size_t tiles_off = 0, sums_off = 0;
  const size_t need = q4k_group_bytes(items, count, info.sms, &tiles_off, &sums_off);
  if (workspace_bytes < need)
    return fail(MAMBO_EWORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  GemvGroupPre g;
  std::memset(&g, 0, sizeof(g));
  g.count = count;
  GroupXtilesParams xp;
  std::memset(&xp, 0, sizeof(xp));
  int units = 0, tiles = 0, xtiles = 0;
  const int box = 8 * nt;
  float* sums = (float*)((uint8_t*)workspace + sums_off);
  for (int i = 0; i < count; ++i) {
    const MamboQ4KItem& it = items[i];
    const int rt = (int)((it.n_rows + 127) / 128);
    GemvItem& gi = g.items[i];
    gi.packed = (const uint8_t*)it.packed;
    gi.x = (const uint16_t*)it.x;
    gi.out = it.out;
    gi.ldx = it.ldx;
    gi.ldo = it.ldo;
    gi.n_rows = (int)it.n_rows;
    gi.n_blocks = (int)it.n_blocks;
    gi.m = (int)it.m;
    gi.out_bf16 = it.out_dtype == MAMBO_BF16;
    gi.unit0 = units;
    gi.tile0 = tiles;
    gi.xt0 = xtiles;
    gi.xsum = sums;
    gi.ldsum = it.n_blocks * 8;
    xp.items[i] = GroupXtilesParams::Item{gi.x, gi.ldx, gi.m, gi.n_blocks, gi.xt0, sums, gi.ldsum};
    sums += align256((size_t)it.m * (size_t)it.n_blocks * 8 * sizeof(float)) / sizeof(float);
    xtiles += gi.n_blocks;
    units += rt * gi.n_blocks;
    tiles += rt;
  }
  GemvTmParams p;
  std::memset(&p, 0, sizeof(p));
  p.m = box;
  p.n_blocks = 1;  // per item in the group
  p.packed = g.items[0].packed;
  p.counters = (int*)workspace;
  p.partials = (float*)((uint8_t*)workspace + kCounterBytes);
  p.stages = 8;
  while (p.stages > 2 && (int)gemv_tm_smem_bytes(nt, p.stages, 0, true, true) > info.max_smem_optin) --p.stages;
  if ((int)gemv_tm_smem_bytes(nt, p.stages, 0, true, true) > info.max_smem_optin)
    return fail(MAMBO_EINVAL, "the grouped Q4_K GEMV does not fit in shared memory");
  p.row_tiles = tiles;
  p.total_units = units;
  int grid = units < info.sms ? units : info.sms;
  if (grid > kGemvMaxGrid) grid = kGemvMaxGrid;
  split_group_units(g, units, grid, g.cta_start, true);
  xp.count = count;
  xp.total_tiles = xtiles;
  xp.box = box;
  xp.tiles = (uint8_t*)workspace + tiles_off;
  cudaError_t e = launch_group_xtiles(xp, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "group_xtiles_kernel (Q4_K)");
  g.xtiles = xp.tiles;
  e = launch_gemv_tm_group_pre(p, g, nt, grid, (cudaStream_t)stream, true);
  if (e != cudaSuccess) return cuda_fail(e, "iq3s_gemv_tm_kernel (Q4_K group)");
  return ok();
}

}  // extern "C"

// --------------------------------------------------------------------------
// Row split with the all-reduce fused into the GEMV (mambo_iq3s_linear_fused_ar)
// --------------------------------------------------------------------------
static_assert(MAMBO_AR_HANDLE_BYTES == sizeof(cudaIpcMemHandle_t), "IPC handle size of the C ABI and of CUDA");

struct MamboArComm {
  int world, rank, device, max_rows;
  uint8_t* local;  // this rank's exchange buffer (cudaMalloc, exported by IPC)
  size_t bytes;
  GemvAr ar;       // every rank's buffer as mapped here
  bool connected;
};

namespace {

size_t ar_buffer_bytes(int world, int max_rows) { return gemv_ar_slot_bytes(world, max_rows) + 256; }

}  // namespace

extern "C" {

int mambo_ar_comm_create(int world, int rank, int64_t max_rows, MamboArComm** comm, void* ipc_handle) {
  if (!comm || !ipc_handle) return fail(MAMBO_EINVAL, "null pointer");
  *comm = nullptr;
  if (world < 1 || world > kGemvArMaxRanks) return fail(MAMBO_EINVAL, "world must be 1..%d", kGemvArMaxRanks);
  if (rank < 0 || rank >= world) return fail(MAMBO_EINVAL, "rank must be in [0, world)");
  if (max_rows < 128 || max_rows % 128 || max_rows > (1 << 18))
    return fail(MAMBO_EINVAL, "max_rows must be a positive multiple of 128 up to 2^18");
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  MamboArComm* c = new (std::nothrow) MamboArComm{};
  if (!c) return fail(MAMBO_EINVAL, "out of host memory");
  c->world = world;
  c->rank = rank;
  c->max_rows = (int)max_rows;
  cudaGetDevice(&c->device);
  c->bytes = ar_buffer_bytes(world, (int)max_rows);
  cudaError_t e = cudaMalloc((void**)&c->local, c->bytes);
  if (e != cudaSuccess) {
    delete c;
    return cuda_fail(e, "cudaMalloc(exchange buffer)");
  }
  // Tags and epoch start at zero; every launch then tags its words with epoch + 1.
  e = cudaMemset(c->local, 0, c->bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle((cudaIpcMemHandle_t*)ipc_handle, c->local);
  if (e != cudaSuccess) {
    cudaFree(c->local);
    delete c;
    return cuda_fail(e, "exchange buffer set-up");
  }
  c->ar.world = world;
  c->ar.rank = rank;
  c->ar.max_rows = (int)max_rows;
  c->ar.ctl_offset = (uint32_t)gemv_ar_slot_bytes(world, (int)max_rows);
  c->ar.base[rank] = c->local;
  *comm = c;
  return ok();
}

int mambo_ar_comm_connect(MamboArComm* c, const void* ipc_handles) {
  if (!c || !ipc_handles) return fail(MAMBO_EINVAL, "null pointer");
  if (c->connected) return fail(MAMBO_EINVAL, "communicator already connected");
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != c->device) return fail(MAMBO_EINVAL, "connect on the device the communicator was created on");
  const cudaIpcMemHandle_t* h = (const cudaIpcMemHandle_t*)ipc_handles;
  for (int j = 0; j < c->world; ++j) {
    if (j == c->rank) continue;
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h[j], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int i = 0; i < j; ++i)
        if (i != c->rank && c->ar.base[i]) cudaIpcCloseMemHandle(c->ar.base[i]);
      return cuda_fail(e, "cudaIpcOpenMemHandle(peer exchange buffer)");
    }
    c->ar.base[j] = (uint8_t*)p;
  }
  c->connected = true;
  return ok();
}

int mambo_ar_comm_destroy(MamboArComm* c) {
  if (!c) return ok();
  if (c->connected)
    for (int j = 0; j < c->world; ++j)
      if (j != c->rank && c->ar.base[j]) cudaIpcCloseMemHandle(c->ar.base[j]);
  if (c->local) cudaFree(c->local);
  delete c;
  return ok();
}

int mambo_iq3s_linear_fused_ar(const void* x, int x_dtype, int64_t ldx, int64_t m, const MamboIQ3SWeight* w,
                               const uint32_t* fp8_table, void* out, int out_dtype, int64_t ldo, MamboArComm* comm,
                               const MamboLinearConfig* cfg, void* workspace, size_t workspace_bytes,
                               mambo_stream_t stream) {
  if (!x || !w || !fp8_table || !out || !comm) return fail(MAMBO_EINVAL, "null pointer");
  if (!comm->connected) return fail(MAMBO_EINVAL, "communicator not connected");
  if (!weight_fields_ok(w) || !w->packed) return fail(MAMBO_EINVAL, "the fused all-reduce needs the packed weight copy");
  if (x_dtype != MAMBO_BF16) return fail(MAMBO_EINVAL, "the fused all-reduce takes bf16 activations");
  if (m < 1 || m >= kGemmMinTokens) return fail(MAMBO_EINVAL, "the fused all-reduce takes 1 to %d tokens",
                                                 kGemmMinTokens - 1);
  if (w->n_rows < 1 || w->n_blocks < 1 || w->n_rows % 8) return fail(MAMBO_EINVAL, "weight must be [N, K] with N % 8 == 0");
  const int64_t k = w->n_blocks * 256;
  if (ldx < k || ldx % 8 || (uintptr_t)x % 16) return fail(MAMBO_EINVAL, "bf16 activations need 16-byte aligned rows of K");
  if (out_dtype != MAMBO_F32 && out_dtype != MAMBO_BF16) return fail(MAMBO_EINVAL, "out must be f32 or bf16");
  if (ldo < w->n_rows) return fail(MAMBO_EINVAL, "out row stride is smaller than N");
  if ((w->n_rows + 127) / 128 * 128 > comm->max_rows)
    return fail(MAMBO_EINVAL, "N=%lld exceeds the communicator's %d rows", (long long)w->n_rows, comm->max_rows);
  const uintptr_t fields[6] = {(uintptr_t)w->d, (uintptr_t)w->qs, (uintptr_t)w->qh, (uintptr_t)w->signs,
                               (uintptr_t)w->scales, (uintptr_t)w->packed};
  for (uintptr_t f : fields)
    if (f % 16) return fail(MAMBO_EINVAL, "weight fields must be 16-byte aligned");
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != MAMBO_OK) return st;
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != comm->device) return fail(MAMBO_EINVAL, "call on the device the communicator was created on");
  MamboLinearConfig c;
  if (cfg) c = *cfg; else default_config(m, w->n_rows, w->n_blocks, &c, info.max_smem_optin, info.sms);
  resolve_auto(&c, m, w->n_rows, w->n_blocks, info.max_smem_optin, info.sms);
  // Every row's sum over this rank's K slice forms in one CTA (whole row
  // tiles, or a cluster K split summed in its rank 0): the exchange runs there.
  c.kernel = MAMBO_KERNEL_GEMV;
  c.loader = 0;
  c.warps = 8;
  if (c.split != 1) c.split = 2;
  st = validate_config(&c, m, w->n_blocks, info);
  if (st != MAMBO_OK) return st;
  const GemvPlan P = plan_gemv(m, w->n_rows, w->n_blocks, c, info.sms, info.max_smem_optin);
  if (P.kparts < 1) return fail(MAMBO_EINVAL, "no whole-tile plan for this shape");
  while (c.stages > 2 && (int)gemv_tm_smem_bytes(P.nt, c.stages, P.kparts, true) > info.max_smem_optin) --c.stages;
  if ((int)gemv_tm_smem_bytes(P.nt, c.stages, P.kparts, true) > info.max_smem_optin)
    return fail(MAMBO_EINVAL, "the fused all-reduce GEMV does not fit in shared memory");
  const size_t need = P.counters_bytes + P.partial_bytes;
  if (!workspace || workspace_bytes < need)
    return fail(MAMBO_EWORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if ((uintptr_t)workspace % 256) return fail(MAMBO_EINVAL, "workspace must be 256-byte aligned");
  GemvTmMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  if (!make_gemv_xb_map((const uint16_t*)x, ldx, (int)m, (int)k, 8 * P.nt, &maps.xb))
    return fail(MAMBO_EINVAL, "bf16 activations need 16-byte aligned rows");
  GemvTmParams p{};
  p.m = (int)m;
  p.n_rows = (int)w->n_rows;
  p.n_blocks = (int)w->n_blocks;
  p.d = (const uint8_t*)w->d;
  p.qs = (const uint8_t*)w->qs;
  p.qh = (const uint8_t*)w->qh;
  p.signs = (const uint8_t*)w->signs;
  p.scales = (const uint8_t*)w->scales;
  p.packed = (const uint8_t*)w->packed;
  p.table = fp8_table;
  p.out = out;
  p.out_bf16 = out_dtype == MAMBO_BF16;
  p.ldo = ldo;
  p.counters = (int*)workspace;
  p.partials = (float*)((uint8_t*)workspace + P.counters_bytes);
  p.stages = c.stages;
  p.prefetch = c.prefetch;
  p.kparts = P.kparts;
  p.row_tiles = P.row_tiles;
  p.total_units = P.units;
  p.x_bf16 = (const uint16_t*)x;
  p.ldx = ldx;
  cudaError_t e = launch_gemv_tm_ar(p, comm->ar, P.nt, maps, P.grid, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "iq3s_gemv_tm_kernel (fused all-reduce)");
  return ok();
}

}  // extern "C"
