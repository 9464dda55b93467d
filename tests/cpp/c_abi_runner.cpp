// A native consumer of libmambo_b200.so: the whole IQ3_S x MXFP8 linear path
// driven through the C ABI (include/mambo_b200.h) from C++, with no Python.
// It plays the role of the reference's C++ loader test
// (tests/cpp/loadtest/loadtest.cpp:201-412, which loads the exported cubins
// and launches them): prepare and pack a weight, quantize activations, run the
// two-step, fused and grouped linears, and check every result against the C
// oracle (oracle/iq3s_ref.c) on the host.
//
// Usage: c_abi_runner GRID.bin FP8_TABLE.bin
//   GRID.bin       512 little-endian uint32: the IQ3_S codebook magnitudes
//   FP8_TABLE.bin  512 uint32: the same codebook re-encoded as E4M3 bytes
// (the test that builds this program writes both from the GGUF format's own
// package). Exit status 0 when every check passes.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "mambo_b200.h"

extern "C" {
void oracle_mxfp8_quantize(const float* x, int64_t m, int64_t k, int rounding, uint8_t* q, uint8_t* s);
int oracle_iq3s_linear(const uint8_t* xq, const uint8_t* xs, int64_t m, int64_t k, const uint8_t* raw,
                       int64_t n_rows, const uint32_t* grid, double* out, int64_t ldo);
}

namespace {

int g_failures = 0;

void check(bool ok, const char* what) {
  std::printf("%s %s\n", ok ? "ok  " : "FAIL", what);
  if (!ok) ++g_failures;
}

void mambo_or_die(int status, const char* call) {
  if (status == MAMBO_OK) return;
  char msg[512];
  mambo_last_error(msg, sizeof msg);
  std::fprintf(stderr, "%s: status %d: %s\n", call, status, msg);
  std::exit(2);
}

void cuda_or_die(cudaError_t e, const char* call) {
  if (e == cudaSuccess) return;
  std::fprintf(stderr, "%s: %s\n", call, cudaGetErrorString(e));
  std::exit(2);
}

#define MAMBO(call) mambo_or_die((call), #call)
#define CUDA(call) cuda_or_die((call), #call)

struct Rng {  // xorshift64*
  uint64_t s;
  uint32_t next() {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return (uint32_t)((s * 2685821657736338717ull) >> 32);
  }
  float uniform(float lo, float hi) { return lo + (hi - lo) * (float)(next() >> 8) * (1.0f / 16777216.0f); }
};

// Random GGUF IQ3_S blocks [n][b][110]; d is a float16 in [2^-10, 2^-7).
std::vector<uint8_t> make_weight(int64_t n, int64_t b, uint64_t seed) {
  Rng r{seed};
  std::vector<uint8_t> raw((size_t)(n * b * 110));
  for (auto& v : raw) v = (uint8_t)r.next();
  for (int64_t i = 0; i < n * b; ++i) {
    const uint16_t d = (uint16_t)(((5u + r.next() % 3u) << 10) | (r.next() & 0x3FFu));
    std::memcpy(&raw[(size_t)i * 110], &d, 2);
  }
  return raw;
}

uint16_t bf16_of(float f) {  // round to nearest even (finite inputs)
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float float_of_bf16(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

template <class T>
T* device_copy(const std::vector<T>& host) {
  T* p = nullptr;
  CUDA(cudaMalloc(&p, host.size() * sizeof(T)));
  CUDA(cudaMemcpy(p, host.data(), host.size() * sizeof(T), cudaMemcpyHostToDevice));
  return p;
}

void* device_zeros(size_t bytes) {
  void* p = nullptr;
  CUDA(cudaMalloc(&p, bytes ? bytes : 1));
  CUDA(cudaMemset(p, 0, bytes ? bytes : 1));
  return p;
}

template <class T>
std::vector<T> host_copy(const T* dev, size_t count) {
  std::vector<T> h(count);
  CUDA(cudaMemcpy(h.data(), dev, count * sizeof(T), cudaMemcpyDeviceToHost));
  return h;
}

double relative_frobenius(const std::vector<float>& a, const std::vector<double>& ref) {
  double num = 0, den = 0;
  for (size_t i = 0; i < a.size(); ++i) {
    num += ((double)a[i] - ref[i]) * ((double)a[i] - ref[i]);
    den += ref[i] * ref[i];
  }
  return std::sqrt(num / (den > 0 ? den : 1));
}

// A prepared and packed weight on the device.
struct Weight {
  int64_t n, b;
  std::vector<uint8_t> raw;
  MamboIQ3SWeight w;
};

Weight upload_weight(int64_t n, int64_t b, uint64_t seed) {
  Weight out{n, b, make_weight(n, b, seed), {}};
  uint8_t* raw = device_copy(out.raw);
  void* d = device_zeros((size_t)(b * n * 2));
  void* qs = device_zeros((size_t)(b * n * 64));
  void* qh = device_zeros((size_t)(b * n * 8));
  void* signs = device_zeros((size_t)(b * n * 32));
  void* scales = device_zeros((size_t)(b * n * 4));
  MAMBO(mambo_iq3s_prepare(raw, n, b, b * 110, 110, 1, d, qs, qh, signs, scales, nullptr));
  out.w = MamboIQ3SWeight{d, qs, qh, signs, scales, n, b, nullptr};
  void* packed = device_zeros(mambo_iq3s_packed_bytes(n, b));
  MAMBO(mambo_iq3s_pack(&out.w, packed, nullptr));
  out.w.packed = packed;
  CUDA(cudaDeviceSynchronize());
  CUDA(cudaFree(raw));
  return out;
}

std::vector<uint32_t> read_table(const char* path) {
  std::vector<uint32_t> t(512);
  FILE* f = std::fopen(path, "rb");
  if (!f || std::fread(t.data(), 4, 512, f) != 512) {
    std::fprintf(stderr, "cannot read 512 uint32 from %s\n", path);
    std::exit(2);
  }
  std::fclose(f);
  return t;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 3) {
    std::fprintf(stderr, "usage: %s GRID.bin FP8_TABLE.bin\n", argv[0]);
    return 2;
  }
  const std::vector<uint32_t> grid = read_table(argv[1]);
  const std::vector<uint32_t> fp8 = read_table(argv[2]);
  std::printf("library %s\n", mambo_version());
  MAMBO(mambo_device_check());
  uint32_t* table = device_copy(fp8);

  const int64_t n = 1024, b = 8, k = b * 256;
  Weight wt = upload_weight(n, b, 0x5EEDull);

  // Two-step (quantize, then linear), fused, against the C oracle.
  for (int64_t m : {1, 5, 8, 40}) {
    Rng r{0xA11CEull + (uint64_t)m};
    std::vector<uint16_t> xb((size_t)(m * k));
    std::vector<float> xf(xb.size());
    for (size_t i = 0; i < xb.size(); ++i) {
      xb[i] = bf16_of(r.uniform(-3.f, 3.f) * (r.next() % 97 == 0 ? 40.f : 1.f));
      xf[i] = float_of_bf16(xb[i]);
    }
    uint16_t* x = device_copy(xb);
    uint8_t* q = (uint8_t*)device_zeros((size_t)(m * k));
    uint8_t* s = (uint8_t*)device_zeros((size_t)(m * k / 32));
    float* out1 = (float*)device_zeros((size_t)(m * n * 4));
    float* out2 = (float*)device_zeros((size_t)(m * n * 4));
    const size_t wsb = mambo_iq3s_linear_workspace_bytes(m, n, b, nullptr);
    const size_t fwsb = mambo_iq3s_linear_fused_workspace_bytes(m, n, b, nullptr);
    void* ws = device_zeros(wsb);
    void* fws = device_zeros(fwsb);
    MAMBO(mambo_quantize_mxfp8(x, MAMBO_BF16, m, k, k, q, k, s, k / 32, MAMBO_ROUND_NEAREST_EVEN, nullptr));
    MAMBO(mambo_iq3s_linear(q, k, s, k / 32, m, &wt.w, table, out1, MAMBO_F32, n, nullptr, ws, wsb, nullptr));
    MAMBO(mambo_iq3s_linear_fused(x, MAMBO_BF16, k, m, &wt.w, table, out2, MAMBO_F32, n, nullptr, fws, fwsb,
                                  nullptr));
    CUDA(cudaDeviceSynchronize());
    const auto hq = host_copy(q, (size_t)(m * k));
    const auto hs = host_copy(s, (size_t)(m * k / 32));
    const auto y1 = host_copy(out1, (size_t)(m * n));
    const auto y2 = host_copy(out2, (size_t)(m * n));

    std::vector<uint8_t> rq((size_t)(m * k)), rs((size_t)(m * k / 32));
    oracle_mxfp8_quantize(xf.data(), m, k, 0, rq.data(), rs.data());
    std::vector<double> ref((size_t)(m * n));
    if (oracle_iq3s_linear(rq.data(), rs.data(), m, k, wt.raw.data(), n, grid.data(), ref.data(), n) != 0) {
      std::fprintf(stderr, "oracle failed\n");
      return 2;
    }
    char what[160];
    std::snprintf(what, sizeof what, "M=%lld: MXFP8 bytes and scales equal the oracle's", (long long)m);
    check(hq == rq && hs == rs, what);
    const double err = relative_frobenius(y1, ref);
    std::snprintf(what, sizeof what, "M=%lld: linear vs float64 oracle, relative Frobenius %.2e < 1e-4",
                  (long long)m, err);
    check(err < 1e-4, what);
    std::snprintf(what, sizeof what, "M=%lld: fused quantize + linear bit-identical to the two steps",
                  (long long)m);
    check(std::memcmp(y1.data(), y2.data(), y1.size() * 4) == 0, what);
    for (void* p : {(void*)x, (void*)q, (void*)s, (void*)out1, (void*)out2, ws, fws}) CUDA(cudaFree(p));
  }

  // A group of two linears in one call, each against its own fused call.
  Weight w2 = upload_weight(256, 4, 0xBEEFull);
  const int64_t ms[2] = {3, 8};
  const Weight* ws_[2] = {&wt, &w2};
  MamboLinearItem items[2];
  std::vector<void*> bufs;
  for (int i = 0; i < 2; ++i) {
    const int64_t kk = ws_[i]->b * 256, nn = ws_[i]->n;
    Rng r{0xC0FFEEull + (uint64_t)i};
    std::vector<uint16_t> xb((size_t)(ms[i] * kk));
    for (auto& v : xb) v = bf16_of(r.uniform(-2.f, 2.f));
    uint16_t* x = device_copy(xb);
    void* out = device_zeros((size_t)(ms[i] * nn * 4));
    bufs.push_back(x);
    bufs.push_back(out);
    items[i] = MamboLinearItem{x, MAMBO_BF16, kk, ms[i], &ws_[i]->w, out, MAMBO_F32, nn};
  }
  const size_t gwsb = mambo_iq3s_linear_group_workspace_bytes(items, 2);
  void* gws = device_zeros(gwsb);
  MAMBO(mambo_iq3s_linear_group(items, 2, table, gws, gwsb, nullptr));
  CUDA(cudaDeviceSynchronize());
  for (int i = 0; i < 2; ++i) {
    const int64_t nn = ws_[i]->n, bb = ws_[i]->b;
    const size_t count = (size_t)(ms[i] * nn);
    const auto yg = host_copy((const float*)items[i].out, count);
    float* one = (float*)device_zeros(count * 4);
    const size_t fwsb = mambo_iq3s_linear_fused_workspace_bytes(ms[i], nn, bb, nullptr);
    void* fws = device_zeros(fwsb);
    MAMBO(mambo_iq3s_linear_fused(items[i].x, MAMBO_BF16, items[i].ldx, ms[i], &ws_[i]->w, table, one, MAMBO_F32,
                                  nn, nullptr, fws, fwsb, nullptr));
    CUDA(cudaDeviceSynchronize());
    const auto y1 = host_copy(one, count);
    std::vector<double> ref(y1.begin(), y1.end());
    const double err = relative_frobenius(yg, ref);
    char what[160];
    std::snprintf(what, sizeof what, "group item %d (M=%lld, N=%lld): vs its own call, relative Frobenius %.2e < 1e-5",
                  i, (long long)ms[i], (long long)nn, err);
    check(err < 1e-5, what);
    CUDA(cudaFree(one));
    CUDA(cudaFree(fws));
  }
  for (void* p : bufs) CUDA(cudaFree(p));
  CUDA(cudaFree(gws));
  std::printf("%s: %d failure(s)\n", g_failures ? "FAILED" : "PASSED", g_failures);
  return g_failures ? 1 : 0;
}
