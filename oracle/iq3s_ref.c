/*
 * C restatement of the IQ3_S x MXFP8 linear path -- CPU oracle, TEST
 * INFRASTRUCTURE ONLY (used by tests/ and as bench.py's timed CPU baseline;
 * never linked into libmambo_b200).
 *
 * Restates (paths relative to the Menooker/Mambo tree):
 *   - IQ3_S block decode as in ggml's dequantize_row_iq3_s, the CPU decode that
 *     tests/cpp/reference/ggml_reference.cpp:495-510 calls through
 *     traits->to_float, and gguf-py's IQ3_S.dequantize_blocks;
 *   - the float64 dot of tests/cpp/reference/ggml_reference.cpp:508-523;
 *   - MXFP8 quantization of src/python/mambo/kernels/quantize_fp8.py:23-39
 *     (exact power-of-two exponent, RNE) and of the reference test oracle
 *     tests/python/utils/fp8_reference.py:64-86 (ties to the smaller magnitude).
 * The 512-entry codebook is passed in by the caller (it is data of the
 * llama.cpp format, read at run time from gguf-py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define BLOCK_BYTES 110
#define BLOCK_VALUES 256

static float half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  float v;
  if (exp == 0) {
    v = ldexpf((float)man, -24);
  } else if (exp == 31) {
    v = man ? NAN : INFINITY;
  } else {
    v = ldexpf((float)(man | 0x400u), (int)exp - 25);
  }
  uint32_t bits;
  memcpy(&bits, &v, 4);
  bits |= sign;
  memcpy(&v, &bits, 4);
  return v;
}

/* Decode n_blocks consecutive 110-byte blocks into 256 floats each. */
void oracle_iq3s_dequant(const uint8_t* raw, int64_t n_blocks, const uint32_t* grid, float* out) {
  for (int64_t b = 0; b < n_blocks; ++b) {
    const uint8_t* blk = raw + b * BLOCK_BYTES;
    const float d = half_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
    const uint8_t* qs = blk + 2;
    const uint8_t* qh = blk + 66;
    const uint8_t* signs = blk + 74;
    const uint8_t* scales = blk + 106;
    float* y = out + b * BLOCK_VALUES;
    for (int g = 0; g < 8; ++g) {
      const int nib = (scales[g / 2] >> (4 * (g % 2))) & 0xF;
      const float dg = d * (float)(1 + 2 * nib);
      for (int c = 0; c < 8; ++c) {
        const int code = 8 * g + c;
        const uint32_t idx = qs[code] | (((qh[g] >> c) & 1u) << 8);
        const uint32_t word = grid[idx];
        for (int j = 0; j < 4; ++j) {
          const int k = 4 * code + j;
          const float mag = (float)((word >> (8 * j)) & 0xFFu);
          const int neg = (signs[k / 8] >> (k % 8)) & 1;
          y[k] = neg ? -(dg * mag) : dg * mag;
        }
      }
    }
  }
}

/* Nearest E4M3FN code of a finite |y| <= 448 (saturating); rounding 0 = RNE,
 * 1 = exact ties to the smaller magnitude. */
static uint8_t encode_e4m3(double y, int rounding) {
  double a = fabs(y);
  int ex;
  frexp(a, &ex);
  int e = (a < ldexp(1.0, -6)) ? -6 : ex - 1;
  double r = ldexp(a, 3 - e);
  double fl = floor(r);
  double frac = r - fl;
  double q;
  if (frac > 0.5) {
    q = fl + 1.0;
  } else if (frac < 0.5) {
    q = fl;
  } else if (rounding == 0) {
    q = (fmod(fl, 2.0) == 0.0) ? fl : fl + 1.0;
  } else {
    q = fl;
  }
  long code = (e == -6) ? (long)q : ((long)(e + 7) << 3) + (long)q - 8;
  if (code > 0x7E) code = 0x7E;
  if (signbit(y)) code |= 0x80;
  return (uint8_t)code;
}

static int mxfp8_exponent(double amax) {
  if (amax == 0.0) return 0;
  int ex;
  double mant = frexp(amax, &ex); /* 448 = 0.875 * 2^9 */
  int e = (mant <= 0.875) ? ex - 9 : ex - 8;
  if (e < -127) e = -127;
  if (e > 127) e = 127;
  return e;
}

void oracle_mxfp8_quantize(const float* x, int64_t m, int64_t k, int rounding, uint8_t* q, uint8_t* s) {
  for (int64_t i = 0; i < m; ++i) {
    for (int64_t g = 0; g < k / 32; ++g) {
      const float* v = x + i * k + g * 32;
      double amax = 0.0;
      for (int j = 0; j < 32; ++j) {
        double a = fabs((double)v[j]);
        if (a > amax) amax = a;
      }
      const int e = mxfp8_exponent(amax);
      s[i * (k / 32) + g] = (uint8_t)(e + 127);
      for (int j = 0; j < 32; ++j) q[i * k + g * 32 + j] = encode_e4m3(ldexp((double)v[j], -e), rounding);
    }
  }
}

static double e4m3_value(uint8_t b) {
  int exp = (b >> 3) & 0xF, man = b & 7;
  double v = exp == 0 ? ldexp((double)man, -9) : ldexp(1.0 + man / 8.0, exp - 7);
  if (exp == 15 && man == 7) v = NAN;
  return (b & 0x80) ? -v : v;
}

/* out[i*ldo + r] (float64) = decode_mxfp8(xq, xs)[i] . dequant(raw row r), for
 * i < M and r < n_rows; raw holds n_rows rows of K/256 blocks. Callers split
 * the rows across host threads (ctypes releases the GIL during the call). */
int oracle_iq3s_linear(const uint8_t* xq, const uint8_t* xs, int64_t m, int64_t k, const uint8_t* raw, int64_t n_rows,
                       const uint32_t* grid, double* out, int64_t ldo) {
  const int64_t nb = k / BLOCK_VALUES;
  double lut[256];
  for (int b = 0; b < 256; ++b) lut[b] = e4m3_value((uint8_t)b);
  float* wrow = (float*)malloc(sizeof(float) * (size_t)k);
  if (wrow == NULL) return 1;
  for (int64_t r = 0; r < n_rows; ++r) {
    oracle_iq3s_dequant(raw + r * nb * BLOCK_BYTES, nb, grid, wrow);
    for (int64_t i = 0; i < m; ++i) {
      double acc = 0.0;
      for (int64_t g = 0; g < k / 32; ++g) {
        const double sc = ldexp(1.0, (int)xs[i * (k / 32) + g] - 127);
        double part = 0.0;
        for (int j = 0; j < 32; ++j) part += lut[xq[i * k + g * 32 + j]] * (double)wrow[g * 32 + j];
        acc += part * sc;
      }
      out[i * ldo + r] = acc;
    }
  }
  free(wrow);
  return 0;
}
