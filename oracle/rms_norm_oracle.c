/*
 * CPU oracle for the fused residual-add + RMSNorm path and the companion ReLU.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
 * compared against; it is never linked into, loaded by or called from the
 * product library.  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg may use it.
 *
 * It restates, element by element and in plain C, the arithmetic of the
 * reference implementation (HydraQYH/hp_rms_norm):
 *
 *   hp_rms_norm/csrc/cuda/hp_rms_norm.cuh:186-193  s   = f32(x) + f32(r)   (fp32 add)
 *                                                  r'  = round_T(s)         (RN-even)
 *                                                  ss += s * s              (unrounded s)
 *   hp_rms_norm/csrc/cuda/hp_rms_norm.cuh:231      inv = rsqrt(eps + ss / H)
 *   hp_rms_norm/csrc/cuda/hp_rms_norm.cuh:104-110  y   = round_T(f32(r') * f32(w) * inv)
 *
 * and the reference test's eager formula (test/test_hp_rms_norm.py:6-19:
 * inp_res = inp + res in T, then torch.rms_norm on the rounded sum), which
 * differs only in squaring the rounded residual: select it with
 * ss_mode = ORACLE_SS_ROUNDED.
 *
 * The sum of squares is accumulated in double and the inverse RMS is computed
 * in double then rounded once to float, so the oracle is at least as accurate
 * as any fp32-accumulating kernel.  The output product is then formed in float,
 * left to right, exactly as hp_rms_norm.cuh:108-109 writes it.
 *
 * ReLU follows torch.relu as computed on CUDA, bit for bit: x <= 0 ? +0 : x,
 * so negatives, -inf and -0.0 become +0 and NaNs pass through with their bits
 * (torch's CPU kernel differs in keeping -0.0 and rewriting NaN payloads).
 * (The reference's "relu" kernel,
 * hp_rms_norm/csrc/cuda/activation_kernels.cuh:99-119, is a plain copy; the
 * product follows torch.relu instead.)
 *
 * Storage is raw 16-bit patterns (uint16_t) for both bf16 and fp16.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_BF16 0
#define ORACLE_FP16 1
#define ORACLE_SS_UNROUNDED 0 /* the CUDA kernel (hp_rms_norm.cuh:190-193) */
#define ORACLE_SS_ROUNDED 1   /* the test's eager formula (test_hp_rms_norm.py:13-19) */

/* ---- bf16 ------------------------------------------------------------- */

static inline float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* Round to nearest, ties to even.  NaN maps to 0x7fff, the canonical NaN the
 * GPU's cvt.rn.bf16.f32 produces. */
static inline uint16_t f32_to_bf16_rn(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)0x7fffu;
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* ---- fp16 (IEEE binary16 through the compiler's _Float16, RN-even) ----- */

static inline float f16_to_f32(uint16_t b) {
  _Float16 h;
  memcpy(&h, &b, 2);
  return (float)h;
}

static inline uint16_t f32_to_f16_rn(float f) {
  if (f != f) return (uint16_t)0x7fffu; /* the GPU's canonical NaN (cvt.rn.f16.f32) */
  _Float16 h = (_Float16)f;
  uint16_t b;
  memcpy(&b, &h, 2);
  return b;
}

static inline float to_f32(int dtype, uint16_t b) {
  return dtype == ORACLE_BF16 ? bf16_to_f32(b) : f16_to_f32(b);
}

static inline uint16_t from_f32(int dtype, float f) {
  return dtype == ORACLE_BF16 ? f32_to_bf16_rn(f) : f32_to_f16_rn(f);
}

/* Exported conversion helpers, so the Python side can pin them against numpy. */
void oracle_to_f32(int dtype, const uint16_t* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = to_f32(dtype, in[i]);
}

void oracle_from_f32(int dtype, const float* in, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = from_f32(dtype, in[i]);
}

/* One row: the whole per-row computation of hp_rms_norm.cuh:149-252. */
static void fused_add_rms_norm_row(int dtype, uint16_t* x, const uint16_t* w, uint16_t* r,
                                   int64_t hidden, double eps, int ss_mode) {
  double ss = 0.0;
  for (int64_t j = 0; j < hidden; ++j) {
    float s = to_f32(dtype, x[j]) + to_f32(dtype, r[j]);
    uint16_t rr = from_f32(dtype, s);
    r[j] = rr;
    double v = (ss_mode == ORACLE_SS_ROUNDED) ? (double)to_f32(dtype, rr) : (double)s;
    ss += v * v;
  }
  float inv = (float)(1.0 / sqrt(ss / (double)hidden + eps));
  for (int64_t j = 0; j < hidden; ++j) {
    float y = to_f32(dtype, r[j]) * to_f32(dtype, w[j]) * inv;
    x[j] = from_f32(dtype, y);
  }
}

/*
 * In place, like rms_norm(input, weight, residual, eps)
 * (hp_rms_norm/csrc/cuda/hp_rms_norm.cu:7-50): residual <- input + residual,
 * input <- RMSNorm(residual) * weight.  Row i of input starts at
 * input + i * in_stride, row i of residual at residual + i * res_stride
 * (both in elements).
 */
void oracle_fused_add_rms_norm(int dtype, uint16_t* input, const uint16_t* weight,
                               uint16_t* residual, int64_t rows, int64_t hidden,
                               int64_t in_stride, int64_t res_stride, double eps,
                               int ss_mode) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < rows; ++i) {
    fused_add_rms_norm_row(dtype, input + i * in_stride, weight, residual + i * res_stride,
                           hidden, eps, ss_mode);
  }
}

/* ---- fp8 e4m3 (OCP "E4M3FN": bias 7, no infinities, max 448, NaN 0x7f) ---
 * Round to nearest even, saturating to +-448 (the "satfinite" rule), NaN to
 * 0x7f: written from the format definition. */
static uint8_t f32_to_e4m3_satfinite(float f) {
  if (f != f) return 0x7f;
  uint8_t sign = signbit(f) ? 0x80 : 0x00;
  float a = fabsf(f);
  if (a >= 448.0f) return (uint8_t)(sign | 0x7e);
  /* Smallest normal 2^-6; subnormals step by 2^-9. */
  int e;
  float m = frexpf(a, &e); /* a = m * 2^e, m in [0.5, 1) */
  int exp_unbiased = e - 1;  /* a = 1.xxx * 2^(e-1) */
  float quantum = exp_unbiased < -6 ? ldexpf(1.0f, -9) : ldexpf(1.0f, exp_unbiased - 3);
  float q = a / quantum;            /* exact: power-of-two scaling */
  float r = nearbyintf(q);          /* ties to even under the default rounding mode */
  float v = r * quantum;
  if (v >= 448.0f) return (uint8_t)(sign | 0x7e);
  if (v == 0.0f) return sign;
  int ve;
  float vm = frexpf(v, &ve);
  int ue = ve - 1;
  if (ue < -6) { /* subnormal: mantissa = v / 2^-9 */
    return (uint8_t)(sign | (uint8_t)(v / ldexpf(1.0f, -9)));
  }
  int mant = (int)((vm * 2.0f - 1.0f) * 8.0f); /* 3 fraction bits */
  return (uint8_t)(sign | (uint8_t)((ue + 7) << 3) | (uint8_t)mant);
}

void oracle_f32_to_e4m3(const float* in, uint8_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = f32_to_e4m3_satfinite(in[i]);
}

/*
 * The generalised row operation (an extension past the reference, which only
 * has the in-place fused form): RMSNorm with or without the residual add, its
 * output either 16-bit (T) or fp8 e4m3.
 *   residual == NULL: s_j = f32(x_j)                           (plain RMSNorm)
 *   otherwise:        s_j = f32(x_j) + f32(r_j), r_j <- round_T(s_j), and
 *                     the normalised value uses the rounded residual.
 *   y_j = (v_j * f32(w_j)) * inv, v_j = rounded residual or f32(x_j),
 *   inv = rsqrt(eps + sum s_j^2 / H).
 *   out_fp8 == 0: out_j = round_T(y_j)
 *   static scale (row_scales == NULL): out_j = e4m3(y_j * (1 / scale))
 *   dynamic (row_scales != NULL): amax = max_j |y_j| (NaNs ignored),
 *     scale_i = max(amax, 1e-12) / 448, out_j = e4m3(y_j * (1 / scale_i)),
 *     row_scales[i] = scale_i.
 * The input is left unchanged unless out == input.
 */
void oracle_rms_norm_out(int dtype, void* out, const uint16_t* input, const uint16_t* weight,
                         uint16_t* residual, int64_t rows, int64_t hidden, int64_t out_stride,
                         int64_t in_stride, int64_t res_stride, double eps, int out_fp8,
                         float scale, float* row_scales) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < rows; ++i) {
    const uint16_t* x = input + i * in_stride;
    uint16_t* r = residual ? residual + i * res_stride : 0;
    double ss = 0.0;
    float* v = (float*)malloc(sizeof(float) * (size_t)hidden);
    for (int64_t j = 0; j < hidden; ++j) {
      float s = to_f32(dtype, x[j]);
      if (r) {
        s = s + to_f32(dtype, r[j]);
        r[j] = from_f32(dtype, s);
        v[j] = to_f32(dtype, r[j]);
      } else {
        v[j] = s;
      }
      ss += (double)s * (double)s;
    }
    float inv = (float)(1.0 / sqrt(ss / (double)hidden + eps));
    float inv_scale = 1.0f;
    if (out_fp8) {
      if (row_scales) {
        float amax = 0.0f;
        for (int64_t j = 0; j < hidden; ++j) amax = fmaxf(amax, fabsf(v[j] * to_f32(dtype, weight[j]) * inv));
        float sc = fmaxf(amax, 1e-12f) / 448.0f;
        row_scales[i] = sc;
        inv_scale = 1.0f / sc;
      } else {
        inv_scale = 1.0f / scale;
      }
    }
    for (int64_t j = 0; j < hidden; ++j) {
      float y = v[j] * to_f32(dtype, weight[j]) * inv;
      if (out_fp8) {
        ((uint8_t*)out)[i * out_stride + j] = f32_to_e4m3_satfinite(y * inv_scale);
      } else {
        ((uint16_t*)out)[i * out_stride + j] = from_f32(dtype, y);
      }
    }
    free(v);
  }
}

/* Per-token-group fp8: the row op of oracle_rms_norm_out (residual optional),
 * then for each group g of `group` consecutive elements of a row
 *   s_g = max(max_j |y_j|, 1e-12) / 448, rounded up to a power of two if pow2
 *   q_j = e4m3_satfinite(y_j * (1 / s_g))
 * y_j = (v_j * w_j) * inv in fp32 (v the rounded residual or the input), as
 * in the other outputs.  out: rows x hidden bytes; scales: rows x hidden/group
 * floats, row-major.  Fixes the semantics of the library's
 * hprn_rms_norm_fp8_group (no reference counterpart). */
static float pow2_ceil_f(float s) {
  int e;
  float m = frexpf(s, &e); /* s = m * 2^e, m in [0.5, 1) */
  return m == 0.5f ? s : ldexpf(1.0f, e);
}

void oracle_rms_norm_fp8_group(int dtype, uint8_t* out, float* scales, const uint16_t* input,
                               const uint16_t* weight, uint16_t* residual, int64_t rows,
                               int64_t hidden, double eps, int group, int pow2) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < rows; ++i) {
    const uint16_t* x = input + i * hidden;
    uint16_t* r = residual ? residual + i * hidden : 0;
    double ss = 0.0;
    float* y = (float*)malloc(sizeof(float) * (size_t)hidden);
    for (int64_t j = 0; j < hidden; ++j) {
      float s = to_f32(dtype, x[j]);
      if (r) {
        s = s + to_f32(dtype, r[j]);
        r[j] = from_f32(dtype, s);
        y[j] = to_f32(dtype, r[j]);
      } else {
        y[j] = s;
      }
      ss += (double)s * (double)s;
    }
    float inv = (float)(1.0 / sqrt(ss / (double)hidden + eps));
    for (int64_t j = 0; j < hidden; ++j) y[j] = y[j] * to_f32(dtype, weight[j]) * inv;
    const int64_t ngroups = hidden / group;
    for (int64_t g = 0; g < ngroups; ++g) {
      float amax = 0.0f;
      for (int64_t j = g * group; j < (g + 1) * group; ++j) amax = fmaxf(amax, fabsf(y[j]));
      float sc = fmaxf(amax, 1e-12f) / 448.0f;
      if (pow2) sc = pow2_ceil_f(sc);
      scales[i * ngroups + g] = sc;
      const float inv_scale = 1.0f / sc;
      for (int64_t j = g * group; j < (g + 1) * group; ++j)
        out[i * hidden + j] = f32_to_e4m3_satfinite(y[j] * inv_scale);
    }
    free(y);
  }
}

/* ---- fp4 e2m1 (values 0, 0.5, 1, 1.5, 2, 3, 4, 6; no inf/NaN) -------------
 * Round to nearest even, saturating to +-6, from the format definition:
 * sign bit 3, two exponent bits (bias 1), one mantissa bit; exponent 0 is the
 * subnormal 0.5 step. */
static uint8_t f32_to_e2m1_satfinite(float f) {
  static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  uint8_t sign = signbit(f) ? 0x8 : 0x0;
  float a = fabsf(f);
  if (a != a) return 0x7; /* NaN: positive maximum, as the GPU conversion does */
  if (a >= 6.0f) return (uint8_t)(sign | 0x7);
  int best = 0;
  for (int c = 1; c < 8; ++c) {
    float dc = fabsf(a - mag[c]), db = fabsf(a - mag[best]);
    if (dc < db || (dc == db && (c & 1) == 0 && (best & 1) == 1)) best = c;
  }
  return (uint8_t)(sign | best);
}

void oracle_f32_to_e2m1(const float* in, uint8_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = f32_to_e2m1_satfinite(in[i]);
}

/*
 * NVFP4 output of the row op (an extension past the reference): y as in
 * oracle_rms_norm_out; for each 16-element block b of a row,
 *   sf_b  = e4m3_satfinite(gs * (max_j |y_j| / 6))         (stored, one byte)
 *   q_j   = e2m1_satfinite(y_j * (gs / float(sf_b)))   (0 when sf_b is 0)
 * two codes per byte, element 2k in the low nibble.  gs is the per-tensor
 * global scale.  out: rows x hidden/2 bytes; block_scales: rows x hidden/16.
 */
void oracle_rms_norm_nvfp4(int dtype, uint8_t* out, uint8_t* block_scales, const uint16_t* input,
                           const uint16_t* weight, uint16_t* residual, int64_t rows,
                           int64_t hidden, double eps, float gs) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < rows; ++i) {
    const uint16_t* x = input + i * hidden;
    uint16_t* r = residual ? residual + i * hidden : 0;
    double ss = 0.0;
    float* y = (float*)malloc(sizeof(float) * (size_t)hidden);
    for (int64_t j = 0; j < hidden; ++j) {
      float s = to_f32(dtype, x[j]);
      if (r) {
        s = s + to_f32(dtype, r[j]);
        r[j] = from_f32(dtype, s);
        y[j] = to_f32(dtype, r[j]);
      } else {
        y[j] = s;
      }
      ss += (double)s * (double)s;
    }
    float inv = (float)(1.0 / sqrt(ss / (double)hidden + eps));
    for (int64_t j = 0; j < hidden; ++j) y[j] = y[j] * to_f32(dtype, weight[j]) * inv;
    for (int64_t b = 0; b < hidden / 16; ++b) {
      float amax = 0.0f;
      for (int k = 0; k < 16; ++k) amax = fmaxf(amax, fabsf(y[b * 16 + k]));
      uint8_t sf = f32_to_e4m3_satfinite(gs * (amax / 6.0f));
      block_scales[i * (hidden / 16) + b] = sf;
      float sfv = 0.0f;
      {
        /* exact value of the e4m3 code */
        int e = (sf >> 3) & 0xf, m = sf & 0x7;
        sfv = e == 0 ? ldexpf((float)m, -9) : ldexpf(1.0f + (float)m / 8.0f, e - 7);
      }
      float qs = sfv != 0.0f ? gs / sfv : 0.0f;
      for (int k = 0; k < 16; k += 2) {
        uint8_t lo = f32_to_e2m1_satfinite(y[b * 16 + k] * qs);
        uint8_t hi = f32_to_e2m1_satfinite(y[b * 16 + k + 1] * qs);
        out[i * (hidden / 2) + (b * 16 + k) / 2] = (uint8_t)(lo | (hi << 4));
      }
    }
    free(y);
  }
}

/* torch.relu (CUDA) on raw 16-bit patterns: every value <= 0 (negatives, -inf,
 * -0.0) becomes +0; NaNs and positives pass through unchanged. */
void oracle_relu(int dtype, uint16_t* out, const uint16_t* in, int64_t n) {
  const uint16_t inf_bits = dtype == ORACLE_BF16 ? 0x7f80u : 0x7c00u;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    uint16_t b = in[i];
    uint16_t mag = (uint16_t)(b & 0x7fffu);
    int non_positive = (b & 0x8000u) && mag <= inf_bits; /* sign set, not NaN */
    out[i] = non_positive ? (uint16_t)0 : b;
  }
}

/* Gated activations: out[i, j] = round_T(act(x[i, j]) * x[i, d + j]) in fp32,
 * act per the published GELU / SiLU definitions (0: silu, 1: gelu erf,
 * 2: gelu tanh), with the C library's expf / erff / tanhf. */
static float oracle_act(int act, float a) {
  if (act == 0) return a / (1.0f + expf(-a));
  if (act == 1) return 0.5f * a * (1.0f + erff(a * 0.70710678118654752f));
  return 0.5f * a * (1.0f + tanhf(0.79788456080286536f * (a + 0.044715f * a * a * a)));
}

void oracle_act_and_mul(int dtype, int act, uint16_t* out, const uint16_t* in, int64_t rows,
                        int64_t d) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < rows; ++i) {
    for (int64_t j = 0; j < d; ++j) {
      float g = to_f32(dtype, in[i * 2 * d + j]);
      float u = to_f32(dtype, in[i * 2 * d + d + j]);
      out[i * d + j] = from_f32(dtype, oracle_act(act, g) * u);
    }
  }
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
