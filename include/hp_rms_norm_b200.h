/*
 * hp_rms_norm_b200: C ABI of the B200-native (sm_100a) fused residual-add +
 * RMSNorm and ReLU kernels.
 *
 * Everything here is plain C: device pointers, element counts and strides, a
 * dtype code and a CUDA stream handle passed as void*.  No torch types cross
 * this boundary.  The torch-extension binding (torch.ops.hp_rms_norm.*) and
 * any cgo / JNI / ctypes caller bind these same symbols.
 *
 * Conventions shared by every entry point:
 *   - All tensor pointers are device pointers on the CURRENT CUDA device of
 *     the calling thread (cudaSetDevice before calling).
 *   - Work is enqueued asynchronously on `stream` (a cudaStream_t; NULL means
 *     the legacy default stream).  Nothing synchronises; nothing allocates.
 *   - Return value: HPRN_OK (0) or a negative hprn_status code; on error no
 *     kernel was launched (except HPRN_ERR_CUDA, which reports a failed
 *     launch) and hprn_last_error() returns a message for this thread.
 *   - Strides are in ELEMENTS, between consecutive rows; elements within a
 *     row are contiguous.
 */
#ifndef HP_RMS_NORM_B200_H_
#define HP_RMS_NORM_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HPRN_VERSION 10000 /* 1.0.0 */

#if defined(__GNUC__)
#define HPRN_API __attribute__((visibility("default")))
#else
#define HPRN_API
#endif

typedef enum hprn_dtype {
  HPRN_DTYPE_BF16 = 0, /* torch.bfloat16 / __nv_bfloat16 */
  HPRN_DTYPE_FP16 = 1  /* torch.float16  / __half        */
} hprn_dtype;

/*
 * Launch flags for the *_ex entry points.
 *   HPRN_LAUNCH_PDL: launch with programmatic stream serialization (programmatic
 *   dependent launch).  The kernel may then be scheduled while the previous
 *   kernel on the stream is still finishing; it waits (griddepcontrol.wait)
 *   for that kernel to complete before its first memory access, so results
 *   are the same as a plain launch.  Every kernel of this library also lets
 *   its own successor be scheduled early, once all of its CTAs have issued
 *   their last store.
 */
#define HPRN_LAUNCH_PDL 1u
#define HPRN_LAUNCH_DEFAULT HPRN_LAUNCH_PDL

/* Output forms of hprn_rms_norm_out. */
typedef enum hprn_out_form {
  HPRN_OUT_SAME = 0,              /* 16-bit, the input's dtype */
  HPRN_OUT_FP8_E4M3_STATIC = 1,   /* fp8 e4m3 (OCP E4M3FN), one scale for the tensor */
  HPRN_OUT_FP8_E4M3_DYNAMIC = 2,  /* fp8 e4m3, one scale per row, written to row_scales */
  HPRN_OUT_NVFP4 = 3,             /* fp4 e2m1 + e4m3 block scales: hprn_rms_norm_nvfp4 only */
  HPRN_OUT_FP8_E4M3_GROUP = 4     /* fp8 e4m3, one scale per group: hprn_rms_norm_fp8_group only */
} hprn_out_form;

/* Activations of hprn_act_and_mul. */
typedef enum hprn_act {
  HPRN_ACT_SILU = 0,      /* a / (1 + exp(-a))                                   */
  HPRN_ACT_GELU = 1,      /* a / 2 * (1 + erf(a / sqrt(2)))                      */
  HPRN_ACT_GELU_TANH = 2  /* a / 2 * (1 + tanh(sqrt(2/pi) * (a + 0.044715 a^3))) */
} hprn_act;

typedef enum hprn_status {
  HPRN_OK = 0,
  HPRN_ERR_INVALID_ARGUMENT = -1, /* bad size, stride, null pointer, overlap */
  HPRN_ERR_UNSUPPORTED_DTYPE = -2,
  HPRN_ERR_UNSUPPORTED_DEVICE = -3, /* not an sm_100 (B200-class) device */
  HPRN_ERR_CUDA = -4                /* a CUDA runtime call or launch failed */
} hprn_status;

/*
 * Fused residual add + RMSNorm, in place:
 *
 *   residual[i, :] <- round_T(f32(input[i, :]) + f32(residual[i, :]))
 *   input[i, :]    <- round_T(f32(residual[i, :]) * f32(weight[:]) * inv_i)
 *   inv_i           = rsqrt(eps + sum_j s_ij^2 / hidden),  s_ij the fp32 sum before rounding
 *
 * for rows i in [0, rows).  input and residual must not overlap.
 *
 * Replaces the reference's torch-op implementation
 *   void rms_norm(Tensor& input, const Tensor& weight, Tensor& residual, double eps)
 *     hp_rms_norm/csrc/cuda/hp_rms_norm.cu:7-50
 * and its launcher hp_rms_norm::launch_rms_norm<T>
 *     hp_rms_norm/csrc/cuda/hp_rms_norm.cuh:562-618
 * (there `rows` is the reference's `tokens` and both strides equal hidden).
 * Unlike the reference it accepts any hidden >= 1, any 2-byte-aligned pointers
 * and independent row strides; the widest vector width the pointers, strides
 * and hidden size allow is chosen per call.
 */
HPRN_API int hprn_rms_norm(void* input, const void* weight, void* residual, int64_t rows,
                           int64_t hidden, int64_t input_row_stride, int64_t residual_row_stride,
                           double eps, int dtype, void* stream);

/*
 * Elementwise ReLU, out-of-place: out[i, :] = input[i, :] <= 0 ? +0 : input[i, :]
 * (torch.relu as computed on CUDA, bit for bit: negatives, -inf and -0.0 give
 * +0; NaNs pass through with their input bits).
 * out and input may be the same pointer (in place) but must not otherwise overlap.
 *
 * Replaces the reference's
 *   void relu(Tensor& out, const Tensor& input)
 *     hp_rms_norm/csrc/cuda/activation_kernels.cu:7-39
 * and hp_rms_norm::launch_relu<T> hp_rms_norm/csrc/cuda/activation_kernels.cuh:122-145.
 * (The reference kernel copies input to out without applying max(x, 0) and
 * drops the row tail when hidden * 2 is not a multiple of 256; this entry point
 * applies ReLU to every element.)
 */
HPRN_API int hprn_relu(void* out, const void* input, int64_t rows, int64_t hidden,
                       int64_t out_row_stride, int64_t input_row_stride, int dtype, void* stream);

/*
 * hprn_rms_norm and hprn_relu with explicit launch flags (HPRN_LAUNCH_*; 0 for
 * a plain launch).  The plain entry points use HPRN_LAUNCH_DEFAULT.
 * (Extensions of the reference's fixed launch: FlashInfer-style enable_pdl.)
 */
HPRN_API int hprn_rms_norm_ex(void* input, const void* weight, void* residual, int64_t rows,
                              int64_t hidden, int64_t input_row_stride,
                              int64_t residual_row_stride, double eps, int dtype, void* stream,
                              unsigned flags);
HPRN_API int hprn_relu_ex(void* out, const void* input, int64_t rows, int64_t hidden,
                          int64_t out_row_stride, int64_t input_row_stride, int dtype,
                          void* stream, unsigned flags);

/*
 * RMSNorm with or without the residual add, into a separate output, 16-bit or
 * fp8 (an extension past the reference, whose only form is hprn_rms_norm's):
 *
 *   residual == NULL (plain RMSNorm):  s_j = f32(input[i, j])
 *   residual != NULL (fused add):      s_j = f32(input[i, j]) + f32(residual[i, j]),
 *                                      residual[i, j] <- round_T(s_j)  (in place)
 *   inv_i = rsqrt(eps + sum_j s_j^2 / hidden)
 *   y_ij  = v_ij * f32(weight[j]) * inv_i, v_ij the rounded residual (fused) or f32(input)
 *   HPRN_OUT_SAME:             out[i, j] = round_T(y_ij)      (out may be `input` itself)
 *   HPRN_OUT_FP8_E4M3_STATIC:  out[i, j] = e4m3(y_ij * (1 / *scale))
 *   HPRN_OUT_FP8_E4M3_DYNAMIC: row_scales[i] = max(max_j |y_ij|, 1e-12) / 448,
 *                              out[i, j] = e4m3(y_ij * (1 / row_scales[i]))
 * e4m3 conversion rounds to nearest even and saturates to +-448 (NaN stays NaN).
 * `input` is not written unless out == input.  `scale` (one float) and
 * `row_scales` (rows floats) are device pointers.  fp8 output needs
 * hidden % 4 == 0 with 8-byte aligned input/weight/residual rows and 4-byte
 * aligned output rows, and rows of at most 16384 vectors (262144 elements at
 * full alignment).  Output row stride is in output elements.
 */
HPRN_API int hprn_rms_norm_out(void* out, const void* input, const void* weight, void* residual,
                               int64_t rows, int64_t hidden, int64_t out_row_stride,
                               int64_t input_row_stride, int64_t residual_row_stride, double eps,
                               int dtype, int out_form, const float* scale, float* row_scales,
                               void* stream, unsigned flags);

/*
 * Gated activation (an extension past the reference):
 *   out[i, j] = round_T(act(f32(input[i, j])) * f32(input[i, d + j])),  j < d
 * Input rows hold [gate | up] (2d elements), output rows d elements; fp32
 * arithmetic with CUDA's expf / erff / tanhf.  out and input must not overlap.
 * Strides are in elements.  `act` is an hprn_act value.
 */
HPRN_API int hprn_act_and_mul(void* out, const void* input, int64_t rows, int64_t d,
                              int64_t out_row_stride, int64_t input_row_stride, int act,
                              int dtype, void* stream, unsigned flags);

/*
 * The same row operation as hprn_rms_norm_out (residual optional) with an
 * NVFP4 output (an extension past the reference): for every 16-element block
 * b of a row, with gs = *global_scale (one float on the device),
 *   block_scales[i, b] = sf = e4m3_satfinite(gs * (max_j |y_ij| / 6))
 *   q_ij = e2m1_satfinite(y_ij * (gs / sf))     (0 when sf == 0; NaN -> +6)
 * so y ~ q * sf / gs.  `out` holds two e2m1 codes per byte, element 2k in the
 * low nibble; out_row_stride counts fp4 elements (a multiple of 16).
 * block_scales is rows x hidden/16 bytes, row-major.  Needs hidden % 16 == 0,
 * 32-byte aligned input/weight/residual rows and 8-byte aligned output rows.
 */
HPRN_API int hprn_rms_norm_nvfp4(void* out, uint8_t* block_scales, const void* input,
                                 const void* weight, void* residual, int64_t rows, int64_t hidden,
                                 int64_t out_row_stride, int64_t input_row_stride,
                                 int64_t residual_row_stride, double eps, int dtype,
                                 const float* global_scale, void* stream, unsigned flags);

/*
 * The same row operation as hprn_rms_norm_out (residual optional) with a
 * per-token-group fp8 output (an extension past the reference; the
 * quantisation FP8 GEMMs with block-wise scales consume): for every group g of
 * `group_size` consecutive elements of row i,
 *   s_ig = max(max_{j in g} |y_ij|, 1e-12) / 448, rounded up to a power of two
 *          when scale_pow2 != 0 (scales an exponent-only format can hold)
 *   out[i, j] = e4m3_satfinite(y_ij * (1 / s_ig))
 *   scales[i * scale_row_stride + g * scale_group_stride] = s_ig   (fp32)
 * y_ij is the fp32 normalised value (not rounded to 16 bits first).  The
 * scale strides are in floats: (hidden / group_size, 1) for row-major scales,
 * (1, rows or more) for column-major.  group_size is 32, 64 or 128;
 * hidden % group_size == 0; input/weight/residual rows 32-byte aligned,
 * output rows 16-byte aligned; out_row_stride in bytes (fp8 elements).
 */
HPRN_API int hprn_rms_norm_fp8_group(void* out, float* scales, int64_t scale_row_stride,
                                     int64_t scale_group_stride, const void* input,
                                     const void* weight, void* residual, int64_t rows,
                                     int64_t hidden, int64_t out_row_stride,
                                     int64_t input_row_stride, int64_t residual_row_stride,
                                     double eps, int dtype, int group_size, int scale_pow2,
                                     void* stream, unsigned flags);

/* Message for the last non-OK status returned on this thread ("" if none). */
HPRN_API const char* hprn_last_error(void);

/* Static name of a status code. */
HPRN_API const char* hprn_status_string(int status);

/* HPRN_VERSION of the loaded library. */
HPRN_API int hprn_version(void);

/*
 * Launch-plan introspection (for tests and benchmarks): writes the plan that
 * hprn_rms_norm would use for this problem on the current device into
 * `plan` as a NUL-terminated string "<kind>:vec<V>:vpt<P>:tpr<T>:cluster<C>:rpc<R>"
 * (kind warp | cta | cluster | twopass | tma; V bytes per vector access; P
 * vectors per thread; T threads per CTA, or for kind warp the lanes holding one
 * row (1..32, a power of two); C CTAs per row; R rows per CTA, or for kind tma
 * the depth of the CTA's ring of TMA-staged rows) and returns HPRN_OK.  Performs no launch.  Null input/residual pointers plan for
 * 256-byte-aligned tensors; without a usable device it plans for a 148-SM B200.
 * The weight is assumed to be aligned like the input: a call whose weight is
 * less aligned than its input gets a narrower vector width (and so possibly
 * another plan) than the one returned here.
 */
HPRN_API int hprn_rms_norm_plan(int64_t rows, int64_t hidden, int dtype, const void* input,
                                const void* residual, int64_t input_row_stride,
                                int64_t residual_row_stride, char* plan, int plan_len);

/*
 * Tuning hook: force the launch plan of every later hprn_rms_norm* call in
 * this process (same string format as hprn_rms_norm_plan; NULL or "" restores
 * the built-in heuristic).  A plan may end in ":pf<F>:et<E>", two launch knobs
 * that change timing only, never results: F is the L2 prefetch each CTA issues
 * for its first rows before waiting on the preceding grid (0 none, 1 the
 * grid's first wave of CTAs, 2 every CTA, 3 the first wave, with every CTA also
 * prefetching the row of the CTA one wave later) and E where dependents are triggered
 * (0 after the last store, 1 after the row reduction, 2 once the loads are
 * issued); without them the plan's defaults apply.  "default:pf<F>:et<E>" keeps the built-in plan and sets only
 * the knobs.  hprn_rms_norm_plan echoes knobs an override names.  The
 * HP_RMS_NORM_PLAN environment variable, read at
 * the first call, sets the same override.  A forced plan that does not fit a
 * call makes that call fail with HPRN_ERR_INVALID_ARGUMENT.  Process-global
 * (safe to call concurrently with launches): meant for benchmarks and
 * launch-shape sweeps, not for production callers.
 */
HPRN_API int hprn_set_plan_override(const char* plan);

/*
 * No reference counterpart.  Kernels that stage rows through TMA bulk copies
 * (plan kind tma, reached only through a plan override) wait on mbarriers with
 * a bound (one second); a CTA that gives up a wait leaves the row it gave up
 * on and its remaining rows untouched (input and residual as they were) and
 * counts itself here, on its device.  The call that launched it still returns
 * HPRN_OK: a caller that forces a tma plan must read this count.
 * Writes the current device's count into *count and, if `reset` is non-zero,
 * clears it.  Synchronous; synchronise the streams that launched the kernels
 * first.  A non-zero count means the launches since the last reset produced
 * incomplete results.
 */
HPRN_API int hprn_wait_timeouts(unsigned int* count, int reset);

/*
 * No reference counterpart.  Test hook for the bounded waits above: every
 * later launch of a TMA-staged plan in this process makes the staged copy of
 * row `row` (counted from the first row of that call; -1 turns the hook off)
 * expect 16 bytes more than its copies deliver, so the row's mbarrier phase
 * cannot complete and its wait runs out after `wait_limit_ns` nanoseconds
 * (at most one second; 0 keeps the built-in one second).  The CTA holding
 * that row then takes its give-up path: it waits for the copies it still has
 * in flight (releasing the stalled row's 16 extra bytes itself, so that wait
 * ends once its copies have landed), leaves that row and its later rows
 * untouched, and counts itself in hprn_wait_timeouts.  No fault and no hang:
 * every wait stays bounded.  Plans of other kinds ignore it.  Process-global;
 * for tests only.
 */
HPRN_API int hprn_test_stall_bulk_copy(int64_t row, uint64_t wait_limit_ns);

#ifdef __cplusplus
}
#endif

#endif /* HP_RMS_NORM_B200_H_ */
