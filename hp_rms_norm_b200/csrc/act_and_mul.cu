// Gated activations for sm_100a: out = act(gate) * up, with each input row
// holding [gate (d elements) | up (d elements)] and each output row d
// elements (the MLP activation of SwiGLU / GeGLU blocks).  An extension past
// the reference, whose activation source (activation_kernels.cuh:82-145) is a
// scaffold for this family: one streaming kernel, one activation per template
// instance.
//
//   silu(a)      = a / (1 + exp(-a))
//   gelu(a)      = a / 2 * (1 + erf(a / sqrt(2)))
//   gelu_tanh(a) = a / 2 * (1 + tanh(sqrt(2 / pi) * (a + 0.044715 a^3)))
// (Hendrycks & Gimpel, "Gaussian Error Linear Units", 2016), evaluated in fp32
// with CUDA's expf / erff / tanhf (the arithmetic around them in packed fp32x2
// pairs), times f32(up), rounded once to T.  SiLU's
// division is __fdividef (reciprocal approximation and one multiply, within 2
// fp32 ulp): the IEEE division costs more issue slots than the element's 6
// bytes take on the memory side, and 2 fp32 ulp is far below half an ulp of
// the 16-bit result.
//
// Bandwidth-bound: 6 bytes per output element (gate and up read, out
// written).  Each thread keeps U vectors of gate and of up in flight (32-byte
// accesses where alignment allows), grid over (row, chunk of the row).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <string>

#include "runtime.cuh"
#include "vec.cuh"

namespace hprn {

template <int ACT>
__device__ __forceinline__ float activate(float a) {
  if constexpr (ACT == HPRN_ACT_SILU) {
    // -a past ~88.7 makes the denominator +inf and the result -0 (a * 0).
    return __fdividef(a, 1.0f + expf(-a));
  } else if constexpr (ACT == HPRN_ACT_GELU) {
    return 0.5f * a * (1.0f + erff(a * 0.70710678118654752f));
  } else {
    const float k = 0.79788456080286536f;  // sqrt(2 / pi)
    return 0.5f * a * (1.0f + tanhf(k * (a + 0.044715f * a * a * a)));
  }
}

// activate<ACT> on a pair, with the arithmetic around the library function
// in packed fp32x2 instructions (same operations in the same order, so the
// same bits as two scalar calls, in fewer issue slots).
template <int ACT>
__device__ __forceinline__ float2 activate2(float2 a) {
  if constexpr (ACT == HPRN_ACT_GELU) {
    const float2 t = __fmul2_rn(a, make_float2(0.70710678118654752f, 0.70710678118654752f));
    const float2 e = __fadd2_rn(make_float2(1.0f, 1.0f), make_float2(erff(t.x), erff(t.y)));
    return __fmul2_rn(__fmul2_rn(make_float2(0.5f, 0.5f), a), e);
  } else if constexpr (ACT == HPRN_ACT_GELU_TANH) {
    const float2 k = make_float2(0.79788456080286536f, 0.79788456080286536f);  // sqrt(2 / pi)
    const float2 c = __fmul2_rn(__fmul2_rn(__fmul2_rn(make_float2(0.044715f, 0.044715f), a), a), a);
    const float2 t = __fmul2_rn(k, __fadd2_rn(a, c));
    const float2 e = __fadd2_rn(make_float2(1.0f, 1.0f), make_float2(tanhf(t.x), tanhf(t.y)));
    return __fmul2_rn(__fmul2_rn(make_float2(0.5f, 0.5f), a), e);
  } else {
    return make_float2(activate<ACT>(a.x), activate<ACT>(a.y));
  }
}

template <typename T, int VEC, int ACT>
__device__ __forceinline__ Vec<VEC> act_mul(const Vec<VEC>& g, const Vec<VEC>& u) {
  Vec<VEC> o;
  if constexpr (VEC == 2) {
    o.h = pack1<T>(activate<ACT>(unpack1<T>(g.h)) * unpack1<T>(u.h));
  } else {
#pragma unroll
    for (int k = 0; k < Vec<VEC>::kWords; ++k) {
      const float2 y = __fmul2_rn(activate2<ACT>(unpack2<T>(g.w[k])), unpack2<T>(u.w[k]));
      o.w[k] = pack2<T>(y.x, y.y);
    }
  }
  return o;
}

struct ActArgs {
  uint16_t* out;
  const uint16_t* in;
  int64_t rows;
  int64_t d;               // output elements per row (input rows hold 2d)
  int64_t nvec;            // vectors per output row
  int64_t chunks_per_row;  // CTAs per row
  int64_t out_stride;      // elements
  int64_t in_stride;
  int64_t prefetch_ctas;   // CTAs blockIdx.x < this (the first wave) prefetch into L2
};

template <typename T, int VEC, int U, int ACT>
__global__ void __launch_bounds__(256) act_and_mul_rows(ActArgs a) {
  constexpr int EPV = Vec<VEC>::kElems;
  const int64_t row = static_cast<int64_t>(blockIdx.x) / a.chunks_per_row;
  const int64_t chunk = static_cast<int64_t>(blockIdx.x) - row * a.chunks_per_row;
  const uint16_t* gate = a.in + row * a.in_stride;
  const uint16_t* up = gate + a.d;
  uint16_t* dst = a.out + row * a.out_stride;
  const uint64_t pol = policy_evict_first();
  const int64_t base = chunk * (static_cast<int64_t>(blockDim.x) * U) + threadIdx.x;
  const int64_t first = base - threadIdx.x;  // the CTA's first vector
  if (threadIdx.x == 0 && first < a.nvec && blockIdx.x < a.prefetch_ctas) {
    const uint64_t bytes =
        static_cast<uint64_t>(min(static_cast<int64_t>(blockDim.x) * U, a.nvec - first)) * VEC;
    prefetch_l2(gate + first * EPV, bytes);
    prefetch_l2(up + first * EPV, bytes);
  }
  pdl_wait();

  Vec<VEC> g[U], u[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t i = base + static_cast<int64_t>(k) * blockDim.x;
    if (i < a.nvec) {
      g[k] = ld_stream<VEC>(gate + i * EPV, pol);
      u[k] = ld_stream<VEC>(up + i * EPV, pol);
    }
  }
  // Dependents are triggered once the loads are issued (they still wait for
  // this grid to complete before reading): GELU at 512 x 14336 in 10.01
  // against 10.63 us with the trigger after the last store, 58.95 against
  // 59.82 at 4096 x 14336.
  pdl_trigger();
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t i = base + static_cast<int64_t>(k) * blockDim.x;
    if (i < a.nvec) st_global<VEC>(dst + i * EPV, act_mul<T, VEC, ACT>(g[k], u[k]));
  }
}

using ActFn = void (*)(ActArgs);
// 128-thread CTAs, two vectors per thread: at [4096, 2 x 14336] bf16 the
// erf form runs in 60.3 us (0.894 of the copy peak) and the tanh form in 53.5
// (1.008), against 61.1 / 54.6 us with 256 threads; one vector per thread, four,
// or 512-thread CTAs are 8-14% slower for both.  GELU (erf) spends about 30
// instructions per element, most of them in CUDA's erff, and issues at 82% of
// peak: that, not memory, bounds it.
constexpr int kActThreads = 128;
constexpr int kActUnroll = 2;

template <typename T, int ACT>
ActFn pick_act_vec(int vec) {
  switch (vec) {
    case 32: return act_and_mul_rows<T, 32, kActUnroll, ACT>;
    case 16: return act_and_mul_rows<T, 16, kActUnroll, ACT>;
    case 8: return act_and_mul_rows<T, 8, kActUnroll, ACT>;
    case 4: return act_and_mul_rows<T, 4, kActUnroll, ACT>;
    default: return act_and_mul_rows<T, 2, kActUnroll, ACT>;
  }
}

template <typename T>
ActFn pick_act(int act, int vec) {
  switch (act) {
    case HPRN_ACT_SILU: return pick_act_vec<T, HPRN_ACT_SILU>(vec);
    case HPRN_ACT_GELU: return pick_act_vec<T, HPRN_ACT_GELU>(vec);
    default: return pick_act_vec<T, HPRN_ACT_GELU_TANH>(vec);
  }
}

}  // namespace hprn

extern "C" {

int hprn_act_and_mul(void* out, const void* input, int64_t rows, int64_t d,
                     int64_t out_row_stride, int64_t input_row_stride, int act, int dtype,
                     void* stream, unsigned flags) {
  using namespace hprn;
  if (flags & ~static_cast<unsigned>(HPRN_LAUNCH_PDL))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "unknown launch flags");
  if (dtype != HPRN_DTYPE_BF16 && dtype != HPRN_DTYPE_FP16)
    return fail(HPRN_ERR_UNSUPPORTED_DTYPE, "dtype must be kFloat16 or kBFloat16");
  if (act != HPRN_ACT_SILU && act != HPRN_ACT_GELU && act != HPRN_ACT_GELU_TANH)
    return fail(HPRN_ERR_INVALID_ARGUMENT, "unknown activation");
  if (rows < 0 || d < 0) return fail(HPRN_ERR_INVALID_ARGUMENT, "sizes must be >= 0");
  if (rows == 0 || d == 0) return ok();
  if (!out || !input) return fail(HPRN_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned(out, 2) || !aligned(input, 2))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "tensor pointers must be 2-byte aligned");
  if (rows > 1 && (out_row_stride < d || input_row_stride < 2 * d))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "row strides must be >= d (output) and 2d (input)");
  const char* ob = static_cast<const char*>(out);
  const char* ib = static_cast<const char*>(input);
  const char* oe = ob + 2 * ((rows - 1) * out_row_stride + d);
  const char* ie = ib + 2 * ((rows - 1) * input_row_stride + 2 * d);
  if (ob < ie && ib < oe) return fail(HPRN_ERR_INVALID_ARGUMENT, "out and input must not overlap");
  const DeviceInfo* dev = nullptr;
  int st = current_device(&dev);
  if (st != HPRN_OK) return st;

  int vec = 2;
  for (int v : {32, 16, 8, 4}) {
    const int epv = v / 2;
    if (d % epv || !aligned(out, v) || !aligned(input, v)) continue;
    if (rows > 1 && ((out_row_stride * 2) % v || (input_row_stride * 2) % v)) continue;
    vec = v;
    break;
  }
  ActArgs a;
  a.out = static_cast<uint16_t*>(out);
  a.in = static_cast<const uint16_t*>(input);
  a.rows = rows;
  a.d = d;
  a.nvec = d / (vec / 2);
  a.out_stride = out_row_stride;
  a.in_stride = input_row_stride;
  const int64_t per_cta = static_cast<int64_t>(kActThreads) * kActUnroll;
  a.chunks_per_row = (a.nvec + per_cta - 1) / per_cta;
  const int64_t grid = rows * a.chunks_per_row;
  if (grid > 2147483647LL) return fail(HPRN_ERR_INVALID_ARGUMENT, "tensor too large for one launch");
  ActFn fn = dtype == HPRN_DTYPE_BF16 ? pick_act<__nv_bfloat16>(act, vec) : pick_act<__half>(act, vec);
  a.prefetch_ctas = first_wave_ctas(dev, reinterpret_cast<const void*>(fn), kActThreads);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kActThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  if (flags & HPRN_LAUNCH_PDL) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a);
  if (e != cudaSuccess)
    return fail(HPRN_ERR_CUDA, std::string("act_and_mul launch failed: ") + cudaGetErrorString(e));
  return ok();
}

}  // extern "C"
