// Elementwise ReLU for sm_100a and its C-ABI entry point.
//
// out = input <= 0 ? +0 : input, on 16-bit floats: bit for bit what torch.relu
// gives on CUDA for every non-NaN value (negatives, -inf and -0.0 all become
// +0); NaNs pass through with their input bits.  Two elements are handled per
// instruction pair: `set.le.u32.{bf16x2,f16x2}` produces an all-ones mask in
// each 16-bit lane holding a value <= 0 (ordered compare, so NaN gives 0), and
// the lane is cleared with it.
//
// Replaces the reference's activation kernel
// (hp_rms_norm/csrc/cuda/activation_kernels.cuh:82-145), which moves 256 bytes
// per quarter-warp but copies instead of applying ReLU and drops the row tail
// when hidden * 2 is not a multiple of 256.  Here contiguous tensors are
// processed as one flat range (any length, scalar tail), and strided ones row
// by row; each thread keeps U vectors of up to 32 bytes in flight.
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "runtime.cuh"
#include "vec.cuh"

namespace hprn {

template <typename T>
__device__ __forceinline__ uint32_t relu2(uint32_t w);

template <>
__device__ __forceinline__ uint32_t relu2<__nv_bfloat16>(uint32_t w) {
  uint32_t m;
  asm("set.le.u32.bf16x2 %0, %1, %2;" : "=r"(m) : "r"(w), "r"(0u));
  return w & ~m;
}

template <>
__device__ __forceinline__ uint32_t relu2<__half>(uint32_t w) {
  uint32_t m;
  asm("set.le.u32.f16x2 %0, %1, %2;" : "=r"(m) : "r"(w), "r"(0u));
  return w & ~m;
}

template <typename T, int VEC>
__device__ __forceinline__ Vec<VEC> relu_vec(Vec<VEC> v) {
  if constexpr (VEC == 2) {
    v.h = static_cast<uint16_t>(relu2<T>(static_cast<uint32_t>(v.h)));
  } else {
#pragma unroll
    for (int k = 0; k < Vec<VEC>::kWords; ++k) v.w[k] = relu2<T>(v.w[k]);
  }
  return v;
}

struct ReluArgs {
  uint16_t* out;
  const uint16_t* in;
  int64_t rows;
  int64_t nvec;            // vectors per row
  int64_t chunks_per_row;  // CTAs per row
  int64_t out_stride;      // elements
  int64_t in_stride;
  int64_t prefetch_ctas;   // CTAs blockIdx.x < this (the first wave) prefetch into L2
  int64_t prefetch_ahead;  // > 0: each CTA also prefetches the chunk of CTA blockIdx.x + this
  int64_t tail_begin;      // flat mode: first element not covered by vectors
  int64_t tail_end;
};

template <typename T, int VEC, int U>
__global__ void __launch_bounds__(256) relu_rows(ReluArgs a) {
  constexpr int EPV = Vec<VEC>::kElems;
  const int64_t row = static_cast<int64_t>(blockIdx.x) / a.chunks_per_row;
  const int64_t chunk = static_cast<int64_t>(blockIdx.x) - row * a.chunks_per_row;
  const uint16_t* src = a.in + row * a.in_stride;
  uint16_t* dst = a.out + row * a.out_stride;
  const uint64_t pol = policy_evict_first();
  const int64_t base = chunk * (static_cast<int64_t>(blockDim.x) * U) + threadIdx.x;
  const int64_t first = base - threadIdx.x;  // the CTA's first vector
  if (threadIdx.x == 0 && first < a.nvec && blockIdx.x < a.prefetch_ctas)
    prefetch_l2(src + first * EPV,
                static_cast<uint64_t>(min(static_cast<int64_t>(blockDim.x) * U, a.nvec - first)) * VEC);
  pdl_wait();

  Vec<VEC> v[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t i = base + static_cast<int64_t>(k) * blockDim.x;
    if (i < a.nvec) v[k] = ld_stream<VEC>(src + i * EPV, pol);
  }
  // The chunk of the CTA one wave later (the one that takes this CTA's slot):
  // its DRAM reads overlap this CTA's stores.  Config 3: 4096 x 14336 bf16 in
  // 35.10 against 35.43 us, 8192 x 28672 fp16 in 136.71 against 137.10.  (The
  // gated activations, issue-bound, were slower with it: GELU 63.4 vs 59.8.)
  const int64_t later = static_cast<int64_t>(blockIdx.x) + a.prefetch_ahead;
  if (threadIdx.x == 0 && a.prefetch_ahead > 0 && later < gridDim.x) {
    const int64_t lrow = later / a.chunks_per_row;
    const int64_t lfirst = (later - lrow * a.chunks_per_row) * (static_cast<int64_t>(blockDim.x) * U);
    if (lfirst < a.nvec)
      prefetch_l2(a.in + lrow * a.in_stride + lfirst * EPV,
                  static_cast<uint64_t>(min(static_cast<int64_t>(blockDim.x) * U, a.nvec - lfirst)) * VEC);
  }
  // Dependents are triggered once the loads are issued (they still wait for
  // this grid to complete before reading): at 4096 x 14336 bf16 34.25 against
  // 35.24 us with the trigger after the last store.
  pdl_trigger();
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t i = base + static_cast<int64_t>(k) * blockDim.x;
    if (i < a.nvec) st_global<VEC>(dst + i * EPV, relu_vec<T, VEC>(v[k]));
  }
  // Flat mode only: the last CTA finishes the elements past the last full vector.
  if (blockIdx.x == gridDim.x - 1) {
    for (int64_t e = a.tail_begin + threadIdx.x; e < a.tail_end; e += blockDim.x) {
      Vec<2> s;
      s.h = src[e];
      dst[e] = relu_vec<T, 2>(s).h;
    }
  }
}

using ReluFn = void (*)(ReluArgs);

template <typename T>
ReluFn pick_relu(int vec) {
  constexpr int U = 4;
  switch (vec) {
    case 32: return relu_rows<T, 32, U>;
    case 16: return relu_rows<T, 16, U>;
    case 8: return relu_rows<T, 8, U>;
    case 4: return relu_rows<T, 4, U>;
    default: return relu_rows<T, 2, U>;
  }
}

constexpr int kReluThreads = 256;
constexpr int kReluUnroll = 4;

}  // namespace hprn

extern "C" {

int hprn_relu(void* out, const void* input, int64_t rows, int64_t hidden, int64_t out_row_stride,
              int64_t input_row_stride, int dtype, void* stream) {
  return hprn_relu_ex(out, input, rows, hidden, out_row_stride, input_row_stride, dtype, stream,
                      HPRN_LAUNCH_DEFAULT);
}

int hprn_relu_ex(void* out, const void* input, int64_t rows, int64_t hidden,
                 int64_t out_row_stride, int64_t input_row_stride, int dtype, void* stream,
                 unsigned flags) {
  using namespace hprn;
  if (flags & ~static_cast<unsigned>(HPRN_LAUNCH_PDL))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "unknown launch flags");
  if (dtype != HPRN_DTYPE_BF16 && dtype != HPRN_DTYPE_FP16)
    return fail(HPRN_ERR_UNSUPPORTED_DTYPE, "dtype must be kFloat16 or kBFloat16");
  if (rows < 0 || hidden < 0) return fail(HPRN_ERR_INVALID_ARGUMENT, "sizes must be >= 0");
  if (rows == 0 || hidden == 0) return ok();
  if (!out || !input) return fail(HPRN_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned(out, 2) || !aligned(input, 2))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "tensor pointers must be 2-byte aligned");
  if (rows > 1 && (out_row_stride < hidden || input_row_stride < hidden))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "row strides must be >= hidden_dim");
  const bool flat = rows == 1 || (out_row_stride == hidden && input_row_stride == hidden);
  if (out != input) {
    const int64_t ospan = (rows - 1) * out_row_stride + hidden;
    const int64_t ispan = (rows - 1) * input_row_stride + hidden;
    const char* ob = static_cast<const char*>(out);
    const char* ib = static_cast<const char*>(input);
    if (ob < ib + 2 * ispan && ib < ob + 2 * ospan && !(flat && ob == ib))
      return fail(HPRN_ERR_INVALID_ARGUMENT, "out and input must be the same tensor or not overlap");
  } else if (out_row_stride != input_row_stride && rows > 1) {
    return fail(HPRN_ERR_INVALID_ARGUMENT, "in-place relu needs equal row strides");
  }
  const DeviceInfo* dev = nullptr;
  int st = current_device(&dev);
  if (st != HPRN_OK) return st;

  ReluArgs a;
  a.out = static_cast<uint16_t*>(out);
  a.in = static_cast<const uint16_t*>(input);
  int vec = 2;
  for (int v : {32, 16, 8, 4}) {
    if (!aligned(out, v) || !aligned(input, v)) continue;
    if (!flat && (hidden % (v / 2) || (out_row_stride * 2) % v || (input_row_stride * 2) % v)) continue;
    vec = v;
    break;
  }
  const int epv = vec / 2;
  if (flat) {
    const int64_t n = rows * hidden;
    a.rows = 1;
    a.nvec = n / epv;
    a.tail_begin = a.nvec * epv;
    a.tail_end = n;
    a.out_stride = a.in_stride = 0;
  } else {
    a.rows = rows;
    a.nvec = hidden / epv;
    a.tail_begin = a.tail_end = 0;
    a.out_stride = out_row_stride;
    a.in_stride = input_row_stride;
  }
  const int64_t per_cta = static_cast<int64_t>(kReluThreads) * kReluUnroll;
  a.chunks_per_row = (a.nvec + per_cta - 1) / per_cta;
  if (a.chunks_per_row < 1) a.chunks_per_row = 1;
  const int64_t grid = a.rows * a.chunks_per_row;
  if (grid > 2147483647LL) return fail(HPRN_ERR_INVALID_ARGUMENT, "tensor too large for one launch");
  ReluFn fn = dtype == HPRN_DTYPE_BF16 ? pick_relu<__nv_bfloat16>(vec) : pick_relu<__half>(vec);
  a.prefetch_ctas = first_wave_ctas(dev, reinterpret_cast<const void*>(fn), kReluThreads);
  a.prefetch_ahead = a.prefetch_ctas;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kReluThreads, 1, 1);
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
    return fail(HPRN_ERR_CUDA, std::string("relu launch failed: ") + cudaGetErrorString(e));
  return ok();
}

}  // extern "C"
