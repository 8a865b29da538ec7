// TEST INFRASTRUCTURE ONLY: a same-box comparator, never part of the product.
//
// A C-ABI shim around the reference's own CUDA launchers, compiled (by
// oracle/build.py) from the reference sources where they lie, into
// oracle/_ref/libhp_rms_norm_ref.so.  It exists so that GPU tests and bench.py
// can run the UNMODIFIED reference kernels next to the product kernels in one
// process: the reference's op-registration file (hp_rms_norm/csrc/hp_rms_norm.cpp)
// is deliberately not compiled, so the shim does not collide with the product's
// torch.ops.hp_rms_norm namespace.
//
// Entry points wrap:
//   hp_rms_norm::launch_rms_norm<T>   hp_rms_norm/csrc/cuda/hp_rms_norm.cuh:562-618
//   hp_rms_norm::launch_relu<T>       hp_rms_norm/csrc/cuda/activation_kernels.cuh:122-145
// with the same argument meaning the reference's host wrappers give them
// (hp_rms_norm/csrc/cuda/hp_rms_norm.cu:26-46, activation_kernels.cu:14-34).
// Errors the reference raises with TORCH_CHECK come back as a non-zero return
// code and a message in ref_last_error().
#include <cstdio>
#include <cstring>
#include <exception>
#include <string>

#include "hp_rms_norm.cuh"
#include "activation_kernels.cuh"

namespace {
thread_local std::string g_ref_error;
}

extern "C" {

const char* ref_last_error() { return g_ref_error.c_str(); }

// dtype: 0 = bf16, 1 = fp16.  Rows are dense (row stride == hidden), as the
// reference kernels assume.
int ref_rms_norm(int dtype, void* input, const void* weight, void* residual, long long tokens,
                 int hidden, double eps, void* stream) {
  try {
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == 0) {
      hp_rms_norm::launch_rms_norm<__nv_bfloat16>(
          reinterpret_cast<__nv_bfloat16*>(input), reinterpret_cast<const __nv_bfloat16*>(weight),
          reinterpret_cast<__nv_bfloat16*>(residual), static_cast<size_t>(tokens), hidden, eps, s);
    } else {
      hp_rms_norm::launch_rms_norm<__half>(
          reinterpret_cast<__half*>(input), reinterpret_cast<const __half*>(weight),
          reinterpret_cast<__half*>(residual), static_cast<size_t>(tokens), hidden, eps, s);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      g_ref_error = cudaGetErrorString(e);
      return 2;
    }
  } catch (const std::exception& ex) {
    g_ref_error = ex.what();
    return 1;
  }
  return 0;
}

int ref_relu(int dtype, void* out, const void* input, long long tokens, int hidden, void* stream) {
  try {
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    if (dtype == 0) {
      hp_rms_norm::launch_relu<__nv_bfloat16>(reinterpret_cast<const __nv_bfloat16*>(input),
                                              reinterpret_cast<__nv_bfloat16*>(out), tokens, hidden,
                                              sms, s);
    } else {
      hp_rms_norm::launch_relu<__half>(reinterpret_cast<const __half*>(input),
                                       reinterpret_cast<__half*>(out), tokens, hidden, sms, s);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      g_ref_error = cudaGetErrorString(e);
      return 2;
    }
  } catch (const std::exception& ex) {
    g_ref_error = ex.what();
    return 1;
  }
  return 0;
}

}  // extern "C"
