// torch.ops.hp_rms_norm.{rms_norm, relu}: the reference's operator surface,
// implemented on top of the C ABI in include/hp_rms_norm_b200.h.
//
// Mirrors hp_rms_norm/csrc/hp_rms_norm.cpp:4-43 of the reference (the `_C`
// module and the `hp_rms_norm` op namespace with the same op names and
// argument order) and the argument checks of its host wrappers
// (hp_rms_norm/csrc/cuda/hp_rms_norm.cu:12-24, activation_kernels.cu:11-16),
// with the same check messages.  Added on top: dtype/device agreement between
// the tensors, a device guard for the input's device (the reference launches
// on whatever device is current), honest handling of row strides (the
// reference assumes dense rows after view(-1, H)), mutation annotations in the
// schemas and Meta kernels so the ops trace under torch.compile.
#include <Python.h>

#include <ATen/core/Tensor.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "hp_rms_norm_b200.h"

extern "C" {
// An empty `_C` module: importing it loads this library, whose static
// initialisers register the operators below.
PyObject* PyInit__C(void) {
  static struct PyModuleDef module_def = {PyModuleDef_HEAD_INIT, "_C", nullptr, -1, nullptr};
  return PyModule_Create(&module_def);
}
}

namespace {

int dtype_code(const at::Tensor& t) {
  if (t.scalar_type() == at::kBFloat16) return HPRN_DTYPE_BF16;
  if (t.scalar_type() == at::kHalf) return HPRN_DTYPE_FP16;
  TORCH_CHECK(false, "dtype must be kFloat16 or kBFloat16");
}

// Rows of a [..., hidden] tensor whose last dim is contiguous: the number of
// rows and the stride between consecutive rows, or an error when the leading
// dims cannot be walked with one stride (the case where the reference's
// view(-1, hidden) throws).
void rows_of(const at::Tensor& t, const char* name, int64_t* rows, int64_t* stride) {
  const int64_t hidden = t.size(-1);
  int64_t n = 1;
  for (int64_t i = 0; i + 1 < t.dim(); ++i) n *= t.size(i);
  *rows = n;
  *stride = hidden;
  if (n <= 1) return;
  int64_t expect = -1;  // stride the next-outer non-trivial dim must have
  int64_t row_stride = -1;
  for (int64_t i = t.dim() - 2; i >= 0; --i) {
    if (t.size(i) == 1) continue;
    if (row_stride < 0) {
      row_stride = t.stride(i);
      expect = t.stride(i) * t.size(i);
    } else {
      TORCH_CHECK(t.stride(i) == expect, name,
                  " must be viewable as (-1, hidden_dim): its leading dimensions are not "
                  "collapsible into rows of one stride");
      expect = t.stride(i) * t.size(i);
    }
  }
  *stride = row_stride;
}

void check_status(int status) {
  TORCH_CHECK(status == HPRN_OK, hprn_status_string(status), ": ", hprn_last_error());
}

void rms_norm(at::Tensor& input, const at::Tensor& weight, at::Tensor& residual, double eps) {
  // hp_rms_norm/csrc/cuda/hp_rms_norm.cu:12-24
  TORCH_CHECK(input.dim() >= 2, "input.dim() >= 2");
  TORCH_CHECK(input.dim() == residual.dim(), "input.dim() == residual.dim()");
  for (int64_t i = 0; i < input.dim(); ++i) {
    TORCH_CHECK(input.size(i) == residual.size(i), "input.size(i) == residual.size(i)");
  }
  TORCH_CHECK(weight.dim() == 1, "weight.dim() == 1");
  const int64_t hidden = weight.size(0);
  TORCH_CHECK(input.size(-1) == hidden, "input.size(-1) == hidden_dim");
  TORCH_CHECK(input.stride(-1) == 1, "input.stride(-1) == 1");
  TORCH_CHECK(residual.stride(-1) == 1, "residual.stride(-1) == 1");
  // Added checks.
  TORCH_CHECK(input.is_cuda() && weight.is_cuda() && residual.is_cuda(),
              "input, weight and residual must be CUDA tensors");
  TORCH_CHECK(weight.device() == input.device() && residual.device() == input.device(),
              "input, weight and residual must be on the same device");
  TORCH_CHECK(weight.scalar_type() == input.scalar_type() &&
                  residual.scalar_type() == input.scalar_type(),
              "input, weight and residual must have the same dtype");
  TORCH_CHECK(hidden <= 1 || weight.stride(0) == 1, "weight must be contiguous");
  const int dtype = dtype_code(input);
  int64_t rows = 0, xs = 0, rrows = 0, rs = 0;
  rows_of(input, "input", &rows, &xs);
  rows_of(residual, "residual", &rrows, &rs);
  if (rows == 0 || hidden == 0) return;
  const c10::cuda::CUDAGuard guard(input.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(input.device().index()).stream();
  check_status(hprn_rms_norm(input.data_ptr(), weight.data_ptr(), residual.data_ptr(), rows, hidden,
                             xs, rs, eps, dtype, stream));
}

void relu(at::Tensor& out, const at::Tensor& input) {
  // hp_rms_norm/csrc/cuda/activation_kernels.cu:11-16
  TORCH_CHECK(input.dim() >= 2, "input.dim() >= 2");
  TORCH_CHECK(input.dim() == out.dim(), "input.size(i) == out.size(i)");
  for (int64_t i = 0; i < input.dim(); ++i) {
    TORCH_CHECK(input.size(i) == out.size(i), "input.size(i) == out.size(i)");
  }
  // Added checks.
  TORCH_CHECK(input.is_cuda() && out.is_cuda(), "out and input must be CUDA tensors");
  TORCH_CHECK(out.device() == input.device(), "out and input must be on the same device");
  TORCH_CHECK(out.scalar_type() == input.scalar_type(), "out and input must have the same dtype");
  const int dtype = dtype_code(input);
  const int64_t hidden = input.size(-1);
  if (input.numel() == 0) return;
  TORCH_CHECK(hidden == 1 || input.stride(-1) == 1, "input.stride(-1) == 1");
  TORCH_CHECK(hidden == 1 || out.stride(-1) == 1, "out.stride(-1) == 1");
  int64_t rows = 0, is = 0, orows = 0, os = 0;
  rows_of(input, "input", &rows, &is);
  rows_of(out, "out", &orows, &os);
  const c10::cuda::CUDAGuard guard(input.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(input.device().index()).stream();
  check_status(hprn_relu(out.data_ptr(), input.data_ptr(), rows, hidden, os, is, dtype, stream));
}

// Common checks of the out-of-place forms (extensions past the reference).
struct OutCall {
  int64_t rows = 0, hidden = 0, os = 0, xs = 0, rs = 0;
  int dtype = 0;
};

OutCall check_out_call(const at::Tensor& out, const at::Tensor& input, const at::Tensor& weight,
                       const c10::optional<at::Tensor>& residual) {
  OutCall c;
  TORCH_CHECK(input.dim() >= 1, "input.dim() >= 1");
  TORCH_CHECK(weight.dim() == 1, "weight.dim() == 1");
  c.hidden = weight.size(0);
  TORCH_CHECK(input.size(-1) == c.hidden, "input.size(-1) == hidden_dim");
  TORCH_CHECK(out.sizes() == input.sizes(), "out must have the input's shape");
  TORCH_CHECK(input.is_cuda() && weight.is_cuda() && out.is_cuda(), "tensors must be CUDA tensors");
  TORCH_CHECK(weight.device() == input.device() && out.device() == input.device(),
              "tensors must be on the same device");
  TORCH_CHECK(weight.scalar_type() == input.scalar_type(), "input and weight must have the same dtype");
  TORCH_CHECK(c.hidden <= 1 || weight.stride(0) == 1, "weight must be contiguous");
  TORCH_CHECK(input.stride(-1) == 1 || c.hidden == 1, "input.stride(-1) == 1");
  TORCH_CHECK(out.stride(-1) == 1 || c.hidden == 1, "out.stride(-1) == 1");
  c.dtype = dtype_code(input);
  rows_of(input, "input", &c.rows, &c.xs);
  int64_t orows = 0;
  rows_of(out, "out", &orows, &c.os);
  c.rs = c.hidden;
  if (residual.has_value()) {
    const at::Tensor& r = *residual;
    TORCH_CHECK(r.sizes() == input.sizes(), "residual must have the input's shape");
    TORCH_CHECK(r.is_cuda() && r.device() == input.device(), "residual must be on the input's device");
    TORCH_CHECK(r.scalar_type() == input.scalar_type(), "input and residual must have the same dtype");
    TORCH_CHECK(r.stride(-1) == 1 || c.hidden == 1, "residual.stride(-1) == 1");
    int64_t rrows = 0;
    rows_of(r, "residual", &rrows, &c.rs);
  }
  return c;
}

// out <- RMSNorm(input [+ residual]) * weight in the input's dtype; the
// residual (if given) is updated in place; out may be the input itself.
void rms_norm_out(at::Tensor& out, const at::Tensor& input, const at::Tensor& weight,
                  c10::optional<at::Tensor> residual, double eps) {
  TORCH_CHECK(out.scalar_type() == input.scalar_type(), "out must have the input's dtype");
  const OutCall c = check_out_call(out, input, weight, residual);
  if (c.rows == 0 || c.hidden == 0) return;
  const c10::cuda::CUDAGuard guard(input.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(input.device().index()).stream();
  check_status(hprn_rms_norm_out(out.data_ptr(), input.data_ptr(), weight.data_ptr(),
                                 residual.has_value() ? residual->data_ptr() : nullptr, c.rows,
                                 c.hidden, c.os, c.xs, c.rs, eps, c.dtype, HPRN_OUT_SAME, nullptr,
                                 nullptr, stream, HPRN_LAUNCH_DEFAULT));
}

// out (float8_e4m3fn) <- e4m3(RMSNorm(input [+ residual]) * weight / scale):
// with `scale` (one float32) a static per-tensor scale, with `row_scales`
// (float32 [rows], written) a per-row scale max|y| / 448.
void rms_norm_fp8(at::Tensor& out, const at::Tensor& input, const at::Tensor& weight,
                  c10::optional<at::Tensor> residual, double eps, c10::optional<at::Tensor> scale,
                  c10::optional<at::Tensor> row_scales) {
  TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn, "out must be float8_e4m3fn");
  TORCH_CHECK(scale.has_value() != row_scales.has_value(),
              "exactly one of scale (static) and row_scales (dynamic) must be given");
  const OutCall c = check_out_call(out, input, weight, residual);
  const float* sp = nullptr;
  float* rsp = nullptr;
  if (scale.has_value()) {
    TORCH_CHECK(scale->scalar_type() == at::kFloat && scale->numel() == 1 && scale->is_cuda() &&
                    scale->device() == input.device(),
                "scale must be one float32 on the input's device");
    sp = scale->data_ptr<float>();
  } else {
    TORCH_CHECK(row_scales->scalar_type() == at::kFloat && row_scales->numel() == c.rows &&
                    row_scales->is_contiguous() && row_scales->is_cuda() &&
                    row_scales->device() == input.device(),
                "row_scales must be a contiguous float32 tensor with one entry per row");
    rsp = row_scales->data_ptr<float>();
  }
  if (c.rows == 0 || c.hidden == 0) return;
  const c10::cuda::CUDAGuard guard(input.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(input.device().index()).stream();
  check_status(hprn_rms_norm_out(out.data_ptr(), input.data_ptr(), weight.data_ptr(),
                                 residual.has_value() ? residual->data_ptr() : nullptr, c.rows,
                                 c.hidden, c.os, c.xs, c.rs, eps, c.dtype,
                                 sp ? HPRN_OUT_FP8_E4M3_STATIC : HPRN_OUT_FP8_E4M3_DYNAMIC, sp,
                                 rsp, stream, HPRN_LAUNCH_DEFAULT));
}

// NVFP4 output (extension past the reference): out uint8 [..., hidden/2] holds
// e2m1 pairs (element 2k in the low nibble), block_scales (uint8 or
// float8_e4m3fn) [..., hidden/16] one e4m3 scale per 16 elements, global_scale
// one float32: y ~ e2m1 * scale / global_scale.
void rms_norm_nvfp4(at::Tensor& out, at::Tensor& block_scales, const at::Tensor& input,
                    const at::Tensor& weight, c10::optional<at::Tensor> residual, double eps,
                    const at::Tensor& global_scale) {
  TORCH_CHECK(input.dim() >= 1 && weight.dim() == 1 && input.size(-1) == weight.size(0),
              "input.size(-1) == hidden_dim");
  const int64_t hidden = weight.size(0);
  TORCH_CHECK(hidden % 16 == 0, "NVFP4 output needs hidden_dim % 16 == 0");
  TORCH_CHECK(out.scalar_type() == at::kByte, "out must be uint8 (two e2m1 codes per byte)");
  TORCH_CHECK(block_scales.scalar_type() == at::kByte ||
                  block_scales.scalar_type() == at::kFloat8_e4m3fn,
              "block_scales must be uint8 or float8_e4m3fn");
  TORCH_CHECK(out.dim() == input.dim() && block_scales.dim() == input.dim(),
              "out and block_scales must have the input's rank");
  for (int64_t i = 0; i + 1 < input.dim(); ++i)
    TORCH_CHECK(out.size(i) == input.size(i) && block_scales.size(i) == input.size(i),
                "out and block_scales must agree with the input on leading dimensions");
  TORCH_CHECK(out.size(-1) == hidden / 2 && block_scales.size(-1) == hidden / 16,
              "out.size(-1) == hidden_dim / 2 and block_scales.size(-1) == hidden_dim / 16");
  TORCH_CHECK(block_scales.is_contiguous(), "block_scales must be contiguous");
  TORCH_CHECK(global_scale.scalar_type() == at::kFloat && global_scale.numel() == 1,
              "global_scale must be one float32");
  const at::Tensor* all[] = {&out, &block_scales, &input, &weight, &global_scale};
  for (const at::Tensor* t : all)
    TORCH_CHECK(t->is_cuda() && t->device() == input.device(), "tensors must share a CUDA device");
  TORCH_CHECK(weight.scalar_type() == input.scalar_type(), "input and weight must have the same dtype");
  TORCH_CHECK(input.stride(-1) == 1 && out.stride(-1) == 1 && weight.stride(0) == 1,
              "input, out and weight must be contiguous in the last dimension");
  const int dtype = dtype_code(input);
  int64_t rows = 0, xs = 0, orows = 0, os = 0, rs = hidden;
  rows_of(input, "input", &rows, &xs);
  rows_of(out, "out", &orows, &os);
  void* rp = nullptr;
  if (residual.has_value()) {
    TORCH_CHECK(residual->sizes() == input.sizes() && residual->scalar_type() == input.scalar_type() &&
                    residual->is_cuda() && residual->device() == input.device() &&
                    residual->stride(-1) == 1,
                "residual must match the input's shape, dtype and device");
    int64_t rrows = 0;
    rows_of(*residual, "residual", &rrows, &rs);
    rp = residual->data_ptr();
  }
  if (rows == 0 || hidden == 0) return;
  const c10::cuda::CUDAGuard guard(input.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(input.device().index()).stream();
  check_status(hprn_rms_norm_nvfp4(out.data_ptr(), static_cast<uint8_t*>(block_scales.data_ptr()),
                                   input.data_ptr(), weight.data_ptr(), rp, rows, hidden, os * 2,
                                   xs, rs, eps, dtype, global_scale.data_ptr<float>(), stream,
                                   HPRN_LAUNCH_DEFAULT));
}

// Per-token-group fp8 output (extension past the reference): out
// float8_e4m3fn [..., hidden]; scales float32 [rows, hidden / group_size]
// (rows = the input's leading dimensions flattened), any strides, so a
// transposed view gives column-major scales.
void rms_norm_fp8_group(at::Tensor& out, at::Tensor& scales, const at::Tensor& input,
                        const at::Tensor& weight, c10::optional<at::Tensor> residual, double eps,
                        int64_t group_size, bool scale_pow2) {
  TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn, "out must be float8_e4m3fn");
  const OutCall c = check_out_call(out, input, weight, residual);
  TORCH_CHECK(group_size == 32 || group_size == 64 || group_size == 128,
              "group_size must be 32, 64 or 128");
  TORCH_CHECK(c.hidden % group_size == 0, "hidden_dim must be a multiple of group_size");
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.dim() == 2 &&
                  scales.size(0) == c.rows && scales.size(1) == c.hidden / group_size,
              "scales must be float32 [rows, hidden / group_size]");
  TORCH_CHECK(scales.is_cuda() && scales.device() == input.device(),
              "scales must be on the input's device");
  if (c.rows == 0 || c.hidden == 0) return;
  const c10::cuda::CUDAGuard guard(input.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(input.device().index()).stream();
  check_status(hprn_rms_norm_fp8_group(
      out.data_ptr(), scales.data_ptr<float>(), scales.stride(0), scales.stride(1),
      input.data_ptr(), weight.data_ptr(), residual.has_value() ? residual->data_ptr() : nullptr,
      c.rows, c.hidden, c.os, c.xs, c.rs, eps, c.dtype, static_cast<int>(group_size),
      scale_pow2 ? 1 : 0, stream, HPRN_LAUNCH_DEFAULT));
}

// out[..., d] = act(input[..., :d]) * input[..., d:]  (extension past the reference).
void act_and_mul(at::Tensor& out, const at::Tensor& input, int act) {
  TORCH_CHECK(input.dim() >= 1 && input.size(-1) % 2 == 0, "input.size(-1) must be even");
  const int64_t d = input.size(-1) / 2;
  TORCH_CHECK(out.dim() == input.dim(), "out.dim() == input.dim()");
  for (int64_t i = 0; i + 1 < input.dim(); ++i)
    TORCH_CHECK(out.size(i) == input.size(i), "out and input must agree on leading dimensions");
  TORCH_CHECK(out.size(-1) == d, "out.size(-1) == input.size(-1) / 2");
  TORCH_CHECK(input.is_cuda() && out.is_cuda() && out.device() == input.device(),
              "out and input must be CUDA tensors on the same device");
  TORCH_CHECK(out.scalar_type() == input.scalar_type(), "out and input must have the same dtype");
  const int dtype = dtype_code(input);
  if (out.numel() == 0) return;
  TORCH_CHECK(input.stride(-1) == 1 && (d == 1 || out.stride(-1) == 1),
              "input and out must be contiguous in the last dimension");
  int64_t rows = 0, is = 0, orows = 0, os = 0;
  rows_of(input, "input", &rows, &is);
  rows_of(out, "out", &orows, &os);
  const c10::cuda::CUDAGuard guard(input.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(input.device().index()).stream();
  check_status(hprn_act_and_mul(out.data_ptr(), input.data_ptr(), rows, d, os, is, act, dtype,
                                stream, HPRN_LAUNCH_DEFAULT));
}

void silu_and_mul(at::Tensor& out, const at::Tensor& input) { act_and_mul(out, input, HPRN_ACT_SILU); }
void gelu_and_mul(at::Tensor& out, const at::Tensor& input) { act_and_mul(out, input, HPRN_ACT_GELU); }
void gelu_tanh_and_mul(at::Tensor& out, const at::Tensor& input) {
  act_and_mul(out, input, HPRN_ACT_GELU_TANH);
}

// Shape-only kernels for tracing (torch.compile / FakeTensor): the ops return
// nothing and only mutate their annotated arguments.
void rms_norm_meta(at::Tensor&, const at::Tensor&, at::Tensor&, double) {}
void relu_meta(at::Tensor&, const at::Tensor&) {}
void rms_norm_out_meta(at::Tensor&, const at::Tensor&, const at::Tensor&,
                       c10::optional<at::Tensor>, double) {}
void rms_norm_fp8_meta(at::Tensor&, const at::Tensor&, const at::Tensor&,
                       c10::optional<at::Tensor>, double, c10::optional<at::Tensor>,
                       c10::optional<at::Tensor>) {}
void act_and_mul_meta(at::Tensor&, const at::Tensor&) {}
void rms_norm_nvfp4_meta(at::Tensor&, at::Tensor&, const at::Tensor&, const at::Tensor&,
                         c10::optional<at::Tensor>, double, const at::Tensor&) {}
void rms_norm_fp8_group_meta(at::Tensor&, at::Tensor&, const at::Tensor&, const at::Tensor&,
                             c10::optional<at::Tensor>, double, int64_t, bool) {}

}  // namespace

TORCH_LIBRARY(hp_rms_norm, m) {
  // The reference's two operators.
  m.def("rms_norm(Tensor(a!) input, Tensor weight, Tensor(b!) residual, float eps) -> ()");
  m.def("relu(Tensor(a!) out, Tensor input) -> ()");
  // Extensions: plain / out-of-place RMSNorm and fp8-output RMSNorm.
  m.def("rms_norm_out(Tensor(a!) out, Tensor input, Tensor weight, Tensor(b!)? residual, "
        "float eps) -> ()");
  m.def("rms_norm_fp8(Tensor(a!) out, Tensor input, Tensor weight, Tensor(b!)? residual, "
        "float eps, Tensor? scale, Tensor(c!)? row_scales) -> ()");
  m.def("rms_norm_nvfp4(Tensor(a!) out, Tensor(b!) block_scales, Tensor input, Tensor weight, "
        "Tensor(c!)? residual, float eps, Tensor global_scale) -> ()");
  m.def("rms_norm_fp8_group(Tensor(a!) out, Tensor(b!) scales, Tensor input, Tensor weight, "
        "Tensor(c!)? residual, float eps, int group_size, bool scale_pow2) -> ()");
  // Extensions: gated activations.
  m.def("silu_and_mul(Tensor(a!) out, Tensor input) -> ()");
  m.def("gelu_and_mul(Tensor(a!) out, Tensor input) -> ()");
  m.def("gelu_tanh_and_mul(Tensor(a!) out, Tensor input) -> ()");
}

TORCH_LIBRARY_IMPL(hp_rms_norm, CUDA, m) {
  m.impl("rms_norm", &rms_norm);
  m.impl("relu", &relu);
  m.impl("rms_norm_out", &rms_norm_out);
  m.impl("rms_norm_fp8", &rms_norm_fp8);
  m.impl("rms_norm_nvfp4", &rms_norm_nvfp4);
  m.impl("rms_norm_fp8_group", &rms_norm_fp8_group);
  m.impl("silu_and_mul", &silu_and_mul);
  m.impl("gelu_and_mul", &gelu_and_mul);
  m.impl("gelu_tanh_and_mul", &gelu_tanh_and_mul);
}

TORCH_LIBRARY_IMPL(hp_rms_norm, Meta, m) {
  m.impl("rms_norm", &rms_norm_meta);
  m.impl("relu", &relu_meta);
  m.impl("rms_norm_out", &rms_norm_out_meta);
  m.impl("rms_norm_fp8", &rms_norm_fp8_meta);
  m.impl("rms_norm_nvfp4", &rms_norm_nvfp4_meta);
  m.impl("rms_norm_fp8_group", &rms_norm_fp8_group_meta);
  m.impl("silu_and_mul", &act_and_mul_meta);
  m.impl("gelu_and_mul", &act_and_mul_meta);
  m.impl("gelu_tanh_and_mul", &act_and_mul_meta);
}
