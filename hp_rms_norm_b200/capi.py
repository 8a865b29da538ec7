"""ctypes binding of the C ABI (include/hp_rms_norm_b200.h).

This is what a non-torch caller would bind, and what the GPU parity tests call:
plain device pointers, element counts, row strides, a dtype code and a
``cudaStream_t`` as an integer.  Errors raise ``HprnError`` carrying the
library's status code and message.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libhp_rms_norm_b200.so")

DTYPE_BF16 = 0
DTYPE_FP16 = 1

OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED_DTYPE = -2
ERR_UNSUPPORTED_DEVICE = -3
ERR_CUDA = -4

LAUNCH_PDL = 1
LAUNCH_DEFAULT = LAUNCH_PDL

ACT_SILU = 0
ACT_GELU = 1
ACT_GELU_TANH = 2

OUT_SAME = 0
OUT_FP8_E4M3_STATIC = 1
OUT_FP8_E4M3_DYNAMIC = 2
OUT_NVFP4 = 3
OUT_FP8_E4M3_GROUP = 4

# Every symbol include/hp_rms_norm_b200.h declares.
EXPORTED = (
    "hprn_rms_norm",
    "hprn_relu",
    "hprn_rms_norm_ex",
    "hprn_relu_ex",
    "hprn_rms_norm_out",
    "hprn_act_and_mul",
    "hprn_rms_norm_nvfp4",
    "hprn_last_error",
    "hprn_status_string",
    "hprn_version",
    "hprn_rms_norm_plan",
    "hprn_set_plan_override",
    "hprn_wait_timeouts",
    "hprn_rms_norm_fp8_group",
    "hprn_test_stall_bulk_copy",
)


class HprnError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads the C-ABI library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `python hp_rms_norm_b200/build.py` "
            "(the CUDA library is required; there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    vp, i64, c_int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.hprn_rms_norm.argtypes = [vp, vp, vp, i64, i64, i64, i64, ctypes.c_double, c_int, vp]
    lib.hprn_rms_norm.restype = c_int
    lib.hprn_relu.argtypes = [vp, vp, i64, i64, i64, i64, c_int, vp]
    lib.hprn_relu.restype = c_int
    u32 = ctypes.c_uint
    lib.hprn_rms_norm_ex.argtypes = [vp, vp, vp, i64, i64, i64, i64, ctypes.c_double, c_int, vp, u32]
    lib.hprn_rms_norm_ex.restype = c_int
    lib.hprn_relu_ex.argtypes = [vp, vp, i64, i64, i64, i64, c_int, vp, u32]
    lib.hprn_relu_ex.restype = c_int
    lib.hprn_rms_norm_out.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64, ctypes.c_double,
                                      c_int, c_int, vp, vp, vp, u32]
    lib.hprn_rms_norm_out.restype = c_int
    lib.hprn_act_and_mul.argtypes = [vp, vp, i64, i64, i64, i64, c_int, c_int, vp, u32]
    lib.hprn_act_and_mul.restype = c_int
    lib.hprn_rms_norm_nvfp4.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64,
                                        ctypes.c_double, c_int, vp, vp, u32]
    lib.hprn_rms_norm_nvfp4.restype = c_int
    lib.hprn_last_error.argtypes = []
    lib.hprn_last_error.restype = ctypes.c_char_p
    lib.hprn_status_string.argtypes = [c_int]
    lib.hprn_status_string.restype = ctypes.c_char_p
    lib.hprn_version.argtypes = []
    lib.hprn_version.restype = c_int
    lib.hprn_rms_norm_plan.argtypes = [i64, i64, c_int, vp, vp, i64, i64, ctypes.c_char_p, c_int]
    lib.hprn_rms_norm_plan.restype = c_int
    lib.hprn_set_plan_override.argtypes = [ctypes.c_char_p]
    lib.hprn_set_plan_override.restype = c_int
    lib.hprn_wait_timeouts.argtypes = [ctypes.POINTER(ctypes.c_uint), c_int]
    lib.hprn_wait_timeouts.restype = c_int
    lib.hprn_test_stall_bulk_copy.argtypes = [i64, ctypes.c_uint64]
    lib.hprn_test_stall_bulk_copy.restype = c_int
    lib.hprn_rms_norm_fp8_group.argtypes = [vp, vp, i64, i64, vp, vp, vp, i64, i64, i64, i64, i64,
                                            ctypes.c_double, c_int, c_int, c_int, vp, u32]
    lib.hprn_rms_norm_fp8_group.restype = c_int
    _lib = lib
    return lib


def _check(status: int) -> None:
    if status != OK:
        lib = load()
        raise HprnError(status, lib.hprn_last_error().decode())


def rms_norm(input_ptr: int, weight_ptr: int, residual_ptr: int, rows: int, hidden: int,
             input_row_stride: int, residual_row_stride: int, eps: float, dtype: int,
             stream: int = 0, flags: int | None = None) -> None:
    """hprn_rms_norm, or hprn_rms_norm_ex when launch `flags` are given."""
    lib = load()
    if flags is None:
        st = lib.hprn_rms_norm(input_ptr, weight_ptr, residual_ptr, rows, hidden,
                               input_row_stride, residual_row_stride, eps, dtype, stream)
    else:
        st = lib.hprn_rms_norm_ex(input_ptr, weight_ptr, residual_ptr, rows, hidden,
                                  input_row_stride, residual_row_stride, eps, dtype, stream, flags)
    _check(st)


def relu(out_ptr: int, input_ptr: int, rows: int, hidden: int, out_row_stride: int,
         input_row_stride: int, dtype: int, stream: int = 0, flags: int | None = None) -> None:
    """hprn_relu, or hprn_relu_ex when launch `flags` are given."""
    lib = load()
    if flags is None:
        st = lib.hprn_relu(out_ptr, input_ptr, rows, hidden, out_row_stride, input_row_stride,
                           dtype, stream)
    else:
        st = lib.hprn_relu_ex(out_ptr, input_ptr, rows, hidden, out_row_stride,
                              input_row_stride, dtype, stream, flags)
    _check(st)


def rms_norm_out(out_ptr: int, input_ptr: int, weight_ptr: int, residual_ptr: int | None,
                 rows: int, hidden: int, out_row_stride: int, input_row_stride: int,
                 residual_row_stride: int, eps: float, dtype: int, out_form: int = OUT_SAME,
                 scale_ptr: int | None = None, row_scales_ptr: int | None = None,
                 stream: int = 0, flags: int = LAUNCH_DEFAULT) -> None:
    _check(load().hprn_rms_norm_out(out_ptr, input_ptr, weight_ptr, residual_ptr, rows, hidden,
                                    out_row_stride, input_row_stride, residual_row_stride, eps,
                                    dtype, out_form, scale_ptr, row_scales_ptr, stream, flags))


def rms_norm_nvfp4(out_ptr: int, block_scales_ptr: int, input_ptr: int, weight_ptr: int,
                   residual_ptr: int | None, rows: int, hidden: int, out_row_stride: int,
                   input_row_stride: int, residual_row_stride: int, eps: float, dtype: int,
                   global_scale_ptr: int, stream: int = 0, flags: int = LAUNCH_DEFAULT) -> None:
    _check(load().hprn_rms_norm_nvfp4(out_ptr, block_scales_ptr, input_ptr, weight_ptr,
                                      residual_ptr, rows, hidden, out_row_stride, input_row_stride,
                                      residual_row_stride, eps, dtype, global_scale_ptr, stream,
                                      flags))


def rms_norm_fp8_group(out_ptr: int, scales_ptr: int, scale_row_stride: int,
                       scale_group_stride: int, input_ptr: int, weight_ptr: int,
                       residual_ptr: int | None, rows: int, hidden: int, out_row_stride: int,
                       input_row_stride: int, residual_row_stride: int, eps: float, dtype: int,
                       group_size: int = 128, scale_pow2: bool = False, stream: int = 0,
                       flags: int = LAUNCH_DEFAULT) -> None:
    _check(load().hprn_rms_norm_fp8_group(out_ptr, scales_ptr, scale_row_stride,
                                          scale_group_stride, input_ptr, weight_ptr, residual_ptr,
                                          rows, hidden, out_row_stride, input_row_stride,
                                          residual_row_stride, eps, dtype, group_size,
                                          1 if scale_pow2 else 0, stream, flags))


def act_and_mul(out_ptr: int, input_ptr: int, rows: int, d: int, out_row_stride: int,
                input_row_stride: int, act: int, dtype: int, stream: int = 0,
                flags: int = LAUNCH_DEFAULT) -> None:
    _check(load().hprn_act_and_mul(out_ptr, input_ptr, rows, d, out_row_stride, input_row_stride,
                                   act, dtype, stream, flags))


def plan(rows: int, hidden: int, dtype: int = DTYPE_BF16, input_ptr: int = 0,
         residual_ptr: int = 0, input_row_stride: int | None = None,
         residual_row_stride: int | None = None) -> str:
    buf = ctypes.create_string_buffer(128)
    xs = hidden if input_row_stride is None else input_row_stride
    rs = hidden if residual_row_stride is None else residual_row_stride
    _check(load().hprn_rms_norm_plan(rows, hidden, dtype, input_ptr, residual_ptr, xs, rs, buf, 128))
    return buf.value.decode()


def set_plan_override(plan_str: str | None) -> None:
    _check(load().hprn_set_plan_override(plan_str.encode() if plan_str else None))


def wait_timeouts(reset: bool = False) -> int:
    """CTAs on the current device that gave up a bounded wait (hprn_wait_timeouts)."""
    n = ctypes.c_uint(0)
    _check(load().hprn_wait_timeouts(ctypes.byref(n), 1 if reset else 0))
    return int(n.value)


def test_stall_bulk_copy(row: int | None, wait_limit_ns: int = 0) -> None:
    """Test hook (hprn_test_stall_bulk_copy): later TMA-staged launches make the
    staged copy of `row` stall so its bounded wait runs out; None turns it off."""
    _check(load().hprn_test_stall_bulk_copy(-1 if row is None else row, wait_limit_ns))


def version() -> int:
    return int(load().hprn_version())


# --- torch conveniences (device pointers from tensors) ----------------------

def dtype_code(t) -> int:
    import torch

    if t.dtype == torch.bfloat16:
        return DTYPE_BF16
    if t.dtype == torch.float16:
        return DTYPE_FP16
    raise HprnError(ERR_UNSUPPORTED_DTYPE, "dtype must be kFloat16 or kBFloat16")


def rms_norm_tensors(inp, weight, res, eps: float, stream: int | None = None,
                     flags: int | None = None) -> None:
    """C-ABI call on 2-D CUDA tensors (row stride from the tensors)."""
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(inp.device).cuda_stream
    rows, hidden = inp.shape
    rms_norm(inp.data_ptr(), weight.data_ptr(), res.data_ptr(), rows, hidden, inp.stride(0),
             res.stride(0), eps, dtype_code(inp), stream, flags)


def relu_tensors(out, inp, stream: int | None = None, flags: int | None = None) -> None:
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(inp.device).cuda_stream
    rows, hidden = inp.shape
    relu(out.data_ptr(), inp.data_ptr(), rows, hidden, out.stride(0), inp.stride(0),
         dtype_code(inp), stream, flags)


def rms_norm_out_tensors(out, inp, weight, res, eps: float, scale=None, row_scales=None,
                         stream: int | None = None, flags: int = LAUNCH_DEFAULT) -> None:
    """hprn_rms_norm_out on 2-D CUDA tensors; `res` may be None (plain RMSNorm).
    The output form follows out's dtype (16-bit: same; float8_e4m3fn: static
    with `scale`, dynamic with `row_scales`)."""
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(inp.device).cuda_stream
    rows, hidden = inp.shape
    if out.dtype == torch.float8_e4m3fn:
        form = OUT_FP8_E4M3_STATIC if scale is not None else OUT_FP8_E4M3_DYNAMIC
    else:
        form = OUT_SAME
    rms_norm_out(out.data_ptr(), inp.data_ptr(), weight.data_ptr(),
                 res.data_ptr() if res is not None else None, rows, hidden, out.stride(0),
                 inp.stride(0), res.stride(0) if res is not None else hidden, eps, dtype_code(inp),
                 form, scale.data_ptr() if scale is not None else None,
                 row_scales.data_ptr() if row_scales is not None else None, stream, flags)


def act_and_mul_tensors(out, inp, act: int, stream: int | None = None,
                        flags: int = LAUNCH_DEFAULT) -> None:
    """hprn_act_and_mul on 2-D CUDA tensors: inp [rows, 2d] -> out [rows, d]."""
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(inp.device).cuda_stream
    rows, d = out.shape
    act_and_mul(out.data_ptr(), inp.data_ptr(), rows, d, out.stride(0), inp.stride(0), act,
                dtype_code(inp), stream, flags)


def rms_norm_fp8_group_tensors(out, scales, inp, weight, res, eps: float, group_size: int = 128,
                               scale_pow2: bool = False, stream: int | None = None,
                               flags: int = LAUNCH_DEFAULT) -> None:
    """hprn_rms_norm_fp8_group on 2-D CUDA tensors: out float8_e4m3fn / uint8
    [rows, hidden], scales float32 [rows, hidden / group_size] with any strides
    (row-major, or a transposed view for column-major scales)."""
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(inp.device).cuda_stream
    rows, hidden = inp.shape
    rms_norm_fp8_group(out.data_ptr(), scales.data_ptr(), scales.stride(0), scales.stride(1),
                       inp.data_ptr(), weight.data_ptr(), res.data_ptr() if res is not None else None,
                       rows, hidden, out.stride(0), inp.stride(0),
                       res.stride(0) if res is not None else hidden, eps, dtype_code(inp),
                       group_size, scale_pow2, stream, flags)


def rms_norm_nvfp4_tensors(out, block_scales, inp, weight, res, eps: float, global_scale,
                           stream: int | None = None, flags: int = LAUNCH_DEFAULT) -> None:
    """hprn_rms_norm_nvfp4 on 2-D CUDA tensors: out uint8 [rows, hidden/2] (packed
    e2m1 pairs), block_scales uint8 / float8_e4m3fn [rows, hidden/16]."""
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(inp.device).cuda_stream
    rows, hidden = inp.shape
    rms_norm_nvfp4(out.data_ptr(), block_scales.data_ptr(), inp.data_ptr(), weight.data_ptr(),
                   res.data_ptr() if res is not None else None, rows, hidden, out.stride(0) * 2,
                   inp.stride(0), res.stride(0) if res is not None else hidden, eps,
                   dtype_code(inp), global_scale.data_ptr(), stream, flags)
