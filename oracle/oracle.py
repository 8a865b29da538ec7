"""Python face of the oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module, and only as the checker or the timed CPU baseline; the
product package never imports it.

* ``fused_add_rms_norm`` / ``relu``: the plain-C restatement in
  rms_norm_oracle.c (reference arithmetic: hp_rms_norm/csrc/cuda/hp_rms_norm.cuh:186-251;
  ReLU: torch.relu semantics), on numpy uint16 bit patterns.
* ``eager_formula``: the reference test's own PyTorch-eager formula
  (test/test_hp_rms_norm.py:6-19: ``inp + res`` in the storage dtype, then
  ``torch.rms_norm``), restated here so it runs where the reference tree is
  absent.  bench.py times it on the host cores as the CPU baseline.
* ``ReferenceKernels``: ctypes handle to oracle/_ref/libhp_rms_norm_ref.so, the
  reference's own CUDA launchers compiled from its sources (GPU comparator).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

BF16 = 0
FP16 = 1
SS_UNROUNDED = 0  # the CUDA kernel's sum of squares (hp_rms_norm.cuh:190-193)
SS_ROUNDED = 1    # the test formula's sum of squares (test_hp_rms_norm.py:13-19)

_lib = None


def _load():
    global _lib
    if _lib is None:
        path = _build.ORACLE_SO
        if not os.path.exists(path):
            _build.build_oracle()
        lib = ctypes.CDLL(path)
        u16p = ctypes.POINTER(ctypes.c_uint16)
        f32p = ctypes.POINTER(ctypes.c_float)
        i64 = ctypes.c_int64
        lib.oracle_fused_add_rms_norm.argtypes = [ctypes.c_int, u16p, u16p, u16p, i64, i64, i64,
                                                  i64, ctypes.c_double, ctypes.c_int]
        lib.oracle_fused_add_rms_norm.restype = None
        lib.oracle_relu.argtypes = [ctypes.c_int, u16p, u16p, i64]
        lib.oracle_relu.restype = None
        lib.oracle_to_f32.argtypes = [ctypes.c_int, u16p, f32p, i64]
        lib.oracle_from_f32.argtypes = [ctypes.c_int, f32p, u16p, i64]
        lib.oracle_num_threads.restype = ctypes.c_int
        vp = ctypes.c_void_p
        lib.oracle_rms_norm_out.argtypes = [ctypes.c_int, vp, u16p, u16p, vp, i64, i64, i64, i64,
                                            i64, ctypes.c_double, ctypes.c_int, ctypes.c_float, vp]
        lib.oracle_rms_norm_out.restype = None
        lib.oracle_f32_to_e4m3.argtypes = [vp, vp, i64]
        lib.oracle_f32_to_e4m3.restype = None
        lib.oracle_act_and_mul.argtypes = [ctypes.c_int, ctypes.c_int, u16p, u16p, i64, i64]
        lib.oracle_act_and_mul.restype = None
        lib.oracle_f32_to_e2m1.argtypes = [vp, vp, i64]
        lib.oracle_f32_to_e2m1.restype = None
        lib.oracle_rms_norm_nvfp4.argtypes = [ctypes.c_int, vp, vp, u16p, u16p, vp, i64, i64,
                                              ctypes.c_double, ctypes.c_float]
        lib.oracle_rms_norm_nvfp4.restype = None
        lib.oracle_rms_norm_fp8_group.argtypes = [ctypes.c_int, vp, vp, u16p, u16p, vp, i64, i64,
                                                  ctypes.c_double, ctypes.c_int, ctypes.c_int]
        lib.oracle_rms_norm_fp8_group.restype = None
        _lib = lib
    return _lib


def _u16(a: np.ndarray):
    assert a.dtype == np.uint16 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16))


def dtype_code(name) -> int:
    s = str(name)
    if "bfloat16" in s or s == "bf16":
        return BF16
    if "float16" in s or s in ("fp16", "half"):
        return FP16
    raise ValueError(f"unsupported dtype {name}")


def fused_add_rms_norm(dtype: int, x: np.ndarray, w: np.ndarray, r: np.ndarray, eps: float,
                       ss_mode: int = SS_UNROUNDED) -> tuple[np.ndarray, np.ndarray]:
    """Returns (output, residual) as new uint16 arrays; inputs are not modified."""
    lib = _load()
    hidden = x.shape[-1]
    xo = np.ascontiguousarray(x, dtype=np.uint16).copy()
    ro = np.ascontiguousarray(r, dtype=np.uint16).copy()
    wc = np.ascontiguousarray(w, dtype=np.uint16)
    assert wc.shape == (hidden,) and ro.shape == xo.shape
    rows = xo.size // hidden if hidden else 0
    lib.oracle_fused_add_rms_norm(dtype, _u16(xo), _u16(wc), _u16(ro), rows, hidden, hidden,
                                  hidden, float(eps), ss_mode)
    return xo, ro


def rms_norm_out(dtype: int, x: np.ndarray, w: np.ndarray, eps: float, r: np.ndarray | None = None,
                 fp8: str | None = None, scale: float = 1.0):
    """The generalised row op (rms_norm_oracle.c: oracle_rms_norm_out).

    fp8: None (16-bit output), "static" (e4m3 of y / scale) or "dynamic"
    (per-row scales).  Returns (out, residual or None, row_scales or None);
    inputs are not modified."""
    lib = _load()
    hidden = x.shape[-1]
    xc = np.ascontiguousarray(x, dtype=np.uint16)
    rows = xc.size // hidden
    wc = np.ascontiguousarray(w, dtype=np.uint16)
    rc = None if r is None else np.ascontiguousarray(r, dtype=np.uint16).copy()
    out = np.empty(xc.shape, dtype=np.uint8 if fp8 else np.uint16)
    scales = np.zeros(rows, dtype=np.float32) if fp8 == "dynamic" else None
    lib.oracle_rms_norm_out(dtype, out.ctypes.data, _u16(xc), _u16(wc),
                            None if rc is None else rc.ctypes.data, rows, hidden, hidden, hidden,
                            hidden, float(eps), 1 if fp8 else 0, float(scale),
                            None if scales is None else scales.ctypes.data)
    return out, rc, scales


def f32_to_e4m3(vals: np.ndarray) -> np.ndarray:
    lib = _load()
    v = np.ascontiguousarray(vals, dtype=np.float32)
    out = np.empty(v.shape, dtype=np.uint8)
    lib.oracle_f32_to_e4m3(v.ctypes.data, out.ctypes.data, v.size)
    return out


def f32_to_e2m1(vals: np.ndarray) -> np.ndarray:
    lib = _load()
    v = np.ascontiguousarray(vals, dtype=np.float32)
    out = np.empty(v.shape, dtype=np.uint8)
    lib.oracle_f32_to_e2m1(v.ctypes.data, out.ctypes.data, v.size)
    return out


def rms_norm_nvfp4(dtype: int, x: np.ndarray, w: np.ndarray, eps: float, global_scale: float,
                   r: np.ndarray | None = None):
    """NVFP4 output of the row op: returns (packed fp4 [rows, hidden/2] uint8,
    block scales [rows, hidden/16] e4m3 bytes, residual or None)."""
    lib = _load()
    hidden = x.shape[-1]
    xc = np.ascontiguousarray(x, dtype=np.uint16)
    rows = xc.size // hidden
    rc = None if r is None else np.ascontiguousarray(r, dtype=np.uint16).copy()
    out = np.empty((rows, hidden // 2), dtype=np.uint8)
    sf = np.empty((rows, hidden // 16), dtype=np.uint8)
    lib.oracle_rms_norm_nvfp4(dtype, out.ctypes.data, sf.ctypes.data, _u16(xc),
                              _u16(np.ascontiguousarray(w, dtype=np.uint16)),
                              None if rc is None else rc.ctypes.data, rows, hidden, float(eps),
                              float(global_scale))
    return out, sf, rc


def rms_norm_fp8_group(dtype: int, x: np.ndarray, w: np.ndarray, eps: float, group: int = 128,
                       pow2: bool = False, r: np.ndarray | None = None):
    """Per-token-group fp8 output of the row op: returns (e4m3 codes
    [rows, hidden] uint8, scales [rows, hidden/group] float32, residual or None)."""
    lib = _load()
    hidden = x.shape[-1]
    xc = np.ascontiguousarray(x, dtype=np.uint16)
    rows = xc.size // hidden
    rc = None if r is None else np.ascontiguousarray(r, dtype=np.uint16).copy()
    out = np.empty((rows, hidden), dtype=np.uint8)
    sc = np.empty((rows, hidden // group), dtype=np.float32)
    lib.oracle_rms_norm_fp8_group(dtype, out.ctypes.data, sc.ctypes.data, _u16(xc),
                                  _u16(np.ascontiguousarray(w, dtype=np.uint16)),
                                  None if rc is None else rc.ctypes.data, rows, hidden, float(eps),
                                  int(group), 1 if pow2 else 0)
    return out, sc, rc


ACTS = {"silu": 0, "gelu": 1, "gelu_tanh": 2}


def act_and_mul(dtype: int, act: str, x: np.ndarray) -> np.ndarray:
    """Gated activation on [rows, 2d] bit patterns -> [rows, d]."""
    lib = _load()
    xc = np.ascontiguousarray(x, dtype=np.uint16)
    rows, two_d = xc.shape
    out = np.empty((rows, two_d // 2), dtype=np.uint16)
    lib.oracle_act_and_mul(dtype, ACTS[act], _u16(out), _u16(xc), rows, two_d // 2)
    return out


def relu(dtype: int, x: np.ndarray) -> np.ndarray:
    lib = _load()
    xc = np.ascontiguousarray(x, dtype=np.uint16)
    out = np.empty_like(xc)
    lib.oracle_relu(dtype, _u16(out), _u16(xc), xc.size)
    return out


def to_f32(dtype: int, bits: np.ndarray) -> np.ndarray:
    lib = _load()
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    out = np.empty(b.shape, dtype=np.float32)
    lib.oracle_to_f32(dtype, _u16(b), out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), b.size)
    return out


def from_f32(dtype: int, vals: np.ndarray) -> np.ndarray:
    lib = _load()
    v = np.ascontiguousarray(vals, dtype=np.float32)
    out = np.empty(v.shape, dtype=np.uint16)
    lib.oracle_from_f32(dtype, v.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), _u16(out), v.size)
    return out


def num_threads() -> int:
    return int(_load().oracle_num_threads())


def eager_formula(inp, res, weight, eps):
    """test/test_hp_rms_norm.py:6-19, restated: returns (out, inp_res)."""
    import torch

    inp_res = inp + res
    out = torch.rms_norm(inp_res, normalized_shape=(inp.shape[-1],), weight=weight, eps=eps)
    return out, inp_res


class ReferenceKernels:
    """The reference's CUDA launchers (oracle/_ref), driven through ctypes."""

    def __init__(self, path: str | None = None):
        path = path or _build.REF_SO
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        import torch  # noqa: F401  (the shim resolves libc10/libtorch from the loaded torch)

        lib = ctypes.CDLL(path)
        vp = ctypes.c_void_p
        lib.ref_rms_norm.argtypes = [ctypes.c_int, vp, vp, vp, ctypes.c_longlong, ctypes.c_int,
                                     ctypes.c_double, vp]
        lib.ref_rms_norm.restype = ctypes.c_int
        lib.ref_relu.argtypes = [ctypes.c_int, vp, vp, ctypes.c_longlong, ctypes.c_int, vp]
        lib.ref_relu.restype = ctypes.c_int
        lib.ref_last_error.restype = ctypes.c_char_p
        self.lib = lib

    def rms_norm(self, inp, weight, res, eps, stream: int = 0) -> None:
        h = inp.shape[-1]
        rc = self.lib.ref_rms_norm(dtype_code(inp.dtype), inp.data_ptr(), weight.data_ptr(),
                                   res.data_ptr(), inp.numel() // h, h, float(eps), stream)
        if rc:
            raise RuntimeError(self.lib.ref_last_error().decode())

    def relu(self, out, inp, stream: int = 0) -> None:
        h = inp.shape[-1]
        rc = self.lib.ref_relu(dtype_code(inp.dtype), out.data_ptr(), inp.data_ptr(),
                               inp.numel() // h, h, stream)
        if rc:
            raise RuntimeError(self.lib.ref_last_error().decode())
