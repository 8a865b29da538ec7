"""Comparison helpers shared by the tests (bit patterns, ulp distances)."""
from __future__ import annotations

import numpy as np


def ordered(bits: np.ndarray) -> np.ndarray:
    """Maps 16-bit float patterns to integers whose difference is the ulp distance."""
    b = bits.astype(np.int32)
    mag = b & 0x7FFF
    return np.where(b & 0x8000, -mag, mag)


def is_nan(bits: np.ndarray, dtype_code: int) -> np.ndarray:
    b = bits.astype(np.int32) & 0x7FFF
    return b > (0x7F80 if dtype_code == 0 else 0x7C00)


def ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return np.abs(ordered(a) - ordered(b))


def as_float(bits: np.ndarray, dtype_code: int) -> np.ndarray:
    """Exact float32 values of bf16 (code 0) or fp16 (code 1) bit patterns."""
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    if dtype_code == 0:
        return (b.astype(np.uint32) << 16).view(np.float32)
    return b.view(np.float16).astype(np.float32)


def assert_output_close(got: np.ndarray, want: np.ndarray, dtype_code: int, max_ulp: int = 1,
                        atol: float = 1e-2, rtol: float = 1e-2, label: str = "") -> float:
    """The normalised-output bar: within `max_ulp` ulps of T AND within atol/rtol
    (1e-2 / 1e-2, the tolerance the task states for the normalised output).
    NaN must match NaN.  Returns the fraction of elements that differ at all."""
    got = np.asarray(got).reshape(-1)
    want = np.asarray(want).reshape(-1)
    gn, wn = is_nan(got, dtype_code), is_nan(want, dtype_code)
    assert (gn == wn).all(), f"{label}: NaN positions differ"
    m = ~wn
    d = ulp_diff(got[m], want[m])
    worst = int(d.max()) if d.size else 0
    assert worst <= max_ulp, f"{label}: max ulp difference {worst} > {max_ulp}"
    gf, wf = as_float(got[m], dtype_code), as_float(want[m], dtype_code)
    fin = np.isfinite(wf)
    err = np.abs(gf[fin] - wf[fin])
    tol = atol + rtol * np.abs(wf[fin])
    assert (err <= tol).all(), f"{label}: outside atol/rtol 1e-2 at {np.argmax(err - tol)}"
    assert (gf[~fin] == wf[~fin]).all(), f"{label}: infinities differ"
    return float((d > 0).mean()) if d.size else 0.0


def assert_bits_equal(got: np.ndarray, want: np.ndarray, dtype_code: int, label: str = "",
                      nan_payload: bool = True) -> None:
    """Bit-exact comparison; with nan_payload=False any NaN matches any NaN."""
    got = np.asarray(got).reshape(-1)
    want = np.asarray(want).reshape(-1)
    if not nan_payload:
        gn, wn = is_nan(got, dtype_code), is_nan(want, dtype_code)
        assert (gn == wn).all(), f"{label}: NaN positions differ"
        got, want = got[~wn], want[~wn]
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, (f"{label}: {bad.size} elements differ, first at {bad[0]}: "
                           f"got {got[bad[0]]:#06x} want {want[bad[0]]:#06x}")


def assert_activation_close(got: np.ndarray, want: np.ndarray, dtype_code: int, label: str = "",
                            max_far: float = 0.005, tiny: float = 2.0 ** -10) -> float:
    """Bar for activations: within atol/rtol 1e-2 everywhere, and more than one
    ulp apart in at most `max_far` of the elements whose magnitude is at least
    `tiny`.  Below it are the tails where the result comes from a cancellation
    (1 + erf(a), 1 + tanh(a) as a -> -inf): there one fp32 ulp of the library
    function is many 16-bit ulps of a tiny result, and implementations of
    erff / tanhf legitimately disagree.  Returns the far fraction."""
    got = np.asarray(got).reshape(-1)
    want = np.asarray(want).reshape(-1)
    gn, wn = is_nan(got, dtype_code), is_nan(want, dtype_code)
    assert (gn == wn).all(), f"{label}: NaN positions differ"
    m = ~wn
    gf, wf = as_float(got[m], dtype_code), as_float(want[m], dtype_code)
    assert np.all(np.abs(gf - wf) <= 1e-2 + 1e-2 * np.abs(wf)), f"{label}: outside atol/rtol 1e-2"
    big = np.abs(wf) >= tiny
    far = float((ulp_diff(got[m][big], want[m][big]) > 1).mean()) if big.any() else 0.0
    assert far <= max_far, f"{label}: {far:.4%} of elements more than 1 ulp apart"
    return far
