"""The oracle, pinned against the reference's own test formula (CPU only).

The golden fixtures were produced by importing ``ref_rms_norm`` from the
reference's test/test_hp_rms_norm.py (see tests/golden/make_golden.py).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.numerics import assert_bits_equal, assert_output_close, ulp_diff


def _code(case: str) -> int:
    return O.BF16 if case.startswith("bf16") else O.FP16


def test_golden_cases_present(rms_golden):
    assert len(rms_golden) == 18
    assert {c[:4] for c in rms_golden} == {"bf16", "fp16"}


def test_oracle_matches_reference_formula(rms_golden):
    """SS_ROUNDED restates test_hp_rms_norm.py:6-19: residual bit-exact, output
    bit-exact for bf16 and within 1 ulp for fp16 (torch's CPU reduction order)."""
    for case, c in rms_golden.items():
        d = _code(case)
        out, res = O.fused_add_rms_norm(d, c["x"], c["w"], c["r"], c["eps"], O.SS_ROUNDED)
        assert_bits_equal(res, c["res"], d, label=case + " residual")
        if d == O.BF16:
            assert_bits_equal(out, c["out"], d, label=case + " output")
        else:
            frac = assert_output_close(out, c["out"], d, max_ulp=1, label=case)
            assert frac < 1e-3, case


def test_kernel_arithmetic_within_one_ulp_of_reference_formula(rms_golden):
    """SS_UNROUNDED is the reference CUDA kernel's arithmetic (sum of squares of
    the unrounded fp32 sums, hp_rms_norm.cuh:190-193): the same residual, and an
    output within 1 ulp of the test formula."""
    for case, c in rms_golden.items():
        d = _code(case)
        out, res = O.fused_add_rms_norm(d, c["x"], c["w"], c["r"], c["eps"], O.SS_UNROUNDED)
        assert_bits_equal(res, c["res"], d, label=case)
        assert_output_close(out, c["out"], d, max_ulp=1, label=case)


def test_oracle_does_not_modify_inputs(rms_golden):
    c = rms_golden["bf16_c0_r7_h1024"]
    x0, r0 = c["x"].copy(), c["r"].copy()
    O.fused_add_rms_norm(O.BF16, c["x"], c["w"], c["r"], c["eps"])
    assert (c["x"] == x0).all() and (c["r"] == r0).all()


@pytest.mark.parametrize("code,tdtype", [(O.BF16, torch.bfloat16), (O.FP16, torch.float16)])
def test_conversions_match_torch(code, tdtype):
    g = torch.Generator().manual_seed(1)
    vals = torch.cat([torch.randn(100000, generator=g) * s for s in (1e-6, 1e-3, 1.0, 1e3, 1e5)])
    vals = torch.cat([vals, torch.tensor([0.0, -0.0, 65504.0, 65520.0, -65520.0, 1e-8, 6e-8,
                                          float("inf"), -float("inf")])])
    want = vals.to(tdtype).view(torch.int16).numpy().view(np.uint16)
    got = O.from_f32(code, vals.numpy())
    assert_bits_equal(got, want, code, label="from_f32")
    back = O.to_f32(code, want)
    assert np.array_equal(back, vals.to(tdtype).float().numpy(), equal_nan=True)


def test_relu_oracle_matches_torch_relu(relu_golden):
    """The fixtures are torch.relu on CPU.  The oracle follows torch.relu as it
    computes on CUDA, which differs from the CPU kernel only on -0.0 (CUDA: +0,
    CPU: -0) and on NaN payloads (the CPU kernel rewrites them; the oracle keeps
    the input bits).  Everything else is bit-exact."""
    from tests.numerics import is_nan

    for name, code in (("bf16", O.BF16), ("fp16", O.FP16)):
        x, want = relu_golden[name]
        x, want = x.reshape(-1), want.reshape(-1)
        got = O.relu(code, x)
        nan = is_nan(x, code)
        negzero = x == 0x8000
        assert negzero.any() and nan.any()
        keep = ~nan & ~negzero
        assert_bits_equal(got[keep], want[keep], code, label=name)
        assert (got[nan] == x[nan]).all()
        assert (got[negzero] == 0).all()


def test_eager_formula_is_the_reference_formula(rms_golden):
    c = rms_golden["bf16_rt_r5_h384"]
    t = lambda a: torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    out, res = O.eager_formula(t(c["x"]), t(c["r"]), t(c["w"]), c["eps"])
    assert (res.view(torch.int16).numpy().view(np.uint16) == c["res"]).all()
    assert (out.view(torch.int16).numpy().view(np.uint16) == c["out"]).all()


def test_ulp_helper():
    a = np.array([0x3F80, 0x8001, 0x0000], dtype=np.uint16)
    b = np.array([0x3F81, 0x0001, 0x8000], dtype=np.uint16)
    assert list(ulp_diff(a, b)) == [1, 2, 0]
