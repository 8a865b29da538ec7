"""The oracle's generalised row op (plain RMSNorm, out-of-place fused form,
fp8 e4m3 outputs), pinned against the fused oracle, torch.rms_norm and torch's
float8_e4m3fn conversion (CPU only)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.numerics import assert_bits_equal, assert_output_close


def _inputs(rows, hidden, code, seed):
    g = np.random.default_rng(seed)
    x = O.from_f32(code, g.standard_normal((rows, hidden)).astype(np.float32))
    r = O.from_f32(code, g.standard_normal((rows, hidden)).astype(np.float32))
    w = O.from_f32(code, (1 + 0.1 * g.standard_normal(hidden)).astype(np.float32))
    return x, w, r


@pytest.mark.parametrize("code", [O.BF16, O.FP16])
def test_fused_out_of_place_equals_in_place_oracle(code):
    x, w, r = _inputs(17, 1536, code, 1)
    want_out, want_res = O.fused_add_rms_norm(code, x, w, r, 1e-6)
    out, res, _ = O.rms_norm_out(code, x, w, 1e-6, r=r)
    assert_bits_equal(out, want_out, code)
    assert_bits_equal(res, want_res, code)


@pytest.mark.parametrize("code,tdt", [(O.BF16, torch.bfloat16), (O.FP16, torch.float16)])
def test_plain_rms_norm_matches_torch(code, tdt):
    x, w, _ = _inputs(33, 4096, code, 2)
    out, res, _ = O.rms_norm_out(code, x, w, 1e-5)
    assert res is None
    t = lambda a: torch.from_numpy(a.view(np.int16).copy()).view(tdt)
    want = torch.rms_norm(t(x), (4096,), t(w), 1e-5).view(torch.int16).numpy().view(np.uint16)
    assert_output_close(out, want, code, max_ulp=1)


def test_e4m3_conversion_matches_torch():
    g = torch.Generator().manual_seed(0)
    vals = torch.cat([torch.randn(100000, generator=g) * s for s in (1e-3, 0.1, 1, 30, 300, 3000)])
    vals = torch.cat([vals, torch.tensor([0.0, -0.0, 448.0, -448.0, 464.0, 2 ** -9, 2 ** -10,
                                          1.5 * 2 ** -9, float("inf"), -float("inf")])])
    got = O.f32_to_e4m3(vals.numpy())
    want = vals.clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(got, want)
    assert O.f32_to_e4m3(np.array([np.nan], dtype=np.float32))[0] == 0x7F


@pytest.mark.parametrize("residual", [False, True])
def test_fp8_static_is_the_16bit_path_quantised(residual):
    code = O.BF16
    x, w, r = _inputs(9, 2048, code, 3)
    out16, _, _ = O.rms_norm_out(code, x, w, 1e-6, r=r if residual else None)
    q, res, _ = O.rms_norm_out(code, x, w, 1e-6, r=r if residual else None, fp8="static", scale=0.05)
    y16 = O.to_f32(code, out16)
    # fp8 of y / scale; y here is fp32, out16 its bf16 rounding: within one e4m3 step.
    deq = torch.from_numpy(q.view(np.int8)).view(torch.float8_e4m3fn).float().numpy() * 0.05
    assert np.all(np.abs(deq - y16) <= np.abs(y16) * 2 ** -3 + 2 ** -9 * 0.05 + 1e-6)
    assert (res is not None) == residual


def test_fp8_dynamic_scales():
    code = O.FP16
    x, w, r = _inputs(12, 1024, code, 4)
    q, res, scales = O.rms_norm_out(code, x, w, 1e-6, r=r, fp8="dynamic")
    out16, _, _ = O.rms_norm_out(code, x, w, 1e-6, r=r)
    amax = np.abs(O.to_f32(code, out16)).max(axis=1)
    np.testing.assert_allclose(scales, amax / 448.0, rtol=2e-3)
    deq = torch.from_numpy(q.view(np.int8)).view(torch.float8_e4m3fn).float().numpy()
    assert np.abs(deq).max() <= 448.0
    assert (np.abs(deq).max(axis=1) >= 416.0).all()  # every row reaches the top of the range
