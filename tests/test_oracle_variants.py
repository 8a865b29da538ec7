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


def test_e2m1_conversion_table():
    """e2m1 (NVFP4 element): round to nearest even over {0, .5, 1, 1.5, 2, 3, 4, 6},
    saturating at 6; NaN -> +6 (code 7), the GPU conversion's rule."""
    vals = np.array([0.0, -0.0, 0.25, 0.2501, 0.75, 1.25, 1.7, 1.75, 2.5, 2.51, 3.5, 5.0, 5.01,
                     6.0, 7.0, 1e9, -0.3, -2.5, -100.0, np.nan], dtype=np.float32)
    want = [0x0, 0x8, 0x0, 0x1, 0x2, 0x2, 0x3, 0x4, 0x4, 0x5, 0x6, 0x6, 0x7,
            0x7, 0x7, 0x7, 0x9, 0xC, 0xF, 0x7]
    assert list(O.f32_to_e2m1(vals)) == want


@pytest.mark.parametrize("residual", [False, True])
def test_nvfp4_dequantises_within_half_a_step(residual):
    code = O.BF16
    x, w, r = _inputs(11, 4096, code, 5)
    gs = 448.0 * 6.0 / 8.0
    q, sf, res = O.rms_norm_nvfp4(code, x, w, 1e-6, gs, r=r if residual else None)
    y16, res16, _ = O.rms_norm_out(code, x, w, 1e-6, r=r if residual else None)
    if residual:
        assert (res == res16).all()
    mag = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6], dtype=np.float32)
    lo, hi = q & 0xF, q >> 4
    codes = np.stack([lo, hi], axis=-1).reshape(11, 4096)
    vals = np.where(codes & 8, -1.0, 1.0) * mag[codes & 7]
    sfv = torch.from_numpy(sf.view(np.int8)).view(torch.float8_e4m3fn).float().numpy()
    deq = vals.reshape(11, 256, 16) * (sfv / gs)[..., None]
    y = O.to_f32(code, y16).reshape(11, 256, 16)
    # half of the widest e2m1 step (4 -> 6) in each block's units, plus bf16 rounding of y
    bound = (sfv / gs)[..., None] * 1.0 + np.abs(y) * 2 ** -8
    assert np.all(np.abs(deq - y) <= bound)
    amax = np.abs(y).max(axis=-1)
    np.testing.assert_allclose(sfv, gs * amax / 6.0, rtol=2 ** -3)


@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_fp8_group_is_the_dynamic_scale_per_group(residual, group):
    """Per-token-group fp8: each group takes the per-row dynamic form's scale
    rule (max |y| / 448 with a 1e-12 floor, then e4m3 of y times the inverse
    scale) over its own elements, with the row's inverse RMS; y rebuilt here in
    numpy from the definition, e4m3 from the conversion pinned to torch."""
    x, w, r = _inputs(5, 512, O.BF16, 7)
    rr = r if residual else None
    q, sc, res = O.rms_norm_fp8_group(O.BF16, x, w, 1e-6, group=group, r=rr)
    assert q.shape == (5, 512) and sc.shape == (5, 512 // group)
    _, res16, _ = O.rms_norm_out(O.BF16, x, w, 1e-6, r=rr)
    if residual:
        assert_bits_equal(res, res16, O.BF16)
    sums = O.to_f32(O.BF16, x) + (O.to_f32(O.BF16, r) if residual else np.float32(0))
    inv = (1.0 / np.sqrt((sums.astype(np.float64) ** 2).sum(-1) / 512 + 1e-6)).astype(np.float32)
    v = O.to_f32(O.BF16, res16 if residual else x)
    y = (v * O.to_f32(O.BF16, w)) * inv[:, None]
    for g in range(512 // group):
        yg = y[:, g * group:(g + 1) * group]
        want_sc = np.maximum(np.abs(yg).max(-1), np.float32(1e-12)) / np.float32(448)
        np.testing.assert_array_equal(sc[:, g], want_sc)
        want_q = O.f32_to_e4m3(yg * (np.float32(1) / want_sc)[:, None])
        np.testing.assert_array_equal(q[:, g * group:(g + 1) * group], want_q)


def test_fp8_group_power_of_two_scales():
    x, w, r = _inputs(9, 1024, O.FP16, 8)
    _, sc, _ = O.rms_norm_fp8_group(O.FP16, x, w, 1e-6, group=128, r=r)
    q2, sc2, _ = O.rms_norm_fp8_group(O.FP16, x, w, 1e-6, group=128, pow2=True, r=r)
    m, e = np.frexp(sc2)
    assert (m == 0.5).all()  # exact powers of two
    assert (sc2 >= sc).all() and (sc2 < 2 * sc).all()  # the smallest one not below the scale
    # With a larger scale nothing saturates: every code is within the e4m3 range below 448.
    mag = q2 & 0x7F
    assert (mag != 0x7F).all() and int(mag.max()) <= 0x7E
