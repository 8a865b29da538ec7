"""GPU parity of the extended forms (plain RMSNorm, fused add + RMSNorm into a
separate output, fp8 e4m3 outputs with static or per-row scales), called
through the C ABI (hprn_rms_norm_out) and the torch ops, against the C oracle.

Bar: residual bit-exact; 16-bit outputs within 1 ulp and atol/rtol 1e-2;
fp8 outputs within one e4m3 step (the kernel's rsqrtf may differ from the
oracle's correctly rounded inverse RMS by an ulp, which can move a value
across an e4m3 rounding boundary); per-row scales within 1e-5 relative.
"""
import numpy as np
import pytest
import torch

import hp_rms_norm_b200
from hp_rms_norm_b200 import capi
from oracle import oracle as O
from tests.gpu_helpers import DTYPES, bits, edge_operands, from_bits, make_inputs
from tests.numerics import assert_bits_equal, assert_output_close

pytestmark = pytest.mark.gpu


def fp8_bits(t):
    return t.detach().contiguous().cpu().view(torch.uint8).numpy().copy()


def assert_fp8_close(got, want, label=""):
    got, want = got.reshape(-1).astype(np.int32), want.reshape(-1).astype(np.int32)
    gn, wn = (got & 0x7F) == 0x7F, (want & 0x7F) == 0x7F
    assert (gn == wn).all(), f"{label}: NaN positions differ"
    o = lambda b: np.where(b & 0x80, -(b & 0x7F), b & 0x7F)
    d = np.abs(o(got[~wn]) - o(want[~wn]))
    assert d.size == 0 or int(d.max()) <= 1, f"{label}: max e4m3 step difference {int(d.max())}"
    return float((d > 0).mean()) if d.size else 0.0


VARIANTS = ["plain16", "fused16", "plain_fp8s", "fused_fp8s", "plain_fp8d", "fused_fp8d"]
SHAPES = [(64, 1024), (33, 4096), (9, 16384), (5, 32768), (3, 65536), (128, 5120), (7, 2048)]


def run_variant(variant, x, w, r, eps, device):
    res = r if variant.startswith("fused") else None
    scale = row_scales = None
    if variant.endswith("16"):
        out = torch.empty_like(x)
    else:
        out = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=device)
        if variant.endswith("fp8s"):
            scale = torch.tensor([0.0123], dtype=torch.float32, device=device)
        else:
            row_scales = torch.zeros(x.shape[0], dtype=torch.float32, device=device)
    capi.rms_norm_out_tensors(out, x, w, res, eps, scale=scale, row_scales=row_scales)
    torch.cuda.synchronize()
    return out, scale, row_scales


def check_variant(variant, x, w, r, eps, code, device, label):
    xb, wb, rb = bits(x), bits(w), bits(r)
    fp8 = None if variant.endswith("16") else ("static" if variant.endswith("fp8s") else "dynamic")
    fused = variant.startswith("fused")
    want_out, want_res, want_scales = O.rms_norm_out(code, xb, wb, eps, r=rb if fused else None,
                                                     fp8=fp8, scale=0.0123)
    out, _, row_scales = run_variant(variant, x, w, r, eps, device)
    assert_bits_equal(bits(x), xb, code, label=label + " input unchanged")
    if fused:
        assert_bits_equal(bits(r), want_res, code, label=label + " residual")
    else:
        assert_bits_equal(bits(r), rb, code, label=label + " residual untouched")
    if fp8:
        frac = assert_fp8_close(fp8_bits(out), want_out, label)
        assert frac < 0.01, (label, frac)
        if fp8 == "dynamic":
            np.testing.assert_allclose(row_scales.cpu().numpy(), want_scales, rtol=1e-5)
    else:
        assert_output_close(bits(out), want_out, code, label=label)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("rows,hidden", SHAPES)
@pytest.mark.parametrize("variant", VARIANTS)
def test_variant_vs_oracle(cuda, variant, rows, hidden, dtype):
    tdtype, code = DTYPES[dtype]
    x, w, r, eps = make_inputs(rows, hidden, tdtype, "c2", seed=rows + hidden, device=cuda)
    check_variant(variant, x, w, r, eps, code, cuda, f"{variant} {dtype} {rows}x{hidden}")


FORCED = [
    (64, 1024, "warp:vec32:vpt2:tpr32:cluster1:rpc4"),
    (33, 512, "warp:vec32:vpt1:tpr32:cluster1:rpc8"),
    (17, 2048, "warp:vec32:vpt4:tpr32:cluster1:rpc1"),
    (67, 64, "warp:vec32:vpt1:tpr4:cluster1:rpc64"),
    (37, 256, "warp:vec32:vpt2:tpr8:cluster1:rpc32"),
    (11, 128, "warp:vec32:vpt4:tpr2:cluster1:rpc64"),
    (9, 4096, "cta:vec32:vpt2:tpr128:cluster1:rpc1"),
    (9, 8192, "cta:vec32:vpt4:tpr128:cluster1:rpc1"),
    (9, 8192, "cta:vec16:vpt4:tpr256:cluster1:rpc1"),
    (9, 8192, "cta:vec8:vpt4:tpr512:cluster1:rpc1"),
    (5, 16384, "cluster:vec32:vpt1:tpr512:cluster2:rpc1"),
    (3, 24576, "cluster:vec32:vpt1:tpr768:cluster2:rpc1"),
    (5, 16384, "cluster:vec32:vpt2:tpr256:cluster2:rpc1"),
    (5, 16384, "cluster:vec32:vpt4:tpr64:cluster4:rpc1"),
    (3, 32768, "cluster:vec32:vpt2:tpr128:cluster8:rpc1"),
]


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("rows,hidden,plan", FORCED)
def test_variant_every_plan_kind(cuda, variant, rows, hidden, plan):
    x, w, r, eps = make_inputs(rows, hidden, torch.bfloat16, "c0", seed=hidden + rows, device=cuda)
    capi.set_plan_override(plan)
    try:
        check_variant(variant, x, w, r, eps, O.BF16, cuda, f"{variant} {plan}")
    finally:
        capi.set_plan_override(None)


@pytest.mark.parametrize("knobs", [f"default:pf{pf}:et{et}" for pf in (0, 1, 2, 3) for et in (0, 1, 2)])
@pytest.mark.parametrize("rows,hidden", [(600, 4096), (300, 32768)])
@pytest.mark.parametrize("variant", VARIANTS)
def test_variant_launch_knobs_keep_results(cuda, variant, rows, hidden, knobs):
    """Every pair of launch knobs (L2 prefetch scope, trigger point) gives the
    default launch's bits for every form, on grids of more than one wave."""
    x, w, r, eps = make_inputs(rows, hidden, torch.bfloat16, "c0", seed=hidden + 3, device=cuda)
    r1, r2 = r.clone(), r.clone()
    want = run_variant(variant, x, w, r1, eps, cuda)
    capi.set_plan_override(knobs)
    try:
        got = run_variant(variant, x, w, r2, eps, cuda)
    finally:
        capi.set_plan_override(None)
    assert torch.equal(r1.view(torch.int16), r2.view(torch.int16))
    for a, b in zip(want, got):
        if a is not None:
            assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("variant", VARIANTS)
def test_edge_operands_vs_oracle(cuda, variant, dtype):
    """Products and squares of 16-bit operands are exact in fp32 and must not
    flush subnormal operands or lose a zero's sign: subnormal inputs and
    weights, signed zeros and the largest finite values against the oracle.
    eps is tiny so that the subnormal rows' own sums of squares set their
    scale."""
    tdtype, code = DTYPES[dtype]
    hidden = 4096
    x, w_plain, w_edge = edge_operands(code, hidden, 7 + code)
    for wname, wb in (("weight", w_plain), ("edge weight", w_edge)):
        xt = from_bits(x, tdtype, cuda)
        wt = from_bits(wb, tdtype, cuda)
        rt = from_bits(x[::-1].copy(), tdtype, cuda)
        check_variant(variant, xt, wt, rt, 1e-30, code, cuda, f"{variant} {dtype} {wname}")
        if variant == "plain16":
            # The signed-zero row: y = (x * w) * inv is a zero whose sign is
            # sign(x) xor sign(w), bit for bit.
            want_out, _, _ = O.rms_norm_out(code, x, wb, 1e-30)
            out, _, _ = run_variant(variant, xt, wt, rt, 1e-30, cuda)
            assert np.array_equal(bits(out)[1], want_out[1]), f"{dtype} {wname}: signed zeros"


def nonfinite_rows(code, hidden, seed, weight_special=None):
    """Rows of ordinary values with NaN, +inf and -inf planted, and a clean
    row; with weight_special "nan" or "inf", two weight entries are that
    value, so the clean row's products hold it while its sum of squares stays
    finite (the amaxes must ignore NaN as fmaxf does)."""
    g = np.random.default_rng(seed)
    one, inf, nan = (0x3C00, 0x7C00, 0x7E00) if code == O.FP16 else (0x3F80, 0x7F80, 0x7FC0)
    x = (g.integers(one - 0x400 if code == O.FP16 else one - 0x80, one + 0x200, (4, hidden))
         .astype(np.uint16) | (g.integers(0, 2, (4, hidden)) << 15).astype(np.uint16))
    x[0, 17] = nan
    x[1, 100] = inf
    x[2, 5] = inf | 0x8000
    x[2, 3000] = nan
    r = (g.integers(one - 0x400 if code == O.FP16 else one - 0x80, one, (4, hidden))
         .astype(np.uint16))
    w = g.integers(one - 0x100 if code == O.FP16 else one - 0x20, one + 0x100 if code == O.FP16
                   else one + 0x20, hidden).astype(np.uint16)
    if weight_special:
        w[[7, 2000]] = nan if weight_special == "nan" else inf
    return x, r, w


@pytest.mark.parametrize("weight_special", [None, "nan", "inf"])
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("variant", VARIANTS)
def test_nonfinite_vs_oracle(cuda, variant, dtype, weight_special):
    """NaN and infinities inside rows and in the weight: NaN positions,
    infinities and every finite result as the oracle has them (per-row fp8
    scales included)."""
    tdtype, code = DTYPES[dtype]
    x, r, w = nonfinite_rows(code, 4096, 3 + code, weight_special)
    xt, rt, wt = (from_bits(a, tdtype, cuda) for a in (x, r, w))
    check_variant(variant, xt, wt, rt, 1e-6, code, cuda, f"{variant} {dtype} non-finite")


@pytest.mark.parametrize("hidden", [3, 7, 129, 4097])
def test_plain_odd_hidden(cuda, hidden):
    x, w, r, eps = make_inputs(6, hidden, torch.float16, "c0", seed=hidden, device=cuda)
    check_variant("plain16", x, w, r, eps, O.FP16, cuda, f"plain odd {hidden}")
    check_variant("fused16", x, w, r, eps, O.FP16, cuda, f"fused odd {hidden}")


def test_plain_in_place_and_torch_api(cuda):
    x, w, r, eps = make_inputs(96, 6144, torch.bfloat16, "c0", seed=5, device=cuda)
    want = hp_rms_norm_b200.rms_norm(x, w, eps)
    y = x.clone()
    got = hp_rms_norm_b200.rms_norm(y, w, eps, out=y)
    torch.cuda.synchronize()
    assert got is y and torch.equal(y.view(torch.int16), want.view(torch.int16))
    # 3-D input through the torch op equals the 2-D C-ABI call.
    x3 = x.view(4, 24, 6144)
    out3 = hp_rms_norm_b200.rms_norm(x3, w, eps)
    assert torch.equal(out3.view(-1, 6144).view(torch.int16), want.view(torch.int16))


def test_fused_out_of_place_torch_api_matches_in_place(cuda):
    x, w, r, eps = make_inputs(64, 8192, torch.bfloat16, "c0", seed=6, device=cuda)
    x1, r1 = x.clone(), r.clone()
    hp_rms_norm_b200.hp_rms_norm(x1, w, r1, eps)
    r2 = r.clone()
    out = hp_rms_norm_b200.fused_add_rms_norm(x, r2, w, eps)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), x1.view(torch.int16))
    assert torch.equal(r2.view(torch.int16), r1.view(torch.int16))


@pytest.mark.parametrize("residual", [False, True])
def test_fp8_torch_api(cuda, residual):
    x, w, r, eps = make_inputs(48, 4096, torch.float16, "c2", seed=8, device=cuda)
    r_api, r_capi = r.clone(), r.clone()
    q, scales = hp_rms_norm_b200.rms_norm_fp8(x.view(6, 8, 4096), w, eps,
                                              residual=r_api.view(6, 8, 4096) if residual else None)
    assert q.shape == (6, 8, 4096) and q.dtype == torch.float8_e4m3fn and scales.shape == (6, 8)
    out = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=cuda)
    rs = torch.empty(48, dtype=torch.float32, device=cuda)
    capi.rms_norm_out_tensors(out, x, w, r_capi if residual else None, eps, row_scales=rs)
    torch.cuda.synchronize()
    assert torch.equal(q.view(-1, 4096).view(torch.uint8), out.view(torch.uint8))
    assert torch.equal(scales.view(-1), rs)
    s = torch.tensor([0.02], device=cuda)
    q2, s2 = hp_rms_norm_b200.rms_norm_fp8(x, w, eps, scale=s)
    assert s2 is s and q2.dtype == torch.float8_e4m3fn


def test_variant_argument_errors(cuda):
    x, w, r, eps = make_inputs(4, 4098, torch.bfloat16, "c0", seed=1, device=cuda)
    out = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=cuda)
    with pytest.raises(capi.HprnError, match="fp8 output needs hidden_dim % 4"):
        capi.rms_norm_out_tensors(out, x, w, r, eps, row_scales=torch.zeros(4, device=cuda))
    with pytest.raises(capi.HprnError, match="needs a scale"):
        capi.rms_norm_out(out.data_ptr(), x.data_ptr(), w.data_ptr(), r.data_ptr(), 4, 4098, 4098,
                          4098, 4098, eps, capi.DTYPE_BF16, capi.OUT_FP8_E4M3_STATIC)
    big = torch.zeros(2, 1 << 19, dtype=torch.bfloat16, device=cuda)
    wb = torch.ones(1 << 19, dtype=torch.bfloat16, device=cuda)
    ob = torch.empty(big.shape, dtype=torch.float8_e4m3fn, device=cuda)
    with pytest.raises(capi.HprnError, match="16-bit output only"):
        capi.rms_norm_out_tensors(ob, big, wb, None, eps, scale=torch.ones(1, device=cuda))
    with pytest.raises(RuntimeError, match="exactly one of scale"):
        torch.ops.hp_rms_norm.rms_norm_fp8(out, x, w, None, eps, None, None)
    with pytest.raises(capi.HprnError, match="output must be the input itself or not overlap"):
        capi.rms_norm_out(x.data_ptr() + 2, x.data_ptr(), w.data_ptr(), None, 4, 4098, 4098, 4098,
                          4098, eps, capi.DTYPE_BF16)
