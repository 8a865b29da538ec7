"""Per-token-group fp8 output (hprn_rms_norm_fp8_group / rms_norm_fp8_group)
against the C oracle: residual bit-exact, e4m3 codes within one code, group
scales within rtol 1e-5 (the kernel's inverse RMS is fp32 rsqrt, the oracle's
double), power-of-two scales equal except where the exact scale sits within
1e-5 of a power of two.  Every kernel kind (warp, CTA, cluster with row slices
rounded to whole groups), group sizes 32/64/128, column-major scale views,
strided rows, and the argument errors."""
import numpy as np
import pytest
import torch

import hp_rms_norm_b200 as H
from hp_rms_norm_b200 import capi
from oracle import oracle as O
from tests.gpu_helpers import DTYPES, bits, edge_operands, from_bits
from tests.numerics import assert_bits_equal

pytestmark = pytest.mark.gpu


def _inputs(rows, hidden, tdt, seed, device):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, hidden, generator=g).to(tdt)
    r = torch.randn(rows, hidden, generator=g).to(tdt)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(tdt)
    return x.to(device), w.to(device), r.to(device)


def _code_dist(got, want):
    o = lambda b: np.where(b & 0x80, -(b & 0x7F), b & 0x7F).astype(np.int32)
    return np.abs(o(got.astype(np.int32)) - o(want.astype(np.int32)))


def check(x, w, r, eps, code, group, pow2, label, run):
    """Runs `run(out, scales)` (which must launch the op on x, w, r) and
    compares with the oracle."""
    xb, wb, rb = bits(x), bits(w), bits(r) if r is not None else None
    want_q, want_sc, want_res = O.rms_norm_fp8_group(code, xb, wb, eps, group, pow2, r=rb)
    _, exact_sc, _ = O.rms_norm_fp8_group(code, xb, wb, eps, group, False, r=rb)
    rows, hidden = x.shape
    out = torch.full((rows, hidden), 0x55, dtype=torch.uint8, device=x.device).view(torch.float8_e4m3fn)
    scales = torch.full((rows, hidden // group), -1.0, device=x.device)
    run(out, scales)
    torch.cuda.synchronize()
    got_q = out.view(torch.uint8).cpu().numpy()
    got_sc = scales.cpu().numpy()
    if r is not None:
        assert_bits_equal(bits(r), want_res, code, label=label + " residual")
    assert_bits_equal(bits(x), xb, code, label=label + " input unchanged")
    if pow2:
        m, _ = np.frexp(got_sc)
        assert (m == 0.5).all(), label + ": scales not powers of two"
        mm, _ = np.frexp(exact_sc)  # mantissa in [0.5, 1): near a power of two at either end
        near = (mm - 0.5 < 1e-5) | (1.0 - mm < 1e-5)
        same = got_sc == want_sc
        assert (same | near).all(), f"{label}: {int((~same & ~near).sum())} scales differ"
    else:
        np.testing.assert_allclose(got_sc, want_sc, rtol=1e-5, err_msg=label)
        same = np.ones_like(got_sc, dtype=bool)
    codes_checked = np.repeat(same, group, axis=1)
    d = _code_dist(got_q, want_q)[codes_checked]
    assert d.size and int(d.max()) <= 1, f"{label}: code distance {int(d.max())}"


def run_capi(x, w, r, eps, group, pow2):
    return lambda out, sc: capi.rms_norm_fp8_group_tensors(out, sc, x, w, r, eps, group, pow2)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("residual", [True, False])
@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("pow2", [False, True])
@pytest.mark.parametrize("rows,hidden", [(37, 1024), (19, 4096), (5, 33024), (3, 40960)])
def test_default_plans_vs_oracle(cuda, dtype, residual, group, pow2, rows, hidden):
    tdt, code = DTYPES[dtype]
    x, w, r = _inputs(rows, hidden, tdt, hidden + group, cuda)
    rr = r if residual else None
    check(x, w, rr, 1e-6, code, group, pow2, f"{dtype} {rows}x{hidden} g{group} res={residual}",
          run_capi(x, w, rr, 1e-6, group, pow2))


# Forced plans: every kernel kind and vectors-per-thread compiled for the
# quantised forms, clusters whose even row split is not a whole number of
# groups (slices rounded up; trailing CTAs of a cluster may get no vectors).
FORCED = [
    (33, 1024, "warp:vec32:vpt2:tpr32:cluster1:rpc8"),
    (33, 2048, "warp:vec32:vpt4:tpr32:cluster1:rpc4"),
    (9, 512, "warp:vec32:vpt1:tpr32:cluster1:rpc2"),
    (9, 4096, "cta:vec32:vpt1:tpr256:cluster1:rpc1"),
    (9, 4096, "cta:vec32:vpt2:tpr128:cluster1:rpc1"),
    (9, 4096, "cta:vec32:vpt4:tpr64:cluster1:rpc1"),
    (5, 16384, "cluster:vec32:vpt1:tpr512:cluster2:rpc1"),
    (5, 24576, "cluster:vec32:vpt1:tpr768:cluster2:rpc1"),
    (5, 4096, "cluster:vec32:vpt2:tpr32:cluster8:rpc1"),
    (5, 4096, "cluster:vec32:vpt4:tpr32:cluster4:rpc1"),
    (5, 1152, "cluster:vec32:vpt2:tpr32:cluster8:rpc1"),
    (5, 33024, "cluster:vec32:vpt2:tpr160:cluster8:rpc1"),
    (5, 33024, "cluster:vec32:vpt4:tpr160:cluster4:rpc1"),
]


@pytest.mark.parametrize("residual", [True, False])
@pytest.mark.parametrize("rows,hidden,plan", FORCED)
def test_forced_plans_vs_oracle(cuda, residual, rows, hidden, plan):
    x, w, r = _inputs(rows, hidden, torch.bfloat16, len(plan) + hidden, cuda)
    rr = r if residual else None
    capi.set_plan_override(plan)
    try:
        check(x, w, rr, 1e-6, O.BF16, 128, False, plan, run_capi(x, w, rr, 1e-6, 128, False))
    finally:
        capi.set_plan_override(None)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("residual", [True, False])
@pytest.mark.parametrize("group", [32, 128])
def test_edge_operands_vs_oracle(cuda, dtype, residual, group):
    """Subnormal inputs and weights, signed zeros and large values (the
    products r * w are formed without unpacking the 16-bit operands)."""
    tdtype, code = DTYPES[dtype]
    x, w_plain, w_edge = edge_operands(code, 4096, 13 + code)
    for wname, wb in (("weight", w_plain), ("edge weight", w_edge)):
        xt, wt = from_bits(x, tdtype, cuda), from_bits(wb, tdtype, cuda)
        rt = from_bits(x[::-1].copy(), tdtype, cuda) if residual else None
        check(xt, wt, rt, 1e-30, code, group, False, f"{dtype} {wname} g{group} res={residual}",
              run_capi(xt, wt, rt, 1e-30, group, False))


@pytest.mark.parametrize("weight_special", [None, "nan", "inf"])
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("residual", [True, False])
def test_nonfinite_vs_oracle(cuda, dtype, residual, weight_special):
    """NaN and infinities inside groups and in the weight (group amaxes
    ignore NaN as fmaxf does)."""
    from tests.test_gpu_rms_norm_variants import nonfinite_rows

    tdtype, code = DTYPES[dtype]
    x, r, w = nonfinite_rows(code, 4096, 5 + code, weight_special)
    xt, rt, wt = (from_bits(a, tdtype, cuda) for a in (x, r, w))
    rr = rt if residual else None
    check(xt, wt, rr, 1e-6, code, 128, False, f"{dtype} non-finite res={residual}",
          run_capi(xt, wt, rr, 1e-6, 128, False))


def test_torch_op_column_major_scales_and_3d(cuda):
    x, w, r = _inputs(6 * 7, 2048, torch.bfloat16, 5, cuda)
    x3, r3 = x.view(6, 7, 2048), r.clone().view(6, 7, 2048)
    q_row, s_row = H.rms_norm_fp8_group(x3, w, 1e-5, residual=r3, group_size=64)
    r3b = r.clone().view(6, 7, 2048)
    q_col, s_col = H.rms_norm_fp8_group(x3, w, 1e-5, residual=r3b, group_size=64,
                                        column_major_scales=True)
    assert s_col.stride() == (1, 42)
    assert torch.equal(q_row.view(torch.uint8), q_col.view(torch.uint8))
    assert torch.equal(s_row, s_col)
    assert torch.equal(r3.view(torch.int16), r3b.view(torch.int16))
    want_q, want_sc, want_res = O.rms_norm_fp8_group(O.BF16, bits(x), bits(w), 1e-5, 64, r=bits(r))
    np.testing.assert_allclose(s_row.cpu().numpy(), want_sc, rtol=1e-5)
    assert int(_code_dist(q_row.view(torch.uint8).reshape(42, 2048).cpu().numpy(), want_q).max()) <= 1
    assert_bits_equal(bits(r3), want_res, O.BF16, label="residual")


def test_strided_rows(cuda):
    rows, hidden = 23, 4096
    x0, w, r0 = _inputs(rows, hidden, torch.float16, 6, cuda)
    xb = torch.zeros(rows, hidden + 64, dtype=torch.float16, device=cuda)
    rb = torch.zeros(rows, hidden + 16, dtype=torch.float16, device=cuda)
    x, r = xb[:, 16:16 + hidden], rb[:, :hidden]
    x.copy_(x0)
    r.copy_(r0)
    ob = torch.full((rows, hidden + 48), 0x55, dtype=torch.uint8, device=cuda)
    out = ob[:, :hidden].view(torch.float8_e4m3fn)
    sb = torch.full((rows, 64), -1.0, device=cuda)
    sc = sb[:, :hidden // 128]
    capi.rms_norm_fp8_group_tensors(out, sc, x, w, r, 1e-6, 128, False)
    torch.cuda.synchronize()
    want_q, want_sc, want_res = O.rms_norm_fp8_group(O.FP16, bits(x0), bits(w), 1e-6, 128, r=bits(r0))
    assert int(_code_dist(out.view(torch.uint8).cpu().numpy(), want_q).max()) <= 1
    np.testing.assert_allclose(sc.cpu().numpy(), want_sc, rtol=1e-5)
    assert_bits_equal(bits(r), want_res, O.FP16, label="residual")
    assert int((ob[:, hidden:] == 0x55).sum()) == rows * 48  # output padding untouched
    assert bool((sb[:, hidden // 128:] == -1.0).all())  # scale padding untouched


def test_argument_errors(cuda):
    x, w, r = _inputs(4, 1024, torch.bfloat16, 7, cuda)
    out = torch.empty(4, 1024, dtype=torch.float8_e4m3fn, device=cuda)
    sc = torch.empty(4, 8, device=cuda)
    with pytest.raises(capi.HprnError, match="group_size"):
        capi.rms_norm_fp8_group_tensors(out, sc, x, w, r, 1e-6, 48, False)
    with pytest.raises(capi.HprnError, match="multiple of group_size"):
        capi.rms_norm_fp8_group_tensors(out[:, :1000], sc, x[:, :1000], w[:1000], r[:, :1000], 1e-6, 128, False)
    with pytest.raises(capi.HprnError, match="scales buffer"):
        capi.rms_norm_fp8_group(out.data_ptr(), None, 8, 1, x.data_ptr(), w.data_ptr(), None, 4, 1024,
                                1024, 1024, 1024, 1e-6, capi.DTYPE_BF16)
    xm = torch.empty(4 * 1024 + 8, dtype=torch.bfloat16, device=cuda)[8:].view(4, 1024)
    with pytest.raises(capi.HprnError, match="32-byte aligned"):
        capi.rms_norm_fp8_group_tensors(out, sc, xm, w, None, 1e-6, 128, False)
    with pytest.raises(capi.HprnError, match="hprn_rms_norm_fp8_group"):
        capi.rms_norm_out(out.data_ptr(), x.data_ptr(), w.data_ptr(), None, 4, 1024, 1024, 1024,
                          1024, 1e-6, capi.DTYPE_BF16, capi.OUT_FP8_E4M3_GROUP, None, sc.data_ptr())
    with pytest.raises(RuntimeError, match="scales must be float32"):
        torch.ops.hp_rms_norm.rms_norm_fp8_group(out, torch.empty(4, 7, device=cuda), x, w, None,
                                                 1e-6, 128, False)
