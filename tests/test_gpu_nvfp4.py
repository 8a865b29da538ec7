"""GPU parity of the NVFP4-output form (e2m1 codes + one e4m3 scale per 16
elements + a per-tensor global scale) through the C ABI and the torch op,
against the C oracle.  The kernel's rsqrtf may differ from the oracle's
correctly rounded inverse RMS by an ulp, which can move a block's scale or an
element across a rounding boundary: scale codes and element codes must agree
to within one step, and exactly in at least 99% of cases."""
import numpy as np
import pytest
import torch

import hp_rms_norm_b200
from hp_rms_norm_b200 import capi
from oracle import oracle as O
from tests.gpu_helpers import DTYPES, bits, edge_operands, from_bits, make_inputs
from tests.numerics import assert_bits_equal

pytestmark = pytest.mark.gpu

GS = 448.0 * 6.0 / 8.0


def e2m1_ordered(codes):
    c = codes.astype(np.int32)
    return np.where(c & 8, -(c & 7), c & 7)


def check_nvfp4(q, sf, want_q, want_sf, label):
    sf, want_sf = sf.astype(np.int32), want_sf.astype(np.int32)
    assert int(np.abs(sf - want_sf).max()) <= 1, label + " block scale"
    assert (sf == want_sf).mean() >= 0.99, label + " block scale exactness"
    rows = q.shape[0]
    unpack = lambda b: np.stack([b & 0xF, b >> 4], axis=-1).reshape(rows, -1)
    g, w = unpack(q), unpack(want_q)
    same = np.repeat(sf == want_sf, 16, axis=1)
    d = np.abs(e2m1_ordered(g) - e2m1_ordered(w))[same]
    assert d.size == 0 or int(d.max()) <= 1, label + " e2m1 codes"
    assert d.size == 0 or (d == 0).mean() >= 0.99, label + " e2m1 exactness"


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("rows,hidden", [(64, 4096), (33, 16384), (7, 32768), (5, 65536),
                                         (128, 2048), (1, 1024), (300, 7168)])
def test_nvfp4_vs_oracle(cuda, rows, hidden, residual, dtype):
    tdtype, code = DTYPES[dtype]
    x, w, r, eps = make_inputs(rows, hidden, tdtype, "c0", seed=rows * 3 + hidden, device=cuda)
    xb, wb, rb = bits(x), bits(w), bits(r)
    want_q, want_sf, want_res = O.rms_norm_nvfp4(code, xb, wb, eps, GS, r=rb if residual else None)
    q = torch.empty(rows, hidden // 2, dtype=torch.uint8, device=cuda)
    sf = torch.empty(rows, hidden // 16, dtype=torch.uint8, device=cuda)
    gs = torch.tensor([GS], device=cuda)
    capi.rms_norm_nvfp4_tensors(q, sf, x, w, r if residual else None, eps, gs)
    torch.cuda.synchronize()
    label = f"{dtype} {rows}x{hidden} residual={residual}"
    assert_bits_equal(bits(x), xb, code, label=label + " input unchanged")
    if residual:
        assert_bits_equal(bits(r), want_res, code, label=label + " residual")
    check_nvfp4(q.cpu().numpy(), sf.cpu().numpy(), want_q, want_sf, label)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("residual", [False, True])
def test_nvfp4_edge_operands_vs_oracle(cuda, residual, dtype):
    """Subnormal inputs and weights, signed zeros and large values (the
    products r * w are formed without unpacking the 16-bit operands)."""
    tdtype, code = DTYPES[dtype]
    x, w_plain, w_edge = edge_operands(code, 4096, 11 + code)
    for wname, wb in (("weight", w_plain), ("edge weight", w_edge)):
        rb = x[::-1].copy()
        xt, wt, rt = (from_bits(a, tdtype, cuda) for a in (x, wb, rb))
        want_q, want_sf, want_res = O.rms_norm_nvfp4(code, x, wb, 1e-30, GS,
                                                     r=rb if residual else None)
        q = torch.empty(5, 2048, dtype=torch.uint8, device=cuda)
        sf = torch.empty(5, 256, dtype=torch.uint8, device=cuda)
        capi.rms_norm_nvfp4_tensors(q, sf, xt, wt, rt if residual else None, 1e-30,
                                    torch.tensor([GS], device=cuda))
        torch.cuda.synchronize()
        label = f"{dtype} {wname} residual={residual}"
        if residual:
            assert_bits_equal(bits(rt), want_res, code, label=label + " residual")
        check_nvfp4(q.cpu().numpy(), sf.cpu().numpy(), want_q, want_sf, label)


@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("rows,hidden,plan", [
    (9, 4096, "cta:vec32:vpt2:tpr128:cluster1:rpc1"),
    (9, 8192, "cta:vec32:vpt4:tpr128:cluster1:rpc1"),
    (5, 24576, "cluster:vec32:vpt1:tpr768:cluster2:rpc1"),
    (5, 32768, "cluster:vec32:vpt4:tpr128:cluster4:rpc1"),
    (33, 1024, "warp:vec32:vpt2:tpr32:cluster1:rpc4"),
])
def test_nvfp4_forced_plans_vs_oracle(cuda, rows, hidden, plan, residual):
    """Kernel kinds and vectors-per-thread the heuristic may not pick."""
    x, w, r, eps = make_inputs(rows, hidden, torch.bfloat16, "c0", seed=hidden + rows, device=cuda)
    xb, wb, rb = bits(x), bits(w), bits(r)
    want_q, want_sf, want_res = O.rms_norm_nvfp4(O.BF16, xb, wb, eps, GS, r=rb if residual else None)
    q = torch.empty(rows, hidden // 2, dtype=torch.uint8, device=cuda)
    sf = torch.empty(rows, hidden // 16, dtype=torch.uint8, device=cuda)
    capi.set_plan_override(plan)
    try:
        capi.rms_norm_nvfp4_tensors(q, sf, x, w, r if residual else None, eps,
                                    torch.tensor([GS], device=cuda))
        torch.cuda.synchronize()
    finally:
        capi.set_plan_override(None)
    if residual:
        assert_bits_equal(bits(r), want_res, O.BF16, label=plan + " residual")
    check_nvfp4(q.cpu().numpy(), sf.cpu().numpy(), want_q, want_sf, plan)


def test_nvfp4_torch_op_matches_capi(cuda):
    x, w, r, eps = make_inputs(96, 8192, torch.bfloat16, "c2", seed=4, device=cuda)
    gs = torch.tensor([GS], device=cuda)
    r1, r2 = r.clone(), r.clone()
    codes, scales = hp_rms_norm_b200.rms_norm_nvfp4(x.view(8, 12, 8192), w, eps, gs,
                                                    residual=r1.view(8, 12, 8192))
    assert codes.shape == (8, 12, 4096) and scales.shape == (8, 12, 512)
    assert scales.dtype == torch.float8_e4m3fn
    q = torch.empty(96, 4096, dtype=torch.uint8, device=cuda)
    sf = torch.empty(96, 512, dtype=torch.uint8, device=cuda)
    capi.rms_norm_nvfp4_tensors(q, sf, x, w, r2, eps, gs)
    torch.cuda.synchronize()
    assert torch.equal(codes.view(96, 4096), q)
    assert torch.equal(scales.view(96, 512).view(torch.uint8), sf)
    assert torch.equal(r1.view(torch.int16), r2.view(torch.int16))


def test_nvfp4_argument_errors(cuda):
    x, w, r, eps = make_inputs(4, 1032, torch.bfloat16, "c0", seed=1, device=cuda)
    gs = torch.tensor([GS], device=cuda)
    with pytest.raises(RuntimeError, match="hidden_dim % 16"):
        hp_rms_norm_b200.rms_norm_nvfp4(x, w, eps, gs)
    x2 = torch.empty(4 * 1024 + 8, dtype=torch.bfloat16, device=cuda)[8:].view(4, 1024)
    w2 = torch.ones(1024, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError, match="32-byte aligned"):
        hp_rms_norm_b200.rms_norm_nvfp4(x2, w2, eps, gs)


def test_nvfp4_empty_rows_are_a_no_op(cuda):
    """[N, 0] and [0, H] inputs return empty outputs without a launch, as the
    other out-of-place forms do."""
    gs = torch.tensor([GS], device=cuda)
    for rows, hidden in ((4, 0), (0, 64)):
        x = torch.empty(rows, hidden, dtype=torch.bfloat16, device=cuda)
        w = torch.ones(hidden, dtype=torch.bfloat16, device=cuda)
        r = torch.empty_like(x)
        codes, scales = hp_rms_norm_b200.rms_norm_nvfp4(x, w, 1e-6, gs, residual=r)
        torch.cuda.synchronize()
        assert codes.shape == (rows, hidden // 2) and scales.shape == (rows, hidden // 16)
