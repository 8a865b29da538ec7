"""The TMA-staged row kernel (plan kind `tma`: rows brought into shared memory
by cp.async.bulk with mbarrier completion, a persistent grid walking the rows)
against the C oracle: the fused in-place form, the out-of-place and plain
forms, ring depths from 1 to 16, rows far beyond one pass of the grid, partial
last vectors per thread, strided rows with canaries, PDL chains and CUDA
graphs.  Every case ends with no CTA having given up a bounded wait."""
import numpy as np
import pytest
import torch

from hp_rms_norm_b200 import capi
from oracle import oracle as O
from tests.gpu_helpers import DTYPES, bits, make_inputs
from tests.numerics import assert_bits_equal, assert_output_close

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def no_wait_timeouts(cuda):
    capi.wait_timeouts(reset=True)
    yield
    torch.cuda.synchronize()
    assert capi.wait_timeouts(reset=True) == 0, "a CTA gave up waiting for a bulk copy"


def forced(plan):
    class _Ctx:
        def __enter__(self):
            capi.set_plan_override(plan)

        def __exit__(self, *exc):
            capi.set_plan_override(None)
    return _Ctx()


# (rows, hidden, plan): vectors per thread 1/2/4/8, thread counts that leave
# the last vectors of a row uncovered by some threads, ring depths 1..16, row
# counts below, near and far above the number of resident CTAs.
TMA_PLANS = [
    (3, 1024, "tma:vec16:vpt1:tpr128:cluster1:rpc4"),
    (4096, 1024, "tma:vec16:vpt1:tpr128:cluster1:rpc8"),
    (9000, 1024, "tma:vec16:vpt2:tpr64:cluster1:rpc2"),
    (2000, 2048, "tma:vec16:vpt1:tpr256:cluster1:rpc1"),
    (2000, 2048, "tma:vec16:vpt2:tpr128:cluster1:rpc16"),
    (777, 4096, "tma:vec16:vpt4:tpr128:cluster1:rpc3"),
    (777, 4096, "tma:vec16:vpt8:tpr64:cluster1:rpc6"),
    (300, 8192, "tma:vec16:vpt2:tpr512:cluster1:rpc2"),
    (300, 8192, "tma:vec16:vpt1:tpr1024:cluster1:rpc1"),
    (129, 16384, "tma:vec16:vpt8:tpr256:cluster1:rpc3"),
    (511, 1000, "tma:vec16:vpt1:tpr128:cluster1:rpc5"),
    (257, 5000, "tma:vec16:vpt4:tpr160:cluster1:rpc2"),
    (64, 8, "tma:vec16:vpt1:tpr32:cluster1:rpc2"),
    (4096, 1024, "tma:vec32:vpt1:tpr64:cluster1:rpc4"),
    (1031, 4096, "tma:vec32:vpt2:tpr128:cluster1:rpc2"),
    (300, 8192, "tma:vec32:vpt1:tpr512:cluster1:rpc3"),
    (65, 16384, "tma:vec32:vpt4:tpr256:cluster1:rpc2"),
    (100, 4112, "tma:vec32:vpt8:tpr64:cluster1:rpc1"),
]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("rows,hidden,plan", TMA_PLANS)
def test_tma_fused_in_place(cuda, dtype, rows, hidden, plan):
    tdtype, code = DTYPES[dtype]
    x, w, r, eps = make_inputs(rows, hidden, tdtype, "c0", seed=rows + hidden, device=cuda)
    xb, wb, rb = bits(x), bits(w), bits(r)
    want_out, want_res = O.fused_add_rms_norm(code, xb, wb, rb, eps, O.SS_UNROUNDED)
    with forced(plan):
        capi.rms_norm_tensors(x, w, r, eps)
    torch.cuda.synchronize()
    assert_bits_equal(bits(r), want_res, code, label=plan + " residual")
    assert_output_close(bits(x), want_out, code, label=plan + " output")


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("rows,hidden,plan", [
    (1500, 1024, "tma:vec16:vpt1:tpr128:cluster1:rpc8"),
    (333, 4096, "tma:vec16:vpt2:tpr256:cluster1:rpc4"),
    (65, 12288, "tma:vec16:vpt8:tpr192:cluster1:rpc2"),
])
def test_tma_out_of_place_and_plain(cuda, fused, rows, hidden, plan):
    x, w, r, eps = make_inputs(rows, hidden, torch.bfloat16, "c2", seed=hidden, device=cuda)
    out = torch.full_like(x, 7.0)
    xb, wb, rb = bits(x), bits(w), bits(r)
    with forced(plan):
        capi.rms_norm_out_tensors(out, x, w, r if fused else None, eps)
    torch.cuda.synchronize()
    want_out, want_res, _ = O.rms_norm_out(O.BF16, xb, wb, eps, r=rb if fused else None)
    assert_bits_equal(bits(x), xb, O.BF16, label="input unchanged")
    if fused:
        assert_bits_equal(bits(r), want_res, O.BF16, label="residual")
    assert_output_close(bits(out), want_out, O.BF16, label=plan)


def test_tma_strided_rows_keep_canaries(cuda):
    rows, hidden = 601, 2048
    x0, w, r0, eps = make_inputs(rows, hidden, torch.float16, "c0", seed=5, device=cuda)
    sentinel = -4321
    xbuf = torch.full((rows + 2, hidden + 64), sentinel, dtype=torch.int16, device=cuda)
    rbuf = torch.full((rows + 2, hidden + 8), sentinel, dtype=torch.int16, device=cuda)
    x = xbuf.view(torch.float16)[1:-1, 8:8 + hidden]
    r = rbuf.view(torch.float16)[1:-1, :hidden]
    x.copy_(x0)
    r.copy_(r0)
    want_out, want_res = O.fused_add_rms_norm(O.FP16, bits(x0), bits(w), bits(r0), eps)
    with forced("tma:vec16:vpt2:tpr128:cluster1:rpc6"):
        capi.rms_norm_tensors(x, w, r, eps)
    torch.cuda.synchronize()
    assert_bits_equal(bits(r), want_res, O.FP16, label="strided residual")
    assert_output_close(bits(x), want_out, O.FP16, label="strided output")
    xs = xbuf.cpu().numpy()
    rs = rbuf.cpu().numpy()
    assert (xs[0] == sentinel).all() and (xs[-1] == sentinel).all()
    assert (xs[1:-1, :8] == sentinel).all() and (xs[1:-1, 8 + hidden:] == sentinel).all()
    assert (rs[0] == sentinel).all() and (rs[-1] == sentinel).all()
    assert (rs[1:-1, hidden:] == sentinel).all()


def test_tma_chain_with_and_without_pdl_and_in_a_graph(cuda):
    """Three dependent launches (each reads what the previous one wrote) give
    the same bits with programmatic dependent launch as with plain launches,
    eagerly and as a CUDA graph.  (Bits are compared within the plan: another
    plan sums squares in another order, and the output may differ by an ulp.)"""
    rows, hidden = 2048, 2048
    x0, w, r0, eps = make_inputs(rows, hidden, torch.bfloat16, "c0", seed=9, device=cuda)

    def chain(flags):
        x, r = x0.clone(), r0.clone()
        for _ in range(3):
            capi.rms_norm_tensors(x, w, r, eps, flags=flags)
        return x, r

    with forced("tma:vec16:vpt1:tpr256:cluster1:rpc4"):
        want = chain(0)
        torch.cuda.synchronize()
        for flags in (capi.LAUNCH_PDL, capi.LAUNCH_DEFAULT):
            got = chain(flags)
            torch.cuda.synchronize()
            assert torch.equal(got[0].view(torch.int16), want[0].view(torch.int16))
            assert torch.equal(got[1].view(torch.int16), want[1].view(torch.int16))
        x, r = x0.clone(), r0.clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(3):
                capi.rms_norm_tensors(x, w, r, eps, stream=s.cuda_stream)
        x.copy_(x0)
        r.copy_(r0)
        g.replay()
        torch.cuda.synchronize()
    assert torch.equal(x.view(torch.int16), want[0].view(torch.int16))
    assert torch.equal(r.view(torch.int16), want[1].view(torch.int16))


def test_tma_plan_rejections(cuda):
    x, w, r, eps = make_inputs(4, 16384, torch.bfloat16, "c0", seed=1, device=cuda)
    # Four 64 KB stages do not fit one CTA's shared memory.
    with forced("tma:vec16:vpt8:tpr256:cluster1:rpc4"):
        with pytest.raises(capi.HprnError, match="shared memory"):
            capi.rms_norm_tensors(x, w, r, eps)
    # Rows are staged as 16- or 32-byte vectors; an 8-byte width is not a tma plan.
    with forced("tma:vec8:vpt4:tpr128:cluster1:rpc2"):
        with pytest.raises(capi.HprnError, match="not compiled"):
            capi.rms_norm_tensors(x[:, :4096].contiguous(), w[:4096].contiguous(),
                                  r[:, :4096].contiguous(), eps)
    # Misaligned rows (2-byte offset) cannot be bulk-copied.
    xb = torch.empty(4 * 1024 + 1, dtype=torch.bfloat16, device=cuda)[1:].view(4, 1024)
    with forced("tma:vec16:vpt1:tpr128:cluster1:rpc2"):
        with pytest.raises(capi.HprnError, match="vector width"):
            capi.rms_norm_tensors(xb, w[:1024].contiguous(), r[:, :1024].contiguous(), eps)


def _row_states(got_x, got_r, x0, r0, want_out, want_res, fused):
    """Per row: 'done' (residual bit-exact, output within the parity bar),
    'untouched' (input and residual as they were), or 'mixed'."""
    states = []
    for i in range(got_x.shape[0]):
        untouched = np.array_equal(got_x[i], x0[i]) and (not fused or np.array_equal(got_r[i], r0[i]))
        res_ok = not fused or np.array_equal(got_r[i], want_res[i])
        a = got_x[i].astype(np.int32)
        b = want_out[i].astype(np.int32)
        oa = np.where(a & 0x8000, -(a & 0x7FFF), a)
        ob = np.where(b & 0x8000, -(b & 0x7FFF), b)
        done = res_ok and int(np.abs(oa - ob).max()) <= 1
        states.append("untouched" if untouched else ("done" if done else "mixed"))
    return states


@pytest.mark.parametrize("fused", [True, False])
def test_tma_wait_that_runs_out_is_reported(cuda, fused):
    """The bounded-wait give-up path, made to run on purpose: the test hook
    hprn_test_stall_bulk_copy makes one row's staged copy expect 16 bytes more
    than it delivers, so that row's mbarrier phase cannot complete and its wait
    runs out after 2 ms.  The call still completes; the CTA holding the row
    lets its other copies land, counts itself once in hprn_wait_timeouts and
    returns.  Every row is then either done exactly as the oracle says or
    untouched, and the untouched rows are exactly the stalled row and the
    later rows of the same CTA (rows stall, stall + G, ... of the persistent
    grid of G CTAs).  A second call stalls the second row of a CTA, whose first
    row must be done.  The counter resets to 0, and a call without the hook
    matches the oracle."""
    rows, hidden = 4096, 1024
    plan = "tma:vec16:vpt1:tpr128:cluster1:rpc4"
    x0, w, r0, eps = make_inputs(rows, hidden, torch.bfloat16, "c0", seed=77, device=cuda)
    xb, wb, rb = bits(x0), bits(w), bits(r0)
    want_out, want_res, _ = O.rms_norm_out(O.BF16, xb, wb, eps, r=rb if fused else None)
    sentinel = np.full_like(xb, 0x7E7E)

    def stalled_call(stall_row):
        x, r = x0.clone(), r0.clone()
        out = x if fused else torch.from_numpy(sentinel.view(np.int16)).to(cuda).view(torch.bfloat16)
        capi.wait_timeouts(reset=True)
        try:
            capi.test_stall_bulk_copy(stall_row, 2_000_000)
            with forced(plan):
                if fused:
                    capi.rms_norm_tensors(x, w, r, eps)
                else:
                    capi.rms_norm_out_tensors(out, x, w, None, eps)
            torch.cuda.synchronize()
        finally:
            capi.test_stall_bulk_copy(None)
        assert capi.wait_timeouts(reset=True) == 1, "exactly one CTA gives up"
        assert capi.wait_timeouts() == 0, "the count resets"
        if fused:
            return _row_states(bits(x), bits(r), xb, rb, want_out, want_res, True)
        assert torch.equal(x.view(torch.int16), x0.view(torch.int16)), "plain form: input unchanged"
        return _row_states(bits(out), bits(r), sentinel, rb, want_out, want_res, False)

    states = stalled_call(0)
    assert "mixed" not in states
    untouched = [i for i, s in enumerate(states) if s == "untouched"]
    assert untouched[0] == 0
    grid = untouched[1] if len(untouched) > 1 else rows
    assert untouched == list(range(0, rows, grid)), untouched[:8]
    if grid + 3 < rows:
        states = stalled_call(grid + 3)
        assert "mixed" not in states
        untouched = [i for i, s in enumerate(states) if s == "untouched"]
        assert untouched == list(range(grid + 3, rows, grid)), untouched[:8]
        assert states[3] == "done", "the stalled CTA's rows before the stall are complete"

    x, r = x0.clone(), r0.clone()
    with forced(plan):
        capi.rms_norm_tensors(x, w, r, eps)
    torch.cuda.synchronize()
    want_out_f, want_res_f = O.fused_add_rms_norm(O.BF16, xb, wb, rb, eps, O.SS_UNROUNDED)
    assert_bits_equal(bits(r), want_res_f, O.BF16, label="after the stall: residual")
    assert_output_close(bits(x), want_out_f, O.BF16, label="after the stall: output")
