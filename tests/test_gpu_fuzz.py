"""Seeded randomized parity sweep on the GPU: random row counts, hidden sizes
(1 .. 40000, log-uniform), dtypes, row strides, pointer offsets (any even
byte offset, so every vector width is exercised) and every output form,
through the C ABI, against the C oracle.  Deterministic (fixed seed), a few
hundred cases, each small enough for the oracle."""
import numpy as np
import pytest
import torch

from hp_rms_norm_b200 import capi
from oracle import oracle as O
from tests.gpu_helpers import bits
from tests.numerics import assert_bits_equal, assert_output_close

pytestmark = pytest.mark.gpu

CASES = 240


def _strided(buf_rows, hidden, pad, offset, dtype, device, fill):
    """A [buf_rows, hidden] view with row stride hidden + pad, starting `offset`
    elements into a sentinel-filled buffer; returns (view, backing buffer)."""
    stride = hidden + pad
    raw = torch.int16 if dtype.itemsize == 2 else torch.uint8
    backing = torch.full((offset + buf_rows * stride + 8,), fill, dtype=raw, device=device)
    view = backing[offset:offset + buf_rows * stride].view(buf_rows, stride)[:, :hidden]
    return view.view(dtype), backing


@pytest.mark.parametrize("case", range(CASES))
def test_random_case(cuda, case):
    rng = np.random.default_rng(1000 + case)
    rows = int(rng.integers(1, 300))
    hidden = int(np.exp(rng.uniform(0, np.log(40000))))
    tname = rng.choice(["bf16", "fp16"])
    tdt, code = (torch.bfloat16, O.BF16) if tname == "bf16" else (torch.float16, O.FP16)
    forms = ["fused_in_place", "fused_out", "plain"]
    if hidden % 4 == 0:
        forms += ["fp8_static", "fp8_dynamic"]
    form = str(rng.choice(forms))
    fused = form != "plain" and (form != "fp8_static" or rng.random() < 0.5)
    if form == "fp8_dynamic":
        fused = rng.random() < 0.5
    eps = float(rng.choice([1e-6, 1e-5, 0.0078125]))

    vals = lambda: torch.from_numpy(
        (rng.standard_normal((rows, hidden)) * rng.choice([0.1, 1.0, 4.0])).astype(np.float32)).to(tdt)
    x0, r0 = vals(), vals()
    w0 = torch.from_numpy((1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)).to(tdt)

    fp8 = form.startswith("fp8")
    # fp8 rows need 8-byte aligned inputs (4-element offsets); 16-bit forms take any element offset.
    align = 4 if fp8 else 1
    off = lambda: int(rng.integers(0, 8)) * align
    pad = lambda: int(rng.integers(0, 3)) * (4 if fp8 else int(rng.integers(1, 5)))
    x, xb = _strided(rows, hidden, pad(), off(), tdt, cuda, 0x1234)
    r, rbk = _strided(rows, hidden, pad(), off(), tdt, cuda, 0x2345)
    wbuf = torch.zeros(hidden + 32, dtype=tdt, device=cuda)
    w = wbuf[off():][:hidden]
    x.copy_(x0)
    r.copy_(r0)
    w.copy_(w0)
    xbits, rbits, wbits = bits(x), bits(r), bits(w)
    label = f"case {case}: {rows}x{hidden} {tname} {form} fused={fused}"

    if form == "fused_in_place":
        capi.rms_norm_tensors(x, w, r, eps)
        torch.cuda.synchronize()
        want_out, want_res = O.fused_add_rms_norm(code, xbits, wbits, rbits, eps)
        assert_bits_equal(bits(r), want_res, code, label=label + " residual")
        assert_output_close(bits(x), want_out, code, label=label)
    else:
        scale = row_scales = None
        if fp8:
            out, ob = _strided(rows, hidden, pad(), off() * 2, torch.float8_e4m3fn, cuda, 0x55)
            ofill = 0x55
            if form == "fp8_static":
                scale = torch.tensor([float(rng.uniform(0.005, 0.05))], device=cuda)
            else:
                row_scales = torch.zeros(rows, device=cuda)
        else:
            out, ob = _strided(rows, hidden, pad(), off(), tdt, cuda, 0x3456)
            ofill = 0x3456
        capi.rms_norm_out_tensors(out, x, w, r if (fused or form == "fused_out") else None, eps,
                                  scale=scale, row_scales=row_scales)
        torch.cuda.synchronize()
        use_res = fused or form == "fused_out"
        want_out, want_res, want_scales = O.rms_norm_out(
            code, xbits, wbits, eps, r=rbits if use_res else None,
            fp8=None if not fp8 else ("static" if form == "fp8_static" else "dynamic"),
            scale=float(scale.item()) if scale is not None else 1.0)
        assert_bits_equal(bits(x), xbits, code, label=label + " input unchanged")
        if use_res:
            assert_bits_equal(bits(r), want_res, code, label=label + " residual")
        if fp8:
            got = out.view(torch.uint8).cpu().numpy().astype(np.int32)
            wnt = want_out.astype(np.int32)
            o = lambda b: np.where(b & 0x80, -(b & 0x7F), b & 0x7F)
            assert int(np.abs(o(got) - o(wnt)).max()) <= 1, label
            if row_scales is not None:
                np.testing.assert_allclose(row_scales.cpu().numpy(), want_scales, rtol=1e-5)
        else:
            assert_output_close(bits(out), want_out, code, label=label)
        assert int((ob == ofill).sum()) >= ob.numel() - rows * hidden, label + " out canary"
    # Nothing outside the views was written: every element outside them keeps its sentinel.
    for backing, fill in ((xb, 0x1234), (rbk, 0x2345)):
        assert int((backing == fill).sum()) >= backing.numel() - rows * hidden, label + " canary"
