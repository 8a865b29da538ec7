"""GPU parity of the ReLU kernel, called through the C ABI: bit-exact against
torch.relu (CUDA) on every non-NaN value and against the C oracle on every bit
pattern, NaN payloads included."""
import numpy as np
import pytest
import torch

import hp_rms_norm_b200
from hp_rms_norm_b200 import capi
from oracle import oracle as O
from tests.gpu_helpers import DTYPES, bits, from_bits
from tests.numerics import assert_bits_equal, is_nan

pytestmark = pytest.mark.gpu


def run(out, inp):
    capi.relu_tensors(out, inp)
    torch.cuda.synchronize()


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_every_bit_pattern(cuda, dtype):
    tdtype, code = DTYPES[dtype]
    allbits = np.arange(65536, dtype=np.uint32).astype(np.uint16).reshape(256, 256)
    x = from_bits(allbits, tdtype, cuda)
    out = torch.empty_like(x)
    run(out, x)
    got = bits(out)
    assert_bits_equal(got, O.relu(code, allbits), code, label="vs oracle")
    want_torch = bits(torch.relu(x))
    assert_bits_equal(got, want_torch, code, label="vs torch.relu", nan_payload=False)
    nan = is_nan(allbits.reshape(-1), code)
    assert (got.reshape(-1)[nan] == allbits.reshape(-1)[nan]).all(), "NaN bits pass through"


def test_golden_fixture(cuda, relu_golden):
    """CPU torch.relu fixtures: bit-exact except -0.0 (CUDA's torch.relu, which the
    kernel follows, gives +0) and NaN payloads (kept by the kernel)."""
    for name in ("bf16", "fp16"):
        tdtype, code = DTYPES[name]
        xb, want = relu_golden[name]
        x = from_bits(xb, tdtype, cuda)
        out = torch.zeros_like(x)
        run(out, x)
        got = bits(out).reshape(-1)
        xb, want = xb.reshape(-1), want.reshape(-1)
        keep = ~is_nan(xb, code) & (xb != 0x8000)
        assert_bits_equal(got[keep], want[keep], code, label=name)
        assert_bits_equal(got, O.relu(code, xb), code, label=name + " vs oracle")


@pytest.mark.parametrize("shape,dtype", [((4096, 14336), "bf16"), ((8192, 28672), "fp16")])
def test_config3_shapes_vs_torch_relu(cuda, shape, dtype):
    tdtype, _ = DTYPES[dtype]
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(shape, generator=g, device=cuda).to(tdtype)
    out = torch.empty_like(x)
    run(out, x)
    assert torch.equal(out.view(torch.int16), torch.relu(x).view(torch.int16))


@pytest.mark.parametrize("shape", [(1, 1), (3, 1001), (5, 7), (2, 4095), (7, 16), (1, 100003)])
def test_ragged_sizes_and_canaries(cuda, shape):
    rows, hidden = shape
    n = rows * hidden
    x0 = torch.randn(n, device=cuda).to(torch.bfloat16)
    sentinel = 0x5A5A
    obuf = torch.full((n + 64,), sentinel, dtype=torch.int16, device=cuda)
    out = obuf[16:16 + n].view(torch.bfloat16).view(rows, hidden)
    run(out, x0.view(rows, hidden))
    assert torch.equal(out.reshape(-1).view(torch.int16), torch.relu(x0).view(torch.int16))
    assert bool((obuf[:16] == sentinel).all()) and bool((obuf[16 + n:] == sentinel).all())


def test_strided_rows_misaligned_and_in_place(cuda):
    x = torch.randn(33, 1100, device=cuda).to(torch.float16)
    src = x[:, 3:1003]          # row stride 1100, 6-byte offset
    dst_buf = torch.zeros(33, 1200, dtype=torch.float16, device=cuda)
    dst = dst_buf[:, 100:1100]
    capi.relu_tensors(dst, src)
    torch.cuda.synchronize()
    assert torch.equal(dst.view(torch.int16), torch.relu(src).view(torch.int16))
    assert bool((dst_buf[:, :100] == 0).all()) and bool((dst_buf[:, 1100:] == 0).all())
    y = torch.randn(64, 4096, device=cuda).to(torch.bfloat16)
    want = torch.relu(y)
    capi.relu_tensors(y, y)
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), want.view(torch.int16))


def test_torch_op_api(cuda):
    x = torch.randn(4, 9, 777, device=cuda).to(torch.bfloat16)
    out = torch.zeros_like(x)
    hp_rms_norm_b200.relu(out, x)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), torch.relu(x).view(torch.int16))
    with pytest.raises(RuntimeError, match="same dtype"):
        hp_rms_norm_b200.relu(out.half(), x)
    with pytest.raises(RuntimeError, match="input.size\\(i\\) == out.size\\(i\\)"):
        hp_rms_norm_b200.relu(out[:, :4], x)
