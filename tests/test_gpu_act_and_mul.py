"""GPU parity of the gated activations (silu/gelu/gelu_tanh-and-mul) through
the C ABI and the torch ops: within 1 ulp of the C oracle and of PyTorch's own
activation computed in fp32 (expf / erff / tanhf implementations may differ in
the last fp32 bit, which can move a 16-bit rounding by one ulp)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import hp_rms_norm_b200
from hp_rms_norm_b200 import capi
from oracle import oracle as O
from tests.gpu_helpers import DTYPES, bits
from tests.numerics import assert_activation_close

pytestmark = pytest.mark.gpu

ACTS = {"silu": (capi.ACT_SILU, F.silu, hp_rms_norm_b200.silu_and_mul),
        "gelu": (capi.ACT_GELU, lambda a: F.gelu(a), hp_rms_norm_b200.gelu_and_mul),
        "gelu_tanh": (capi.ACT_GELU_TANH, lambda a: F.gelu(a, approximate="tanh"),
                      hp_rms_norm_b200.gelu_tanh_and_mul)}


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("rows,d", [(4096, 14336), (7, 11008), (33, 4097), (1, 3), (128, 8)])
@pytest.mark.parametrize("act", list(ACTS))
def test_act_and_mul_vs_oracle_and_torch(cuda, act, rows, d, dtype):
    tdtype, code = DTYPES[dtype]
    code_act, torch_act, _ = ACTS[act]
    g = torch.Generator(device=cuda).manual_seed(rows + d)
    x = (2 * torch.randn(rows, 2 * d, generator=g, device=cuda)).to(tdtype)
    out = torch.empty(rows, d, dtype=tdtype, device=cuda)
    capi.act_and_mul_tensors(out, x, code_act)
    torch.cuda.synchronize()
    got = bits(out)
    if rows * d <= 1 << 20:
        assert_activation_close(got, O.act_and_mul(code, act, bits(x)), code, label=act + " oracle")
    want = (torch_act(x[:, :d].float()) * x[:, d:].float()).to(tdtype)
    frac = assert_activation_close(got, bits(want), code, label=act + " torch")
    assert frac < 0.01


@pytest.mark.parametrize("act", list(ACTS))
def test_torch_op_strided_and_3d(cuda, act):
    code_act, torch_act, api = ACTS[act]
    x = torch.randn(4, 9, 2 * 1536, device=cuda).to(torch.bfloat16)
    out = api(x)
    assert out.shape == (4, 9, 1536)
    ref = torch.empty(36, 1536, dtype=torch.bfloat16, device=cuda)
    capi.act_and_mul_tensors(ref, x.view(36, 3072), code_act)
    torch.cuda.synchronize()
    assert torch.equal(out.view(36, 1536).view(torch.int16), ref.view(torch.int16))
    # Strided rows (a slice of a wider buffer) and a row-strided output.
    wide = torch.randn(16, 3072 + 64, device=cuda).to(torch.bfloat16)
    src = wide[:, 32:32 + 3072]
    dst_buf = torch.zeros(16, 1536 + 16, dtype=torch.bfloat16, device=cuda)
    capi.act_and_mul_tensors(dst_buf[:, 16:], src, code_act)
    torch.cuda.synchronize()
    want = (torch_act(src[:, :1536].float()) * src[:, 1536:].float()).to(torch.bfloat16)
    assert int((dst_buf[:, 16:].view(torch.int16).int() - want.view(torch.int16).int()).abs().max()) <= 1
    assert bool((dst_buf[:, :16] == 0).all())


def test_act_and_mul_errors(cuda):
    x = torch.randn(4, 64, device=cuda).to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="even"):
        hp_rms_norm_b200.silu_and_mul(x[:, :63])
    with pytest.raises(capi.HprnError, match="overlap"):
        capi.act_and_mul(x.data_ptr(), x.data_ptr(), 4, 32, 64, 64, capi.ACT_SILU, capi.DTYPE_BF16)
    with pytest.raises(capi.HprnError, match="unknown activation"):
        capi.act_and_mul(x.data_ptr(), x.data_ptr(), 4, 32, 64, 64, 9, capi.DTYPE_BF16)
