"""Gated activations (silu/gelu/gelu_tanh-and-mul): the oracle against plain
PyTorch on CPU (CPU only)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle as O
from tests.numerics import assert_activation_close

TORCH_ACT = {
    "silu": F.silu,
    "gelu": lambda a: F.gelu(a, approximate="none"),
    "gelu_tanh": lambda a: F.gelu(a, approximate="tanh"),
}


@pytest.mark.parametrize("act", list(TORCH_ACT))
@pytest.mark.parametrize("code,tdt", [(O.BF16, torch.bfloat16), (O.FP16, torch.float16)])
def test_oracle_matches_torch_fp32(act, code, tdt):
    g = torch.Generator().manual_seed(0)
    x = (3 * torch.randn(37, 2 * 1000, generator=g)).to(tdt)
    d = 1000
    want = (TORCH_ACT[act](x[:, :d].float()) * x[:, d:].float()).to(tdt)
    got = O.act_and_mul(code, act, x.view(torch.int16).numpy().view(np.uint16))
    frac = assert_activation_close(got, want.view(torch.int16).numpy().view(np.uint16), code,
                                   label=act)
    assert frac < 0.01
