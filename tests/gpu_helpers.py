"""Helpers for the -m gpu tests: seeded inputs, bit-pattern transfers, and the
plain-PyTorch fp32 reference used at full sizes."""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as O

DTYPES = {"bf16": (torch.bfloat16, O.BF16), "fp16": (torch.float16, O.FP16)}


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16).copy()


def from_bits(b: np.ndarray, dtype: torch.dtype, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16).copy()).view(dtype).to(device)


def make_inputs(rows: int, hidden: int, dtype: torch.dtype, dist: str, seed: int, device):
    """BASELINE distributions, generated on the host with a fixed seed.

    c0: input, residual ~ N(0,1), weight ~ N(1, 0.1), eps 1e-6   (configs 0, 1, 4)
    c2: N(0,2) with 1% of elements x50, weight ~ U(0.5, 1.5), eps 1e-5 (config 2)
    rt: the reference test's N(0, 0.1) for all three, eps = finfo(bf16).eps
    """
    if dist == "c0" and rows * hidden >= 1 << 28:  # large: seeded on the device, for speed
        g = torch.Generator(device=device).manual_seed(seed)
        x = torch.randn(rows, hidden, generator=g, device=device)
        r = torch.randn(rows, hidden, generator=g, device=device)
        w = 1.0 + 0.1 * torch.randn(hidden, generator=g, device=device)
        return x.to(dtype), w.to(dtype), r.to(dtype), 1e-6
    g = torch.Generator().manual_seed(seed)
    if dist == "c0":
        x = torch.randn(rows, hidden, generator=g)
        r = torch.randn(rows, hidden, generator=g)
        w = 1.0 + 0.1 * torch.randn(hidden, generator=g)
        eps = 1e-6
    elif dist == "c2":
        x = 2.0 * torch.randn(rows, hidden, generator=g)
        r = 2.0 * torch.randn(rows, hidden, generator=g)
        for t in (x, r):
            t[torch.rand(rows, hidden, generator=g) < 0.01] *= 50.0
        w = 0.5 + torch.rand(hidden, generator=g)
        eps = 1e-5
    else:
        x = 0.1 * torch.randn(rows, hidden, generator=g)
        r = 0.1 * torch.randn(rows, hidden, generator=g)
        w = 0.1 * torch.randn(hidden, generator=g)
        eps = float(torch.finfo(torch.bfloat16).eps)
    return x.to(dtype).to(device), w.to(dtype).to(device), r.to(dtype).to(device), eps


def torch_fp32_reference(x: torch.Tensor, w: torch.Tensor, r: torch.Tensor, eps: float):
    """The fused op in plain PyTorch on the GPU, fp32 arithmetic, fp64 sum of
    squares of the unrounded sums: returns (output, residual)."""
    s = x.float() + r.float()
    res = s.to(x.dtype)
    ss = (s.double() * s.double()).sum(-1, keepdim=True)
    inv = torch.rsqrt(ss / x.shape[-1] + eps).float()
    out = (res.float() * w.float() * inv).to(x.dtype)
    return out, res


def ulp_distance(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Elementwise ulp distance between two 16-bit float tensors (on device)."""
    def ordered(t):
        i = t.view(torch.int16).int()
        mag = i & 0x7FFF
        return torch.where(i < 0, -mag, mag)

    return (ordered(a) - ordered(b)).abs()
