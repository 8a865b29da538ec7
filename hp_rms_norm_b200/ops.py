"""Python API.

The reference's two functions, argument for argument (hp_rms_norm/ops.py:4-24):
``hp_rms_norm(input, weight, residual, eps)`` runs the fused residual add +
RMSNorm in place (``residual += input``; ``input = RMSNorm(residual) * weight``)
and returns None; ``relu(output, input)`` writes ``torch.relu(input)`` into
``output`` and returns None.

Extensions (not in the reference): ``rms_norm`` (plain RMSNorm),
``fused_add_rms_norm`` (the fused op into a separate output) and
``rms_norm_fp8`` (either form with an fp8 e4m3 output, static or per-row
scale), ``rms_norm_nvfp4`` (NVFP4 output), and the gated activations ``silu_and_mul``, ``gelu_and_mul`` and
``gelu_tanh_and_mul``.  Everything dispatches through ``torch.ops.hp_rms_norm``, registered
by this package's compiled ``_C`` extension.
"""
import torch


def hp_rms_norm(
    input,
    weight,
    residual,
    eps,
):
    torch.ops.hp_rms_norm.rms_norm.default(input, weight, residual, eps)


def relu(
    output,
    input,
):
    torch.ops.hp_rms_norm.relu.default(output, input)


def rms_norm(input, weight, eps, out=None):
    """RMSNorm without a residual: out = input * rsqrt(mean(input^2) + eps) * weight,
    in the input's dtype; ``out`` may be ``input`` (in place).  Returns ``out``."""
    if out is None:
        out = torch.empty_like(input)
    torch.ops.hp_rms_norm.rms_norm_out.default(out, input, weight, None, eps)
    return out


def fused_add_rms_norm(input, residual, weight, eps, out=None):
    """``hp_rms_norm`` into a separate output: residual += input (in place);
    out = RMSNorm(residual) * weight; ``input`` is left unchanged unless it is
    ``out``.  Returns ``out``."""
    if out is None:
        out = torch.empty_like(input)
    torch.ops.hp_rms_norm.rms_norm_out.default(out, input, weight, residual, eps)
    return out


def rms_norm_fp8(input, weight, eps, residual=None, scale=None, out=None):
    """RMSNorm (fused with ``residual += input`` when a residual is given) with
    an fp8 e4m3 output.  With ``scale`` (a one-element float32 tensor) the output
    is e4m3(y / scale); without it, each row gets scale max|y| / 448, returned
    as a float32 tensor of shape input.shape[:-1].  Returns (out, scales)."""
    if out is None:
        out = torch.empty(input.shape, dtype=torch.float8_e4m3fn, device=input.device)
    if scale is not None:
        torch.ops.hp_rms_norm.rms_norm_fp8.default(out, input, weight, residual, eps, scale, None)
        return out, scale
    row_scales = torch.empty(input.shape[:-1], dtype=torch.float32, device=input.device)
    torch.ops.hp_rms_norm.rms_norm_fp8.default(out, input, weight, residual, eps, None, row_scales)
    return out, row_scales


def rms_norm_nvfp4(input, weight, eps, global_scale, residual=None):
    """RMSNorm (fused with ``residual += input`` when a residual is given) with
    an NVFP4 output: returns (codes, block_scales), codes uint8
    [..., hidden/2] holding two e2m1 values per byte (element 2k in the low
    nibble), block_scales float8_e4m3fn [..., hidden/16]; the normalised value
    is approximately e2m1 * block_scale / global_scale (``global_scale`` a
    one-element float32 tensor)."""
    h = input.shape[-1]
    codes = torch.empty(input.shape[:-1] + (h // 2,), dtype=torch.uint8, device=input.device)
    scales = torch.empty(input.shape[:-1] + (h // 16,), dtype=torch.float8_e4m3fn,
                         device=input.device)
    torch.ops.hp_rms_norm.rms_norm_nvfp4.default(codes, scales, input, weight, residual, eps,
                                                 global_scale)
    return codes, scales


def rms_norm_fp8_group(input, weight, eps, residual=None, group_size=128, scale_pow2=False,
                       column_major_scales=False):
    """RMSNorm (fused with ``residual += input`` when a residual is given) with a
    per-token-group fp8 output: returns (out, scales), out float8_e4m3fn
    [..., hidden], scales float32 [rows, hidden / group_size] (rows = the
    leading dimensions flattened) with out ~ y / scale per group of
    ``group_size`` elements.  ``scale_pow2`` rounds scales up to powers of two;
    ``column_major_scales`` returns a transposed view of a [hidden /
    group_size, rows] buffer (the layout block-scaled FP8 GEMMs read)."""
    h = input.shape[-1]
    rows = input.numel() // h if h else 0
    out = torch.empty(input.shape, dtype=torch.float8_e4m3fn, device=input.device)
    if column_major_scales:
        scales = torch.empty((h // group_size, rows), dtype=torch.float32, device=input.device).t()
    else:
        scales = torch.empty((rows, h // group_size), dtype=torch.float32, device=input.device)
    torch.ops.hp_rms_norm.rms_norm_fp8_group.default(out, scales, input, weight, residual, eps,
                                                     group_size, scale_pow2)
    return out, scales


def _act_and_mul(op, input, out):
    if out is None:
        out = torch.empty(input.shape[:-1] + (input.shape[-1] // 2,), dtype=input.dtype,
                          device=input.device)
    op(out, input)
    return out


def silu_and_mul(input, out=None):
    """out = silu(input[..., :d]) * input[..., d:], d = input.shape[-1] // 2."""
    return _act_and_mul(torch.ops.hp_rms_norm.silu_and_mul.default, input, out)


def gelu_and_mul(input, out=None):
    """out = gelu(input[..., :d]) * input[..., d:] (erf form)."""
    return _act_and_mul(torch.ops.hp_rms_norm.gelu_and_mul.default, input, out)


def gelu_tanh_and_mul(input, out=None):
    """out = gelu_tanh(input[..., :d]) * input[..., d:] (tanh approximation)."""
    return _act_and_mul(torch.ops.hp_rms_norm.gelu_tanh_and_mul.default, input, out)


__all__ = ["hp_rms_norm", "relu", "rms_norm", "fused_add_rms_norm", "rms_norm_fp8", "rms_norm_nvfp4",
           "rms_norm_fp8_group", "silu_and_mul", "gelu_and_mul", "gelu_tanh_and_mul", "torch"]
