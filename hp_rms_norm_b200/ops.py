"""Python API, argument for argument the reference's (hp_rms_norm/ops.py:4-24).

``hp_rms_norm(input, weight, residual, eps)`` runs the fused residual add +
RMSNorm in place (``residual += input``; ``input = RMSNorm(residual) * weight``)
and returns None; ``relu(output, input)`` writes ``torch.relu(input)`` into
``output`` and returns None.  Both dispatch through ``torch.ops.hp_rms_norm``,
which this package registers from its compiled ``_C`` extension.
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


__all__ = ["hp_rms_norm", "relu", "torch"]
