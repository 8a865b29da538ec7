"""B200-native (sm_100a) fused residual-add + RMSNorm and ReLU.

Drop-in for the ``hp_rms_norm`` package: the same ``hp_rms_norm(input,
weight, residual, eps)`` and ``relu(output, input)`` functions and the same
``torch.ops.hp_rms_norm.{rms_norm,relu}`` operators.  Importing the package
loads the compiled ``_C`` extension (which registers the operators) and,
through it, ``libhp_rms_norm_b200.so`` (the CUDA kernels behind the C ABI in
``include/hp_rms_norm_b200.h``).  There is no CPU implementation: if the
extension has not been built, the import fails.
"""
import torch

from . import _C  # noqa: F401  (registers torch.ops.hp_rms_norm.*)
from .ops import *  # noqa: F401,F403
from .ops import (fused_add_rms_norm, gelu_and_mul, gelu_tanh_and_mul, hp_rms_norm, relu,
                  rms_norm, rms_norm_fp8, rms_norm_fp8_group, rms_norm_nvfp4, silu_and_mul)

__version__ = "1.0.0"
