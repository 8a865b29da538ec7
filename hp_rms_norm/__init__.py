"""Import-name shim: ``import hp_rms_norm`` resolves to hp_rms_norm_b200.

Code written against the reference package (``import hp_rms_norm;
hp_rms_norm.hp_rms_norm(input, weight, residual, eps)``) runs unchanged on the
B200-native implementation.  ``hp_rms_norm._C`` is the same extension module.
"""
import sys as _sys

import hp_rms_norm_b200 as _impl
from hp_rms_norm_b200 import _C  # noqa: F401
from hp_rms_norm_b200.ops import *  # noqa: F401,F403
from hp_rms_norm_b200.ops import hp_rms_norm, relu  # noqa: F401

_sys.modules[__name__ + "._C"] = _C
_sys.modules[__name__ + ".ops"] = _impl.ops
