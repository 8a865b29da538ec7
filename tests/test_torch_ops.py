"""The torch-op surface on CPU: same namespace, op names, argument order and
Python API as the reference (hp_rms_norm/csrc/hp_rms_norm.cpp:35-43,
hp_rms_norm/ops.py:4-24), plus the mutation-annotated schema and Meta kernels."""
import inspect

import pytest
import torch

import hp_rms_norm
import hp_rms_norm_b200


def test_schemas():
    s1 = str(torch.ops.hp_rms_norm.rms_norm.default._schema)
    s2 = str(torch.ops.hp_rms_norm.relu.default._schema)
    assert s1 == ("hp_rms_norm::rms_norm(Tensor(a!) input, Tensor weight, Tensor(b!) residual, "
                  "float eps) -> ()")
    assert s2 == "hp_rms_norm::relu(Tensor(a!) out, Tensor input) -> ()"


def test_python_api_signatures_match_reference():
    assert list(inspect.signature(hp_rms_norm_b200.hp_rms_norm).parameters) == [
        "input", "weight", "residual", "eps"]
    assert list(inspect.signature(hp_rms_norm_b200.relu).parameters) == ["output", "input"]


def test_import_name_shim():
    assert hp_rms_norm.hp_rms_norm is hp_rms_norm_b200.hp_rms_norm
    assert hp_rms_norm.relu is hp_rms_norm_b200.relu
    import importlib

    # The reference exposes its extension as hp_rms_norm._C.
    assert importlib.import_module("hp_rms_norm._C") is hp_rms_norm_b200._C


def test_cpu_tensors_have_no_kernel():
    """Like the reference, only the CUDA dispatch key is implemented: no silent CPU path."""
    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        hp_rms_norm_b200.hp_rms_norm(x, torch.ones(8, dtype=torch.bfloat16), x.clone(), 1e-6)
    with pytest.raises(NotImplementedError):
        hp_rms_norm_b200.relu(torch.empty_like(x), x)


def test_meta_kernels_trace():
    x = torch.empty(4, 8, dtype=torch.bfloat16, device="meta")
    r = torch.empty(4, 8, dtype=torch.bfloat16, device="meta")
    w = torch.empty(8, dtype=torch.bfloat16, device="meta")
    assert torch.ops.hp_rms_norm.rms_norm(x, w, r, 1e-6) is None
    assert torch.ops.hp_rms_norm.relu(torch.empty_like(x), x) is None


def test_fp8_group_schema_and_meta_kernel():
    s = str(torch.ops.hp_rms_norm.rms_norm_fp8_group.default._schema)
    assert s == ("hp_rms_norm::rms_norm_fp8_group(Tensor(a!) out, Tensor(b!) scales, Tensor input, "
                 "Tensor weight, Tensor(c!)? residual, float eps, int group_size, bool scale_pow2) -> ()")
    x = torch.empty(4, 256, dtype=torch.bfloat16, device="meta")
    w = torch.empty(256, dtype=torch.bfloat16, device="meta")
    out = torch.empty(4, 256, dtype=torch.float8_e4m3fn, device="meta")
    sc = torch.empty(4, 2, dtype=torch.float32, device="meta")
    assert torch.ops.hp_rms_norm.rms_norm_fp8_group(out, sc, x, w, None, 1e-6, 128, False) is None
