"""Build recipe for the oracle (TEST INFRASTRUCTURE ONLY).

* ``oracle/liboracle.so``: the plain-C CPU restatement (rms_norm_oracle.c).
* ``oracle/_ref/libhp_rms_norm_ref.so``: the reference's own CUDA launchers
  (hp_rms_norm/csrc/cuda/hp_rms_norm.cuh, activation_kernels.cuh) compiled
  from the reference sources where they lie, with the reference's own nvcc
  flags (setup.py:36-48 of the reference: -O3 -DNDEBUG -std=c++17
  --use_fast_math, sm_100a), behind oracle/ref_shim.cu.  Only built where the
  reference tree exists; the GPU box uses the prebuilt file.

Nothing here is imported by the product package.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_SO = os.path.join(REF_DIR, "libhp_rms_norm_ref.so")
REFERENCE_ROOT = os.environ.get("HP_RMS_NORM_REFERENCE", "/root/reference")


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources if os.path.exists(s))


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "rms_norm_oracle.c")
    if force or _stale(ORACLE_SO, [src, __file__]):
        cmd = ["gcc", "-O2", "-ffp-contract=off", "-fopenmp", "-shared", "-fPIC",
               "-o", ORACLE_SO, src, "-lm"]
        subprocess.check_call(cmd)
    return ORACLE_SO


def build_reference(force: bool = False) -> str | None:
    """Compile the reference's CUDA launchers; returns the .so path or None."""
    cuda_dir = os.path.join(REFERENCE_ROOT, "hp_rms_norm", "csrc", "cuda")
    if not os.path.isdir(cuda_dir):
        return REF_SO if os.path.exists(REF_SO) else None
    shim = os.path.join(HERE, "ref_shim.cu")
    deps = [shim, os.path.join(cuda_dir, "hp_rms_norm.cuh"),
            os.path.join(cuda_dir, "activation_kernels.cuh"), __file__]
    if not (force or _stale(REF_SO, deps)):
        return REF_SO
    import torch
    from torch.utils import cpp_extension

    os.makedirs(REF_DIR, exist_ok=True)
    inc = cpp_extension.include_paths(device_type="cuda")
    libdirs = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["nvcc", "-O3", "-DNDEBUG", "-std=c++17", "--use_fast_math",
           "-gencode", "arch=compute_100a,code=sm_100a",
           "-Xcompiler", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-I", cuda_dir]
    for d in inc:
        cmd += ["-I", d]
    for d in libdirs:
        cmd += ["-L", d, f"-Xlinker", f"-rpath={d}"]
    cmd += ["-o", REF_SO, shim, "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda"]
    subprocess.check_call(cmd)
    return REF_SO


if __name__ == "__main__":
    build_oracle(force="--force" in sys.argv)
    print(build_reference(force="--force" in sys.argv))
