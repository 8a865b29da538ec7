"""In-tree build of the two native libraries (no JIT cache, no pip install).

* ``libhp_rms_norm_b200.so``: the CUDA kernels and the C ABI declared in
  ``include/hp_rms_norm_b200.h``.  nvcc, sm_100a only, CUDA runtime linked
  statically so the library depends on nothing but the driver.
* ``_C.<abi>.so``: the torch operator binding (``torch.ops.hp_rms_norm.*``),
  plain C++ against the installed torch headers, linked to the library above
  through an ``$ORIGIN`` rpath.

Both land next to this file so they travel with the source tree.  Usage:
``python hp_rms_norm_b200/build.py [--force]`` (run as a script: importing the
package needs the built extension; ``setup.py build_ext`` and
``__graft_entry__.build()`` load this file by path and call ``build()``).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB_NAME = "libhp_rms_norm_b200.so"
LIB = os.path.join(PKG, LIB_NAME)
CUDA_SOURCES = ["rms_norm.cu", "relu.cu", "act_and_mul.cu", "runtime.cu"]
HEADERS = ["vec.cuh", "bulk.cuh", "runtime.cuh", "rms_norm_kernels.cuh"]

# HPRN_DEBUG=1 (or the reference's own DEBUG=1, setup.py:23-28 there) builds
# host code without optimisation and with debug symbols (device code keeps -O3
# and -lineinfo, so kernels stay representative).
DEBUG = os.environ.get("HPRN_DEBUG", os.environ.get("DEBUG", "0")) == "1"
# The reference's USE_CUDA=0 builds its extension without kernels; this
# package is its CUDA kernels, so there is no such build.
if os.environ.get("USE_CUDA", "1") == "0":
    raise SystemExit("hp_rms_norm_b200 has no CPU-only build (USE_CUDA=0): it is CUDA kernels "
                     "for sm_100a; unset USE_CUDA")
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-Xptxas", "-v",
] + (["-Xcompiler", "-O0", "-Xcompiler", "-g"] if DEBUG else [])


def ext_path() -> str:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(PKG, "_C" + suffix)


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(cuda_home, "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd: list[str], log: str) -> None:
    with open(log, "w") as f:
        r = subprocess.run(cmd, stdout=f, stderr=subprocess.STDOUT)
    if r.returncode != 0:
        with open(log) as f:
            sys.stderr.write(f.read())
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(cmd)}")


def build_library(force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "hp_rms_norm_b200.h")]
    objs, jobs = [], []
    for src in CUDA_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if force or _stale(o, [s, __file__] + headers):
            cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", s, "-o", o]
            jobs.append((cmd, o + ".log"))
    with cf.ThreadPoolExecutor(max_workers=len(CUDA_SOURCES)) as ex:
        list(ex.map(lambda j: _run(*j), jobs))
    if force or jobs or _stale(LIB, objs):
        cmd = [_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
               "-cudart", "static", "-Xcompiler", "-fPIC", "-o", LIB, *objs]
        _run(cmd, os.path.join(BUILD, "link.log"))
    return LIB


def build_torch_binding(force: bool = False) -> str:
    import torch
    from torch.utils import cpp_extension

    out = ext_path()
    src = os.path.join(CSRC, "torch_ops.cpp")
    if not (force or _stale(out, [src, LIB, __file__, os.path.join(INCLUDE, "hp_rms_norm_b200.h")])):
        return out
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    incs = cpp_extension.include_paths() + [os.path.join(cuda_home, "include"), INCLUDE,
                                            sysconfig.get_paths()["include"]]
    libdirs = cpp_extension.library_paths()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O0" if DEBUG else "-O2", "-std=c++17", "-shared", "-fPIC",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C"]
    if DEBUG:
        cmd.append("-g")
    cmd += [f"-I{d}" for d in incs]
    cmd += [src, "-o", out, f"-L{PKG}", "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN"]
    for d in libdirs:
        cmd += [f"-L{d}", f"-Wl,-rpath,{d}"]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch_cpu"]
    _run(cmd, os.path.join(BUILD, "torch_ops.log"))
    return out


def build(force: bool = False) -> tuple[str, str]:
    lib = build_library(force)
    ext = build_torch_binding(force)
    return lib, ext


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
