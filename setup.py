"""Packaging for hp_rms_norm_b200 (sm_100a only).

    python setup.py build_ext --inplace     # build the two native libraries in-tree
    pip install --no-build-isolation .      # build, then install the packages

The native build itself lives in hp_rms_norm_b200/build.py (nvcc for the CUDA
library, g++ against the installed torch for the operator binding); this file
only hooks it into setuptools and ships the built .so files as package data.
Installs two packages: ``hp_rms_norm_b200`` and the ``hp_rms_norm`` import-name
shim, so code written against the reference (``import hp_rms_norm``) runs
unchanged.
"""
import importlib.util
import os

from setuptools import setup
from setuptools.command.build_ext import build_ext
from setuptools.command.build_py import build_py

ROOT = os.path.dirname(os.path.abspath(__file__))


def _native_build():
    spec = importlib.util.spec_from_file_location(
        "_hprn_build", os.path.join(ROOT, "hp_rms_norm_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build(force=os.environ.get("HPRN_FORCE_BUILD", "0") == "1")


class BuildNative(build_ext):
    def run(self):
        _native_build()


class BuildPy(build_py):
    def run(self):
        _native_build()
        super().run()


setup(
    name="hp_rms_norm_b200",
    version="1.0.0",
    description="B200-native fused residual-add + RMSNorm and ReLU (drop-in for hp_rms_norm)",
    packages=["hp_rms_norm_b200", "hp_rms_norm"],
    package_data={"hp_rms_norm_b200": ["*.so", "csrc/*"]},
    include_package_data=True,
    install_requires=["torch"],
    cmdclass={"build_ext": BuildNative, "build_py": BuildPy},
)
