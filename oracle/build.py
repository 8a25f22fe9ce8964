"""TEST INFRASTRUCTURE ONLY: builds the parity checkers.

* ``oracle/liboracle.so`` -- the C restatement (``fmha_oracle.c``).
* ``oracle/libgpu_ref.so`` -- the plain-CUDA fp32 device oracle
  (``gpu_ref.cu``, restating the reference's naive GPU reference) for full-size
  parity runs.
* ``oracle/_ref/libfmha_ref.so`` -- the reference's OWN CPU oracle and input
  generator, compiled unmodified from ``src/runner/cpu_ref.cpp`` and
  ``src/runner/buffers.cpp`` of the reference tree (needs the tree, so it is
  built only where the tree is mounted; the built ``.so`` then travels with
  the repository snapshot).  The only additions are ``shim/hip/hip_runtime.h``
  (host-memory stand-ins for hipMalloc/hipMemcpy/...) and ``ref_entry.cpp``
  (extern "C" wrappers).

Usage: ``python oracle/build.py [--force] [--reference-root DIR]`` (or set
``FMHA_REFERENCE_ROOT``); without a reference root the reference library is
left as built.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

ORACLE_DIR = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(ORACLE_DIR, "liboracle.so")
REF_DIR = os.path.join(ORACLE_DIR, "_ref")
REF_LIB = os.path.join(REF_DIR, "libfmha_ref.so")
GPU_REF_LIB = os.path.join(ORACLE_DIR, "libgpu_ref.so")
# The reference tree's location comes from the environment (or the
# --reference-root flag); without it the prebuilt library is used as is.
DEFAULT_REFERENCE_ROOT = os.environ.get("FMHA_REFERENCE_ROOT", "")


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build_oracle(force: bool = False) -> str:
    src = os.path.join(ORACLE_DIR, "fmha_oracle.c")
    if force or _stale(ORACLE_LIB, [src]):
        subprocess.run(
            ["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-std=c11", src, "-lm",
             "-o", ORACLE_LIB + ".tmp"],
            check=True,
        )
        os.replace(ORACLE_LIB + ".tmp", ORACLE_LIB)
    return ORACLE_LIB


def build_gpu_ref(force: bool = False) -> str:
    """nvcc-compile the device oracle for sm_100a (cross-compiles without a GPU)."""
    src = os.path.join(ORACLE_DIR, "gpu_ref.cu")
    if force or _stale(GPU_REF_LIB, [src]):
        nvcc = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
        subprocess.run(
            [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
             "-Xcompiler", "-fPIC", "-shared", "--cudart", "static", src,
             "-o", GPU_REF_LIB + ".tmp"],
            check=True,
        )
        os.replace(GPU_REF_LIB + ".tmp", GPU_REF_LIB)
    return GPU_REF_LIB


def build_reference(force: bool = False, reference_root: str = DEFAULT_REFERENCE_ROOT) -> str | None:
    """Compile the reference CPU oracle; returns the .so path, or None when
    the reference tree is not present (e.g. on the GPU box, which uses the
    prebuilt library)."""
    if not reference_root:
        return REF_LIB if os.path.exists(REF_LIB) else None
    runner = os.path.join(reference_root, "src", "runner")
    srcs = [os.path.join(runner, "cpu_ref.cpp"), os.path.join(runner, "buffers.cpp")]
    if not all(os.path.exists(s) for s in srcs):
        return REF_LIB if os.path.exists(REF_LIB) else None
    entry = os.path.join(ORACLE_DIR, "ref_entry.cpp")
    shim = os.path.join(ORACLE_DIR, "shim", "hip", "hip_runtime.h")
    if force or _stale(REF_LIB, srcs + [entry, shim]):
        os.makedirs(REF_DIR, exist_ok=True)
        subprocess.run(
            ["g++", "-std=c++17", "-O2", "-fopenmp", "-fPIC", "-shared",
             "-I", os.path.join(ORACLE_DIR, "shim"), "-I", runner,
             *srcs, entry, "-o", REF_LIB + ".tmp"],
            check=True,
        )
        os.replace(REF_LIB + ".tmp", REF_LIB)
    return REF_LIB


if __name__ == "__main__":
    force = "--force" in sys.argv
    root = DEFAULT_REFERENCE_ROOT
    if "--reference-root" in sys.argv:
        root = sys.argv[sys.argv.index("--reference-root") + 1]
    print(build_oracle(force))
    print(build_gpu_ref(force))
    print(build_reference(force, root))
