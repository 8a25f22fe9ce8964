"""In-tree build of the sm_100a CUDA library (``libfmha_b200.so``).

The library is compiled with nvcc directly (no JIT cache) so the built
``.so`` sits next to this file and travels with the source tree.  Usage::

    python -m fmha_native_b200.build          # build if sources are newer
    python -m fmha_native_b200.build --force  # always rebuild
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_PATH = os.path.join(PKG_DIR, "libfmha_b200.so")

SOURCES = [os.path.join(CSRC, "fmha_fwd_kernel.cu")]
DEPS = SOURCES + [
    os.path.join(CSRC, "sm100_ptx.cuh"),
    os.path.join(REPO_DIR, "include", "fmha_fwd.h"),
]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_library(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> str:
    """Compile ``libfmha_b200.so`` for sm_100a; returns its path."""
    if not force and not extra_flags and not _stale(LIB_PATH, DEPS):
        return LIB_PATH
    cmd = [
        nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC", "-shared", "--cudart", "static",
        "-I", os.path.join(REPO_DIR, "include"),
        *(extra_flags or []),
        *SOURCES, "-o", LIB_PATH + ".tmp",
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


TRACE_LIB_PATH = os.path.join(PKG_DIR, "libfmha_b200_trace.so")


def build_trace_library(force: bool = False) -> str:
    """The same kernel source with -DFMHA_TRACE: ``libfmha_b200_trace.so``,
    which adds the per-role timeline stamps (include/fmha_fwd_trace.h)."""
    deps = DEPS + [os.path.join(REPO_DIR, "include", "fmha_fwd_trace.h")]
    if not force and not _stale(TRACE_LIB_PATH, deps):
        return TRACE_LIB_PATH
    cmd = [
        nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-DFMHA_TRACE",
        "-Xcompiler", "-fPIC", "-shared", "--cudart", "static",
        "-I", os.path.join(REPO_DIR, "include"),
        *SOURCES, "-o", TRACE_LIB_PATH + ".tmp",
    ]
    subprocess.run(cmd, check=True)
    os.replace(TRACE_LIB_PATH + ".tmp", TRACE_LIB_PATH)
    return TRACE_LIB_PATH


CLI_SRC = os.path.join(PKG_DIR, "host", "bench_fmha_fwd.cpp")
CLI_PATH = os.path.join(PKG_DIR, "bench_fmha_fwd")


def build_cli(force: bool = False) -> str:
    """C++17 bench_fmha_fwd CLI over the C ABI (links libfmha_b200.so)."""
    lib = build_library()
    if not force and not _stale(CLI_PATH, [CLI_SRC, lib, os.path.join(REPO_DIR, "include", "fmha_fwd.h")]):
        return CLI_PATH
    cuda = os.path.dirname(os.path.dirname(nvcc_path()))
    subprocess.run(["g++", "-std=c++17", "-O2", "-I", os.path.join(REPO_DIR, "include"),
                    "-I", os.path.join(cuda, "include"), CLI_SRC, "-o", CLI_PATH,
                    "-L", PKG_DIR, "-lfmha_b200", f"-Wl,-rpath,$ORIGIN",
                    "-L", os.path.join(cuda, "lib64"), "-lcudart"], check=True)
    return CLI_PATH


TEST_SRC = os.path.join(REPO_DIR, "tests", "native", "unit_kernels.cu")
TEST_LIB = os.path.join(REPO_DIR, "tests", "native", "libfmha_unit.so")


def build_test_lib(force: bool = False) -> str | None:
    """Test-only library exposing single device helpers of the kernel
    (tests/native/unit_kernels.cu); skipped when the tests tree is absent."""
    if not os.path.exists(TEST_SRC):
        return None
    deps = [TEST_SRC, os.path.join(CSRC, "sm100_ptx.cuh")]
    if not force and not _stale(TEST_LIB, deps):
        return TEST_LIB
    subprocess.run([nvcc_path(), *ARCH_FLAGS, "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                    "-shared", "--cudart", "static", TEST_SRC, "-o", TEST_LIB + ".tmp"],
                   check=True)
    os.replace(TEST_LIB + ".tmp", TEST_LIB)
    return TEST_LIB


CPP_TEST_SRC = os.path.join(REPO_DIR, "tests", "cpp", "test_fmha_fwd_d64.cpp")
CPP_TEST_BIN = os.path.join(REPO_DIR, "tests", "cpp", "test_fmha_fwd_d64")
ORACLE_C = os.path.join(REPO_DIR, "oracle", "fmha_oracle.c")


def build_cpp_tests(force: bool = False) -> str | None:
    """The C++17 gtest-format parity suite (tests/cpp) over the C ABI, linked
    with the C oracle; skipped when the tests tree is absent."""
    if not os.path.exists(CPP_TEST_SRC):
        return None
    lib = build_library()
    cpp_dir = os.path.dirname(CPP_TEST_SRC)
    deps = [CPP_TEST_SRC, ORACLE_C, lib, os.path.join(cpp_dir, "mini_gtest.h"),
            os.path.join(cpp_dir, "test_cases.inc"), os.path.join(REPO_DIR, "include", "fmha_fwd.h")]
    if not force and not _stale(CPP_TEST_BIN, deps):
        return CPP_TEST_BIN
    cuda = os.path.dirname(os.path.dirname(nvcc_path()))
    obj = CPP_TEST_BIN + ".oracle.o"
    subprocess.run(["gcc", "-O2", "-fopenmp", "-std=c11", "-c", ORACLE_C, "-o", obj], check=True)
    subprocess.run(["g++", "-std=c++17", "-O2", "-fopenmp", "-I", os.path.join(REPO_DIR, "include"),
                    "-I", os.path.join(cuda, "include"), CPP_TEST_SRC, obj,
                    "-o", CPP_TEST_BIN + ".tmp", "-L", PKG_DIR, "-lfmha_b200",
                    f"-Wl,-rpath,{PKG_DIR}", "-Wl,-rpath,$ORIGIN/../../fmha_native_b200",
                    "-L", os.path.join(cuda, "lib64"), "-lcudart", "-lm"], check=True)
    os.replace(CPP_TEST_BIN + ".tmp", CPP_TEST_BIN)
    os.remove(obj)
    return CPP_TEST_BIN


if __name__ == "__main__":
    build_library(force="--force" in sys.argv, verbose="-v" in sys.argv)
    build_cli(force="--force" in sys.argv)
    build_trace_library(force="--force" in sys.argv)
    build_test_lib(force="--force" in sys.argv)
    build_cpp_tests(force="--force" in sys.argv)
    print(LIB_PATH)
