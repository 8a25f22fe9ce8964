"""CPU tests of the C-ABI boundary: every function declared in
include/fmha_fwd.h is exported by the built library, the ctypes mirror of
FmhaFwdParams has the C layout, and host-side argument validation (which
runs before any CUDA call) rejects what the reference's callers could pass
but the TMA data path cannot serve."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

import fmha_native_b200 as fm

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "fmha_fwd.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fmha_fwd_\w+)\s*\(", text)))


def test_header_declares_the_four_reference_entries():
    names = declared_functions()
    for n in ("fmha_fwd_d64_bf16_msk0", "fmha_fwd_d64_bf16_msk1",
              "fmha_fwd_d64_bf16_msk0_varlen", "fmha_fwd_d64_bf16_msk1_varlen"):
        assert n in names


def test_library_exports_every_declared_symbol():
    assert os.path.exists(fm.LIB_PATH), "build the library first"
    out = subprocess.run(["nm", "-D", "--defined-only", fm.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(\w+)", out))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing


def test_library_loads_without_gpu():
    lib = fm.load_library()
    assert lib.fmha_fwd_d64_error_string(fm.FMHA_ERR_ARG) == b"invalid argument"


def test_params_layout_matches_c(tmp_path):
    src = tmp_path / "layout.c"
    fields = [f[0] for f in fm.FmhaFwdParams._fields_]
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "fmha_fwd.h"\nint main(void){\n'
                   + "".join(f'printf("%zu\\n", offsetof(FmhaFwdParams, {f}));\n' for f in fields)
                   + 'printf("%zu\\n", sizeof(FmhaFwdParams));\nreturn 0;}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)],
                   check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    want = [getattr(fm.FmhaFwdParams, f).offset for f in fields] + [ctypes.sizeof(fm.FmhaFwdParams)]
    assert got == want


def _valid_params():
    p = fm.FmhaFwdParams()
    base = 1 << 20  # fake, 16-byte aligned device addresses (never dereferenced)
    p.q, p.k, p.v, p.o = base, base * 2, base * 3, base * 4
    p.seqlen_q = p.seqlen_k = 256
    p.nhead_q = p.nhead_k = 2
    p.scale = 0.18
    for t in "qkvo":
        setattr(p, f"stride_{t}", 64)
        setattr(p, f"nhead_stride_{t}", 256 * 64)
        setattr(p, f"batch_stride_{t}", 2 * 256 * 64)
    return p


@pytest.mark.parametrize("mutate", [
    lambda p: setattr(p, "q", None),
    lambda p: setattr(p, "o", (1 << 20) + 2),            # misaligned output
    lambda p: setattr(p, "nhead_k", 3),                   # nhead_q % nhead_k != 0
    lambda p: setattr(p, "stride_k", 60),                 # not a 16-byte multiple
    lambda p: setattr(p, "nhead_stride_q", 4),            # not a 16-byte multiple
    lambda p: setattr(p, "seqlen_q", -1),
])
def test_invalid_arguments_rejected_on_host(mutate):
    p = _valid_params()
    mutate(p)
    assert fm.call_entry(p, 1, False, False) == fm.FMHA_ERR_ARG


def test_varlen_entry_needs_seqstart():
    p = _valid_params()
    assert fm.call_entry(p, 1, True, True, 256, 256) == fm.FMHA_ERR_ARG


def test_dense_entry_rejects_seqstart():
    p = _valid_params()
    p.seqstart_q = 1 << 20
    lib = fm.load_library()
    assert lib.fmha_fwd_d64_bf16_msk0(ctypes.byref(p), 1, None) == fm.FMHA_ERR_ARG


def test_null_params_rejected():
    lib = fm.load_library()
    assert lib.fmha_fwd_d64_bf16(None, 1, 0, 0, 0, None) == fm.FMHA_ERR_ARG


def test_valid_call_without_gpu_returns_a_status():
    """A well-formed call on a machine without a usable sm_100 device goes
    through validation and tensor-map encoding and returns FMHA_ERR_DEVICE
    (never crashes); on a B200 this test is skipped (it would launch)."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present: this call would launch on fake pointers")
    p = _valid_params()
    for causal in (False, True):
        assert fm.call_entry(p, 1, causal, False) == fm.FMHA_ERR_DEVICE
    tiles = (ctypes.c_int32 * 4)(0, 0, 1, 1)
    lib = fm.load_library()
    lib.fmha_fwd_d64_bf16_tiles_noalloc.argtypes = [
        ctypes.POINTER(fm.FmhaFwdParams), ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    assert lib.fmha_fwd_d64_bf16_tiles_noalloc(ctypes.byref(p), 1, 0, 0, 0,
                                               ctypes.cast(tiles, ctypes.c_void_p), 2,
                                               None) == fm.FMHA_ERR_DEVICE
    bad = (ctypes.c_int32 * 2)(5, 0)  # (batch, head) index outside B1 H2
    assert lib.fmha_fwd_d64_bf16_tiles_noalloc(ctypes.byref(p), 1, 0, 0, 0,
                                               ctypes.cast(bad, ctypes.c_void_p), 1,
                                               None) == fm.FMHA_ERR_ARG
