"""Allocation-free entry point (fmha_fwd_d64_bf16_tiles_noalloc).

Some callers must not allocate device memory themselves -- code that runs
where cudaMalloc is refused or would stall the whole device, or a plug-in
whose host framework owns every allocation.  This entry keeps its scratch in
a fixed array inside the library.  The test calls it through the C ABI, twice
in a row on the same inputs, and checks each result against the regular
entry point within the tolerance the other parity tests use (and, since the
same kernel runs, bit for bit).  It also checks the capacity limit.

Collected last on purpose (file name), so a run that stops at the first
failure has already run every other test; it also passes on its own in a
fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import fmha_native_b200 as fm
import oracle as O
from fmha_native_b200 import shard
from fmha_native_b200.synth import Workload, make_inputs

pytestmark = pytest.mark.gpu


def _noalloc_lib():
    lib = fm.load_library()
    lib.fmha_fwd_d64_bf16_tiles_noalloc.argtypes = [
        ctypes.POINTER(fm.FmhaFwdParams), ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    lib.fmha_fwd_d64_bf16_tiles_noalloc.restype = ctypes.c_int
    lib.fmha_fwd_d64_noalloc_status.argtypes = [ctypes.c_void_p]
    lib.fmha_fwd_d64_noalloc_status.restype = ctypes.c_int
    return lib


@pytest.mark.parametrize("causal", [False, True])
def test_noalloc_matches_regular_entry_twice(cuda_device, causal):
    import torch

    lib = _noalloc_lib()
    w = Workload("noalloc", 2, 4, 1000, causal, True)
    q, k, v, _ = make_inputs(w, cuda_device, seed_base=21)
    o_ref, lse_ref = fm.fmha_fwd(q, k, v, causal=causal, return_lse=True)
    torch.cuda.synchronize()
    host_tiles = np.ascontiguousarray(
        shard.tiles_array(shard.plan_blocks(2, 4, 1000, 1000, causal)), dtype=np.int32)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        o = torch.full_like(q, float("nan"))
        lse = torch.full_like(lse_ref, float("nan"))
        params, batch, tq, tk = fm.params_from_tensors(q, k, v, o, lse, "bshd")
        st = lib.fmha_fwd_d64_bf16_tiles_noalloc(
            ctypes.byref(params), batch, int(causal), tq, tk,
            host_tiles.ctypes.data_as(ctypes.c_void_p), host_tiles.shape[0],
            ctypes.c_void_p(stream))
        assert st == fm.FMHA_OK
        assert lib.fmha_fwd_d64_noalloc_status(ctypes.c_void_p(stream)) == fm.FMHA_OK
        v_ = O.compare(o.float().cpu().numpy(), o_ref.float().cpu().numpy(),
                       lse.cpu().numpy(), lse_ref.cpu().numpy())
        assert v_["ref_pass"] and v_["baseline_pass"] and v_["lse_pass"], v_
        assert torch.equal(o.view(torch.int16), o_ref.view(torch.int16))


def test_noalloc_rejects_work_list_beyond_capacity(cuda_device):
    import torch

    lib = _noalloc_lib()
    w = Workload("noalloc", 1, 2, 256, False, False)
    q, k, v, _ = make_inputs(w, cuda_device)
    o = torch.zeros_like(q)
    params, batch, tq, tk = fm.params_from_tensors(q, k, v, o, None, "bshd")
    too_many = np.zeros((16385, 2), np.int32)
    st = lib.fmha_fwd_d64_bf16_tiles_noalloc(ctypes.byref(params), batch, 0, tq, tk,
                                             too_many.ctypes.data_as(ctypes.c_void_p), 16385, None)
    assert st == fm.FMHA_ERR_SCRATCH
    assert b"scratch" in lib.fmha_fwd_d64_error_string(st)
    torch.cuda.synchronize()
    assert int(o.abs().sum().item()) == 0  # nothing was launched


def test_noalloc_varlen_with_lse_matches_regular_entry_twice(cuda_device):
    """Varlen (THD, cu_seqlens on the device) with LSE through the
    allocation-free entry, twice, against the regular varlen entry."""
    import torch

    lib = _noalloc_lib()
    seqs = (300, 17, 1029, 256)
    w = Workload("noalloc-varlen", len(seqs), 4, 0, True, True, layout="thd", varlen_seqs=seqs)
    q, k, v, cu = make_inputs(w, cuda_device, seed_base=23)
    o_ref, lse_ref = fm.fmha_fwd(q, k, v, causal=True, return_lse=True, layout="thd",
                                 cu_seqlens_q=cu, cu_seqlens_k=cu)
    torch.cuda.synchronize()
    host_tiles = np.ascontiguousarray(
        shard.tiles_array(shard.plan_blocks(len(seqs), 4, max(seqs), max(seqs), True, seqs)),
        dtype=np.int32)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        o = torch.full_like(q, float("nan"))
        lse = torch.full_like(lse_ref, float("nan"))
        params, batch, tq, tk = fm.params_from_tensors(q, k, v, o, lse, "thd", cu, cu)
        st = lib.fmha_fwd_d64_bf16_tiles_noalloc(
            ctypes.byref(params), batch, 1, tq, tk, host_tiles.ctypes.data_as(ctypes.c_void_p),
            host_tiles.shape[0], ctypes.c_void_p(stream))
        assert st == fm.FMHA_OK
        assert lib.fmha_fwd_d64_noalloc_status(ctypes.c_void_p(stream)) == fm.FMHA_OK
        assert torch.equal(o.view(torch.int16), o_ref.view(torch.int16))
        assert torch.equal(lse.view(torch.int32), lse_ref.view(torch.int32))


_ALLOC_PROBE = r"""
import ctypes, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
import fmha_native_b200 as fm
from fmha_native_b200 import shard
from fmha_native_b200.synth import Workload, make_inputs
dev = torch.device("cuda:0")
w = Workload("probe", 2, 4, 777, True, True)
q, k, v, _ = make_inputs(w, dev, seed_base=5)
o = torch.empty_like(q)
lse = torch.empty(2, 4, 777, device=dev, dtype=torch.float32)
lib = fm.load_library()
lib.fmha_fwd_d64_bf16_tiles_noalloc.argtypes = [ctypes.POINTER(fm.FmhaFwdParams)] + \
    [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
params, batch, tq, tk = fm.params_from_tensors(q, k, v, o, lse, "bshd")
tiles = np.ascontiguousarray(shard.tiles_array(shard.plan_blocks(2, 4, 777, 777, True)), np.int32)
def call():
    st = lib.fmha_fwd_d64_bf16_tiles_noalloc(ctypes.byref(params), batch, 1, tq, tk,
        tiles.ctypes.data_as(ctypes.c_void_p), tiles.shape[0], None)
    assert st == 0, st
call()                      # first call: module load + scratch address
torch.cuda.synchronize()
free0, _ = torch.cuda.mem_get_info()
for _ in range(4):
    call()
torch.cuda.synchronize()
free1, _ = torch.cuda.mem_get_info()
print("FREE", free0, free1)
"""


def test_noalloc_allocates_no_device_memory(cuda_device):
    """In a fresh process: after the first call (which loads the kernels and
    resolves the scratch address), further calls leave the device's free
    memory unchanged to the byte -- nothing is allocated per call."""
    import os
    import subprocess
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _ALLOC_PROBE, repo], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("FREE")][-1]
    _, free0, free1 = line.split()
    assert int(free0) == int(free1), line
