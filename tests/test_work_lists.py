"""Work-list validation (GPU).

* Malformed work-list entries (a (batch, head) index or query block outside
  the problem, an inverted KV range) are skipped without any memory access:
  O and LSE are views inside a larger canary-filled allocation, and every
  byte outside the listed valid blocks keeps its canary.  The reference grid
  can never name a block outside the problem (src/fused/kernel.cpp:55-99); a
  list must not be able to either.
* The allocation-free entry rejects the same entries on the host with
  FMHA_ERR_ARG before anything is queued.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import fmha_native_b200 as fm
from fmha_native_b200 import shard
from fmha_native_b200.synth import Workload, make_inputs

pytestmark = pytest.mark.gpu

CANARY = 0x7FA1  # a bf16 NaN pattern no kernel result can produce


def _bits(t):
    import torch

    return t.contiguous().view(torch.int16)


def _canary_views(q, lse_shape, dev, pad=4096):
    """O and LSE as views into the middle of canary-filled buffers."""
    import torch

    n = q.numel()
    obuf = torch.full((n + 2 * pad,), CANARY, dtype=torch.int16, device=dev)
    o = obuf[pad:pad + n].view(torch.bfloat16).view(q.shape)
    nl = int(np.prod(lse_shape))
    lbuf = torch.full((nl + 2 * pad,), -12345.0, dtype=torch.float32, device=dev)
    lse = lbuf[pad:pad + nl].view(lse_shape)
    return obuf, o, lbuf, lse


@pytest.mark.parametrize("causal", [False, True])
def test_malformed_tile_entries_touch_nothing(cuda_device, causal):
    import torch

    B, H, S = 2, 3, 520
    w = Workload("t", B, H, S, causal, True)
    q, k, v, _ = make_inputs(w, cuda_device, seed_base=9)
    o_full, lse_full = fm.fmha_fwd(q, k, v, causal=causal, return_lse=True)
    mb = -(-S // 128)
    good = [(1, 0), (4, 3), (5, mb - 1)]
    bad = [(-1, 0), (B * H, 0), (0, -1), (0, mb), (2**30, 2), (3, 2**30), (-2**31, -2**31)]
    lst = []
    for g_, b_ in zip(good + good, bad):
        lst += [g_, b_]
    tiles = torch.tensor(lst, dtype=torch.int32, device=cuda_device)
    obuf, o, lbuf, lse = _canary_views(q, lse_full.shape, cuda_device)
    fm.fmha_fwd(q, k, v, causal=causal, return_lse=True, out=o, lse_out=lse, tiles=tiles)
    torch.cuda.synchronize()
    assert fm.status() == fm.FMHA_OK
    pad = 4096
    assert bool((obuf[:pad] == CANARY).all()) and bool((obuf[-pad:] == CANARY).all())
    assert bool((lbuf[:pad] == -12345.0).all()) and bool((lbuf[-pad:] == -12345.0).all())
    # Listed valid blocks equal the full launch; every other row kept its canary.
    written = torch.zeros(B, S, H, dtype=torch.bool, device=cuda_device)
    for hb, m in good:
        b_, h_ = divmod(hb, H)
        written[b_, m * 128:(m + 1) * 128, h_] = True
    ob = _bits(o)
    assert torch.equal(ob[written], _bits(o_full)[written])
    assert bool((ob[~written] == CANARY).all())
    lw = written.permute(0, 2, 1)
    assert torch.equal(lse[lw], lse_full[lw])
    assert bool((lse[~lw] == -12345.0).all())


def test_malformed_items_touch_nothing(cuda_device):
    import torch

    B, H, S = 1, 2, 700
    w = Workload("i", B, H, S, True, True)
    q, k, v, _ = make_inputs(w, cuda_device, seed_base=13)
    o_full, lse_full = fm.fmha_fwd(q, k, v, causal=True, return_lse=True)
    items = [(1, 5, 0, 3), (1, 5, 3, 6),          # block (h1, m5) split in two
             (0, 2, 0, -1),                         # whole block
             (2, 0, 0, -1), (0, -1, 0, -1), (-5, 1, 0, 2), (0, 9, 0, -1),
             (0, 1, 4, 2), (0, 1, -3, 1)]           # malformed
    it = torch.tensor(items, dtype=torch.int32, device=cuda_device)
    obuf, o, lbuf, lse = _canary_views(q, lse_full.shape, cuda_device)
    fm.fmha_fwd(q, k, v, causal=True, return_lse=True, out=o, lse_out=lse, items=it)
    torch.cuda.synchronize()
    assert fm.status() == fm.FMHA_OK
    pad = 4096
    assert bool((obuf[:pad] == CANARY).all()) and bool((obuf[-pad:] == CANARY).all())
    assert bool((lbuf[:pad] == -12345.0).all()) and bool((lbuf[-pad:] == -12345.0).all())
    written = torch.zeros(B, S, H, dtype=torch.bool, device=cuda_device)
    written[0, 5 * 128:6 * 128, 1] = True
    written[0, 2 * 128:3 * 128, 0] = True
    ob = _bits(o)
    assert bool((ob[~written] == CANARY).all())
    assert (o.float()[written] - o_full.float()[written]).abs().max().item() <= 2 ** -7
    lw = written.permute(0, 2, 1)
    assert (lse[lw] - lse_full[lw]).abs().max().item() <= 1e-4
    assert bool((lse[~lw] == -12345.0).all())


def test_noalloc_rejects_malformed_entries(cuda_device):
    import torch

    lib = fm.load_library()
    lib.fmha_fwd_d64_bf16_tiles_noalloc.argtypes = [
        ctypes.POINTER(fm.FmhaFwdParams), ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    w = Workload("n", 1, 2, 300, False, False)
    q, k, v, _ = make_inputs(w, cuda_device)
    o = torch.zeros_like(q)
    params, batch, tq, tk = fm.params_from_tensors(q, k, v, o, None, "bshd")
    for bad in ([(0, 0), (2, 0)], [(0, 3)], [(-1, 0)], [(1, -1)]):
        arr = np.ascontiguousarray(np.asarray(bad, np.int32))
        st = lib.fmha_fwd_d64_bf16_tiles_noalloc(ctypes.byref(params), batch, 0, tq, tk,
                                                 arr.ctypes.data_as(ctypes.c_void_p),
                                                 arr.shape[0], None)
        assert st == fm.FMHA_ERR_ARG, bad
    torch.cuda.synchronize()
    assert int(o.abs().sum().item()) == 0  # nothing was launched
