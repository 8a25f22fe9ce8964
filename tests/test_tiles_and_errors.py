"""GPU tests of the work-list entry (multi-GPU sharding emulated on one GPU)
and of the bounded-wait error path.

* Running a problem as several disjoint tile lists (what several ranks do)
  writes exactly the bits of the one-launch result.
* The timeout path: a test hook makes the producer withhold one K/V tile, the
  device waits run out after a short limit, the kernel frees its resources and
  returns, the host reads FMHA_ERR_TIMEOUT, and the context stays usable (the
  next normal launch is correct).  No fault, trap or endless loop is involved.
"""
from __future__ import annotations

import numpy as np
import pytest

import fmha_native_b200 as fm
from fmha_native_b200 import shard
from fmha_native_b200.synth import Workload, make_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("causal,world", [(True, 2), (True, 3), (False, 4)])
def test_tile_partition_reproduces_full_launch(cuda_device, causal, world):
    import torch

    w = Workload("t", 2, 4, 1100, causal, True)
    q, k, v, _ = make_inputs(w, cuda_device, seed_base=11)
    o_full, lse_full = fm.fmha_fwd(q, k, v, causal=causal, return_lse=True)
    o = torch.full_like(q, float("nan"))
    lse = torch.full_like(lse_full, float("nan"))
    parts = shard.partition(shard.plan_blocks(2, 4, 1100, 1100, causal), world)
    for part in parts:
        tiles = torch.from_numpy(shard.tiles_array(part)).to(cuda_device)
        fm.fmha_fwd(q, k, v, causal=causal, return_lse=True, out=o, lse_out=lse, tiles=tiles)
    torch.cuda.synchronize()
    assert torch.equal(o.view(torch.int16), o_full.view(torch.int16))
    assert torch.equal(lse, lse_full)


def test_empty_tile_list_is_a_no_op(cuda_device):
    import torch

    w = Workload("t", 1, 2, 256, False, False)
    q, k, v, _ = make_inputs(w, cuda_device)
    o = torch.zeros_like(q)
    tiles = torch.zeros(0, 2, dtype=torch.int32, device=cuda_device)
    fm.fmha_fwd(q, k, v, out=o, tiles=tiles)
    torch.cuda.synchronize()
    assert int(o.abs().sum().item()) == 0


def test_pipeline_timeout_reports_and_recovers(cuda_device):
    import torch

    lib = fm.load_library()
    w = Workload("t", 1, 2, 512, False, False)
    q, k, v, _ = make_inputs(w, cuda_device, seed_base=5)
    good = fm.fmha_fwd(q, k, v)
    torch.cuda.synchronize()
    assert fm.status() == fm.FMHA_OK
    try:
        lib.fmha_fwd_d64_set_wait_limit_ns(20_000_000)  # 20 ms
        lib.fmha_fwd_d64_debug_set_stall(1)
        fm.fmha_fwd(q, k, v)
        assert fm.status() == fm.FMHA_ERR_TIMEOUT
    finally:
        lib.fmha_fwd_d64_debug_set_stall(0)
        lib.fmha_fwd_d64_set_wait_limit_ns(0)
    again = fm.fmha_fwd(q, k, v)
    torch.cuda.synchronize()
    assert fm.status() == fm.FMHA_OK
    assert torch.equal(again.view(torch.int16), good.view(torch.int16))
