"""GPU parity on the five north-star configurations, at full size, on the
exact seeded inputs bench.py times (fmha_native_b200.synth.make_inputs).

Oracle: the device restatement of the reference's GPU reference
(oracle/gpu_ref.cu, src/runner/gpu_ref.cpp:12-126), itself pinned to the C
restatement of cpu_ref.cpp (tests/test_gpu_ref.py) on every reference config
and on row samples of these configurations.  Bars (the north star's, not
loosened): O max-abs <= 2e-2 and rel-L2 <= 5e-3 against the fp32 oracle,
LSE max |d| <= 1e-3 with -inf == -inf.

Besides the plain entries, C5a also runs through the split-KV path and C5b
through the LPT work lists, exactly as `bench.py --shard` runs them on 8
GPUs (here the 8 ranks' lists run one after another on one GPU, covering
every query block once).  Each case prints its verdict (pytest -s).
"""
from __future__ import annotations

import json

import pytest

import fmha_native_b200 as fm
import oracle as O
from fmha_native_b200 import shard
from fmha_native_b200.synth import WORKLOADS, make_inputs

pytestmark = pytest.mark.gpu

BASELINE_KEYS = ["c1", "c2", "c3", "c4", "c4c", "c5a", "c5b"]


def _run(w, dev, mode: str = "entry", world: int = 8):
    import torch

    q, k, v, cu = make_inputs(w, dev, seed_base=0)
    o = torch.full_like(q, float("nan"))
    lse = None
    if w.lse:
        shape = (w.heads, w.tokens()) if w.varlen_seqs else (w.batch, w.heads, w.seqlen)
        lse = torch.full(shape, float("nan"), device=dev, dtype=torch.float32)
    if mode == "entry":
        fm.fmha_fwd(q, k, v, causal=w.causal, layout=w.layout, cu_seqlens_q=cu,
                    cu_seqlens_k=cu, out=o, lse_out=lse, return_lse=lse is not None)
    else:
        blocks = shard.plan_blocks(w.batch, w.heads, w.seqlen, w.seqlen, w.causal, w.varlen_seqs)
        for part in shard.partition(blocks, world):
            tiles = torch.from_numpy(shard.tiles_array(part)).to(dev)
            if mode == "items":
                items = torch.from_numpy(shard.items_array(shard.plan_items(part))).to(dev)
                fm.fmha_fwd(q, k, v, causal=w.causal, layout=w.layout, cu_seqlens_q=cu,
                            cu_seqlens_k=cu, out=o, lse_out=lse, return_lse=lse is not None,
                            items=items)
                continue
            splits = shard.choose_splits(tiles.shape[0]) if mode == "splitkv" else 1
            fm.fmha_fwd(q, k, v, causal=w.causal, layout=w.layout, cu_seqlens_q=cu,
                        cu_seqlens_k=cu, out=o, lse_out=lse, return_lse=lse is not None,
                        tiles=tiles, num_splits=splits)
    torch.cuda.synchronize()
    assert fm.status() == fm.FMHA_OK
    o_ref, lse_ref = O.gpu_ref_fwd(q, k, v, layout=w.layout, causal=w.causal, seqstart_q=cu,
                                   seqstart_k=cu, with_lse=lse is not None)
    torch.cuda.synchronize()
    verdict = O.compare_device(o.float(), o_ref, lse, lse_ref)
    verdict["config"] = w.name
    verdict["path"] = mode
    print(json.dumps(verdict))
    return verdict


def _assert(v):
    assert v["nonfinite"] == 0, v
    assert v["max_abs"] <= O.BASE_TOL_MAX_ABS, v
    assert v["rel_l2"] <= O.BASE_TOL_REL_L2, v
    if "lse_pass" in v:
        assert v["lse_pass"], v


@pytest.mark.parametrize("key", BASELINE_KEYS)
def test_baseline_config_entry(cuda_device, key):
    _assert(_run(WORKLOADS[key], cuda_device))


@pytest.mark.parametrize("key", ["c5b_gqa4", "c5b_mqa", "c2_gqa4"])
def test_grouped_kv_config_entry(cuda_device, key):
    """c5b / c2 shapes with 4 query heads per K/V head and with one K/V head
    (the reference's GQA/MQA ratios), full size, against the device oracle."""
    _assert(_run(WORKLOADS[key], cuda_device))


def test_c5a_splitkv_shards(cuda_device):
    """B1 H2 S40000 causal: each of 8 ranks' LPT shares through uniform
    split-KV (shard.choose_splits), as bench.py --shard --gpus 8."""
    _assert(_run(WORKLOADS["c5a"], cuda_device, mode="splitkv"))


def test_c5a_item_shards(cuda_device):
    """B1 H2 S40000 causal: each of 8 ranks' LPT shares cut into one wave of
    work items (shard.plan_items), as bench.py --shard --items --gpus 8."""
    _assert(_run(WORKLOADS["c5a"], cuda_device, mode="items"))


def test_c5b_lpt_shards(cuda_device):
    """B32 H32 S4096 causal: the 8 ranks' LPT work lists, as bench.py --shard."""
    _assert(_run(WORKLOADS["c5b"], cuda_device, mode="tiles"))
