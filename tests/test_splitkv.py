"""Split-KV (row f1): every query block split into KV ranges, partial O/LSE
merged by the combine kernel.  Checked against the oracle with the parity
rules and against the one-pass kernel; CPU checks of the split planner."""
from __future__ import annotations

import numpy as np
import pytest

import fmha_native_b200 as fm
import oracle as O
from fmha_native_b200 import shard
from harness import D, from_device_bf16

pytestmark = []


def test_choose_splits():
    assert shard.choose_splits(314) == 2
    assert shard.choose_splits(39) == 8
    assert shard.choose_splits(79) == 8
    assert shard.choose_splits(100) == 6
    assert shard.choose_splits(600) == 1
    assert shard.choose_splits(10000) == 1


@pytest.mark.gpu
@pytest.mark.parametrize("causal,splits,S", [(True, 2, 1100), (True, 5, 1500), (False, 3, 700),
                                             (True, 8, 300)])
def test_splitkv_matches_oracle(cuda_device, causal, splits, S):
    import torch

    from fmha_native_b200.synth import Workload, make_inputs

    B, H = 1, 3
    w = Workload("s", B, H, S, causal, True)
    q, k, v, _ = make_inputs(w, cuda_device, seed_base=31)
    o1, l1 = fm.fmha_fwd(q, k, v, causal=causal, return_lse=True)
    tiles = torch.from_numpy(shard.tiles_array(shard.plan_blocks(B, H, S, S, causal))).to(cuda_device)
    o2, l2 = fm.fmha_fwd(q, k, v, causal=causal, return_lse=True, tiles=tiles, num_splits=splits)
    torch.cuda.synchronize()
    assert fm.status() == fm.FMHA_OK

    def bits(t):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)

    st = (H * D, D, S * H * D)
    o_ref, lse_ref = O.oracle_fwd(bits(q), bits(k), bits(v), batch=B, nhead_q=H, nhead_k=H,
                                  seqlen_q=S, seqlen_k=S, causal=causal, strides_q=st,
                                  strides_k=st, strides_v=st, out_shape=(B, S, H, D), strides_o=st)
    v2 = O.compare(O.bf16_bits_to_f32(bits(o2)).reshape(B, S, H, D), o_ref, l2.cpu().numpy(), lse_ref)
    assert v2["baseline_pass"] and v2["lse_pass"], v2
    assert (o2.float() - o1.float()).abs().max().item() <= 2 ** -7
    assert (l2 - l1).abs().max().item() <= 1e-4


@pytest.mark.gpu
def test_splitkv_rejects_small_workspace(cuda_device):
    import torch

    from fmha_native_b200.synth import Workload, make_inputs

    w = Workload("s", 1, 2, 512, True, False)
    q, k, v, _ = make_inputs(w, cuda_device)
    o = torch.empty_like(q)
    params, batch, tq, tk = fm.params_from_tensors(q, k, v, o, None, "bshd")
    tiles = torch.from_numpy(shard.tiles_array(shard.plan_blocks(1, 2, 512, 512, True))).to(cuda_device)
    ws = torch.empty(16, device=cuda_device)
    st = fm.call_tiles_splitkv(params, batch, True, tiles.data_ptr(), tiles.shape[0], 4,
                               ws.data_ptr(), 64)
    assert st == fm.FMHA_ERR_ARG


# ---------------------------------------------------------------- work items
def _check_items_cover(blocks, items):
    """Every block's KV range is covered exactly once: one whole item, or
    consecutive partial items tiling [0, n_kv)."""
    n_kv = {(b[0], b[1]): max(0, int(round(b[2] - shard.BLOCK_OVERHEAD))) for b in blocks}
    seen = {}
    prev = None
    for it in items:
        key = (it[0], it[1])
        assert key in n_kv
        if it[3] < 0:
            assert key not in seen
            seen[key] = "whole"
        else:
            if key in seen:
                assert seen[key] != "whole" and prev is not None and prev[:2] == it[:2], it
                assert seen[key] == it[2], it  # contiguous
            else:
                assert it[2] == 0, it
            seen[key] = it[3]
        prev = it
    for key, n in n_kv.items():
        assert key in seen, key
        assert seen[key] == "whole" or seen[key] == n, (key, seen[key], n)


@pytest.mark.parametrize("B,H,S,causal,world", [(1, 2, 40000, True, 8), (1, 2, 40000, True, 1),
                                                (32, 32, 4096, True, 8), (2, 3, 5000, False, 4)])
def test_plan_items_covers_every_block_once(B, H, S, causal, world):
    blocks = shard.plan_blocks(B, H, S, S, causal)
    for part in shard.partition(blocks, world):
        items = shard.plan_items(part)
        _check_items_cover(part, items)


def test_plan_items_fills_one_wave():
    """c5a, rank 0 of 8: the pieces fit in one wave of CTA slots, no piece
    is longer than the smallest cap that does, and the largest comes first."""
    blocks = shard.plan_blocks(1, 2, 40000, 40000, True)
    part = shard.partition(blocks, 8)[0]
    slots = 2 * 148
    items = shard.plan_items(part, slots=slots)
    assert len(items) <= slots
    n_kv = [max(0, int(round(b[2] - shard.BLOCK_OVERHEAD))) for b in part]
    sizes = [(it[3] - it[2]) if it[3] >= 0 else n_kv[[(b[0], b[1]) for b in part].index(
        (it[0], it[1]))] for it in items]
    cap = max(sizes)
    # one tile less per piece would need more CTAs than the wave has
    assert sum(-(-n // (cap - 1)) for n in n_kv if n > 0) > slots
    assert sizes[0] == cap
    # two waves: about twice the pieces, each about half as long
    items2 = shard.plan_items(part, slots=slots, waves=2.0)
    assert slots < len(items2) <= 2 * slots


def test_plan_items_keeps_short_blocks_whole():
    """A share whose blocks already fit the slots is not split at all."""
    blocks = shard.plan_blocks(32, 32, 4096, 4096, True)
    part = shard.partition(blocks, 8)[0]
    assert all(it[3] == -1 for it in shard.plan_items(part))


@pytest.mark.gpu
@pytest.mark.parametrize("causal,S,slots,varlen", [(True, 3000, 40, False),
                                                   (False, 1500, 1000, False),
                                                   (True, 2000, 60, True)])
def test_items_match_oracle(cuda_device, causal, S, slots, varlen):
    """Small problems planned for four waves of CTA slots, so that most
    blocks are split into several partial items (and some stay whole)."""
    import torch

    from fmha_native_b200.synth import Workload, make_inputs

    B, H = (3, 2) if varlen else (1, 3)
    seqs = (S, S // 3, S // 2 + 77) if varlen else None
    w = Workload("s", B, H, S, causal, True, layout="thd" if varlen else "bshd",
                 varlen_seqs=seqs)
    q, k, v, cu = make_inputs(w, cuda_device, seed_base=57)
    layout = w.layout
    o1, l1 = fm.fmha_fwd(q, k, v, causal=causal, return_lse=True, layout=layout,
                         cu_seqlens_q=cu, cu_seqlens_k=cu)
    blocks = shard.plan_blocks(B, H, S, S, causal, seqs)
    items = shard.plan_items(blocks, slots=slots, waves=4.0)
    assert any(it[3] >= 0 for it in items)
    assert any(it[3] < 0 for it in items) or slots >= 1000
    it_d = torch.from_numpy(shard.items_array(items)).to(cuda_device)
    o2, l2 = fm.fmha_fwd(q, k, v, causal=causal, return_lse=True, layout=layout,
                         cu_seqlens_q=cu, cu_seqlens_k=cu, items=it_d)
    torch.cuda.synchronize()
    assert fm.status() == fm.FMHA_OK

    def bits(t):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)

    if varlen:
        T = w.tokens()
        st = (H * D, D, 0)
        ss = np.concatenate([[0], np.cumsum(seqs)]).astype(np.int32)
        o_ref, lse_ref = O.oracle_fwd(bits(q), bits(k), bits(v), batch=B, nhead_q=H, nhead_k=H,
                                      seqlen_q=max(seqs), seqlen_k=max(seqs), causal=causal,
                                      strides_q=st, strides_k=st, strides_v=st,
                                      out_shape=(T, H, D), strides_o=st, seqstart_q=ss,
                                      seqstart_k=ss, total_q=T)
        shape = (T, H, D)
    else:
        st = (H * D, D, S * H * D)
        o_ref, lse_ref = O.oracle_fwd(bits(q), bits(k), bits(v), batch=B, nhead_q=H, nhead_k=H,
                                      seqlen_q=S, seqlen_k=S, causal=causal, strides_q=st,
                                      strides_k=st, strides_v=st, out_shape=(B, S, H, D),
                                      strides_o=st)
        shape = (B, S, H, D)
    v2 = O.compare(O.bf16_bits_to_f32(bits(o2)).reshape(shape), o_ref, l2.cpu().numpy(), lse_ref)
    assert v2["baseline_pass"] and v2["lse_pass"], v2
    assert (o2.float() - o1.float()).abs().max().item() <= 2 ** -7
    assert (l2 - l1).abs().max().item() <= 1e-4


@pytest.mark.gpu
def test_items_rejects_small_workspace(cuda_device):
    import torch

    from fmha_native_b200.synth import Workload, make_inputs

    w = Workload("s", 1, 2, 512, True, False)
    q, k, v, _ = make_inputs(w, cuda_device)
    o = torch.empty_like(q)
    params, batch, tq, tk = fm.params_from_tensors(q, k, v, o, None, "bshd")
    items = shard.plan_items(shard.plan_blocks(1, 2, 512, 512, True), slots=100)
    it_d = torch.from_numpy(shard.items_array(items)).to(cuda_device)
    ws = torch.empty(16, device=cuda_device)
    assert fm.call_items(params, batch, True, it_d.data_ptr(), it_d.shape[0], ws.data_ptr(),
                         64) == fm.FMHA_ERR_ARG
