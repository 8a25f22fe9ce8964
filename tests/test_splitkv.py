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
    assert shard.choose_splits(314) == 1
    assert shard.choose_splits(39) == 8
    assert shard.choose_splits(100) == 3
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
