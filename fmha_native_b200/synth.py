"""Seeded synthetic inputs for the north-star workloads (no dataset exists for
this path; the reference benchmarks on random tensors too,
src/bench_fmha_fwd.cpp:128-129).

Values are generated in fp32 by torch's counter-based generator (one seed per
tensor, so Q/K/V are independent of generation order), then rounded to bf16.
The oracle always consumes the exact bf16 bits handed to the kernel, so
parity never depends on the generator.
"""
from __future__ import annotations

import dataclasses
from typing import Optional, Sequence

import numpy as np


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    heads: int
    seqlen: int
    causal: bool
    lse: bool
    dist: str = "normal"          # "normal" N(0,1) or "uniform" U[-1,1)
    layout: str = "bshd"          # dense "bshd"; varlen "thd"
    varlen_seqs: Optional[Sequence[int]] = None
    kv_heads: int = 0             # K/V heads (GQA/MQA); 0 = heads

    @property
    def heads_k(self) -> int:
        return self.kv_heads or self.heads

    def flops(self) -> float:
        """Reference FLOP convention (src/bench_fmha_fwd.cpp:225-226):
        4*B*H*Sq*Sk*64, x0.5 causal; varlen sums per-sequence Sq*Sk."""
        if self.varlen_seqs:
            f = 4.0 * self.heads * 64 * float(sum(int(s) * int(s) for s in self.varlen_seqs))
        else:
            f = 4.0 * self.batch * self.heads * float(self.seqlen) * self.seqlen * 64
        return f * (0.5 if self.causal else 1.0)

    def tokens(self) -> int:
        return int(sum(self.varlen_seqs)) if self.varlen_seqs else self.batch * self.seqlen


def varlen_lengths(n: int = 16, lo: int = 128, hi: int = 8192, seed: int = 7) -> list[int]:
    """North-star varlen config: lengths uniform-integer in [lo, hi] from `seed`."""
    rng = np.random.default_rng(seed)
    return [int(x) for x in rng.integers(lo, hi + 1, size=n)]


WORKLOADS = {
    "c1": Workload("B1 H2 S256 D64 bf16 non-causal +LSE (uniform)", 1, 2, 256, False, True,
                   dist="uniform"),
    "c2": Workload("B4 H16 S2048 D64 bf16 non-causal", 4, 16, 2048, False, False),
    "c3": Workload("B1 H16 S8192 D64 bf16 causal +LSE", 1, 16, 8192, True, True),
    "c4": Workload("varlen 16 seqs U{128..8192} H16 D64 bf16 non-causal +LSE", 16, 16, 0, False,
                   True, layout="thd", varlen_seqs=tuple(varlen_lengths())),
    "c4c": Workload("varlen 16 seqs U{128..8192} H16 D64 bf16 causal +LSE", 16, 16, 0, True, True,
                    layout="thd", varlen_seqs=tuple(varlen_lengths())),
    "c5a": Workload("B1 H2 S40000 D64 bf16 causal +LSE", 1, 2, 40000, True, True),
    "c5b": Workload("B32 H32 S4096 D64 bf16 causal", 32, 32, 4096, True, False),
    # one eighth of c5b (its per-rank share at 8 GPUs): the profiling case
    "c5b_s8": Workload("B4 H32 S4096 D64 bf16 causal (c5b / 8)", 4, 32, 4096, True, False),
    # c5b's shape with grouped K/V: 4 query heads per K/V head, and one K/V head
    # for all 32 (the reference's GQA/MQA test ratios, tests/test_configs.hpp:27-31,66-67)
    "c5b_gqa4": Workload("B32 H32 Hkv8 S4096 D64 bf16 causal (GQA 4)", 32, 32, 4096, True,
                         False, kv_heads=8),
    "c5b_mqa": Workload("B32 H32 Hkv1 S4096 D64 bf16 causal (MQA)", 32, 32, 4096, True, False,
                        kv_heads=1),
    "c2_gqa4": Workload("B4 H16 Hkv4 S2048 D64 bf16 non-causal (GQA 4)", 4, 16, 2048, False,
                        False, kv_heads=4),
}


def make_tensor(shape, seed: int, dist: str, device):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    if dist == "uniform":
        x = torch.rand(shape, generator=g, device=device, dtype=torch.float32) * 2.0 - 1.0
    else:
        x = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    return x.to(torch.bfloat16)


def make_inputs(w: Workload, device, seed_base: int = 0):
    """(q, k, v, cu_seqlens or None) on `device`, seeds seed_base+{0,1,2}."""
    import torch

    if w.varlen_seqs:
        total = w.tokens()
        shape = (total, w.heads, 64)
        shape_kv = (total, w.heads_k, 64)
        cu = torch.tensor(np.concatenate([[0], np.cumsum(w.varlen_seqs)]).astype(np.int32),
                          device=device)
    else:
        shape = (w.batch, w.seqlen, w.heads, 64)
        shape_kv = (w.batch, w.seqlen, w.heads_k, 64)
        cu = None
    q = make_tensor(shape, seed_base + 0, w.dist, device)
    k = make_tensor(shape_kv, seed_base + 1, w.dist, device)
    v = make_tensor(shape_kv, seed_base + 2, w.dist, device)
    return q, k, v, cu
