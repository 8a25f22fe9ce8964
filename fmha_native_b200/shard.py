"""Work partitioning of one forward pass across GPUs (and ordering within
one GPU).

The unit of work is a query block: 128 query rows of one (sequence, head),
the work one CTA of the kernel performs.  Its cost is the number of 128-key
tiles it visits (causal blocks near the top of a sequence are cheap, blocks
at the bottom are expensive) plus a fixed per-block overhead.  Blocks are independent -- each reads only its own Q rows
and the K/V of its (sequence, kv head) -- so a partition needs no exchange:
every rank holds K/V, runs `fmha_fwd_d64_bf16_tiles` on its own list and
writes disjoint rows of O / LSE.

`plan_blocks` lists the blocks with costs; `partition` assigns them to ranks
with longest-processing-time-first greedy balancing, and returns each rank's
list head-major (blocks of one (batch, head) together, so its K/V stays in
L2), heaviest first within a head.
"""
from __future__ import annotations

import heapq
from typing import List, Optional, Sequence, Tuple

ROWS_PER_TILE = 128


def _rows_per_block() -> int:
    """Query rows per work-list entry of the built kernel (128 or 256)."""
    try:
        import ctypes
        import os

        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libfmha_b200.so")
        return int(ctypes.CDLL(path).fmha_fwd_d64_rows_per_block())
    except Exception:
        return 128


ROWS_PER_BLOCK = _rows_per_block()
KEYS_PER_TILE = 128
BLOCK_OVERHEAD = 2.0  # per-block prologue/epilogue, in KV-tile units

Block = Tuple[int, int, float]  # (b*nhead_q + h, query block index, cost)


def _kv_tiles(r0: int, seqlen_q: int, seqlen_k: int, causal: bool) -> int:
    if r0 >= seqlen_q:
        return 0
    kv_end = seqlen_k
    if causal:
        r_last = min(r0 + ROWS_PER_TILE - 1, seqlen_q - 1)
        kv_end = min(seqlen_k, r_last + (seqlen_k - seqlen_q) + 1)
    return (kv_end + KEYS_PER_TILE - 1) // KEYS_PER_TILE if kv_end > 0 else 0


def block_cost(m: int, seqlen_q: int, seqlen_k: int, causal: bool) -> float:
    r0 = m * ROWS_PER_BLOCK
    n = sum(_kv_tiles(r0 + t * ROWS_PER_TILE, seqlen_q, seqlen_k, causal)
            for t in range(ROWS_PER_BLOCK // ROWS_PER_TILE))
    return float(n) + BLOCK_OVERHEAD


def plan_blocks(batch: int, nhead_q: int, seqlen_q: int, seqlen_k: int, causal: bool,
                varlen_seqs: Optional[Sequence[int]] = None) -> List[Block]:
    """Every query block of the problem with its cost.  Varlen: sequence b
    has Sq = Sk = varlen_seqs[b] (the reference's group-mode convention)."""
    out: List[Block] = []
    for b in range(batch):
        sq = int(varlen_seqs[b]) if varlen_seqs else seqlen_q
        sk = int(varlen_seqs[b]) if varlen_seqs else seqlen_k
        nblk = (sq + ROWS_PER_BLOCK - 1) // ROWS_PER_BLOCK
        for h in range(nhead_q):
            for m in range(nblk):
                out.append((b * nhead_q + h, m, block_cost(m, sq, sk, causal)))
    return out


def partition(blocks: Sequence[Block], world: int) -> List[List[Block]]:
    """LPT greedy: blocks in decreasing cost go to the least-loaded rank.
    Ties break on rank index, so every rank computes the same plan."""
    order = sorted(blocks, key=lambda x: (-x[2], x[0], x[1]))
    heap = [(0.0, r) for r in range(world)]
    parts: List[List[Block]] = [[] for _ in range(world)]
    for blk in order:
        load, r = heapq.heappop(heap)
        parts[r].append(blk)
        heapq.heappush(heap, (load + blk[2], r))
    # Launch order inside a rank: head-major (a head's blocks run together,
    # sharing its K/V in L2), heaviest first within a head.
    return [sorted(p, key=lambda x: (x[0], -x[2], x[1])) for p in parts]


def loads(parts: Sequence[Sequence[Block]]) -> List[float]:
    return [sum(b[2] for b in p) for p in parts]


def tiles_array(part: Sequence[Block]):
    """int32 [n, 2] array of (b*nhead_q + h, m) for the C ABI."""
    import numpy as np

    return np.asarray([(b[0], b[1]) for b in part], dtype=np.int32).reshape(-1, 2)


Item = Tuple[int, int, int, int]  # (b*nhead_q + h, query block, kv_begin, kv_end)


def plan_items(part: Sequence[Block], slots: int = 2 * 148, waves: float = 1.0,
               min_chunk: int = 4) -> List[Item]:
    """Work items for fmha_fwd_d64_bf16_items.

    The launch gets at most `waves` x `slots` CTAs (slots = resident CTAs
    per GPU): the smallest piece size `cap` (KV tiles) is found for which
    cutting every block into ceil(n / cap) near-equal consecutive KV ranges
    stays within that count.  A block no longer than `cap` stays whole
    (kv_end = -1, written directly); the pieces of a split block are partial
    items merged after the launch.  With one wave every CTA slot runs one
    item, so the launch takes about the longest piece -- cutting blocks to
    the count of slots, not to a fixed size, avoids a thin extra wave.
    Blocks are listed by piece size, largest first (the hardware starts CTAs
    in list order); a split block's pieces stay consecutive, as the merge
    expects."""
    if not part:
        return []
    n_kv = [max(0, int(round(b[2] - BLOCK_OVERHEAD))) for b in part]
    target = max(1, int(waves * slots))
    lo, hi = max(1, min_chunk), max(max(n_kv), 1)
    while lo < hi:
        mid = (lo + hi) // 2
        if sum(-(-n // mid) for n in n_kv if n > 0) <= target:
            hi = mid
        else:
            lo = mid + 1
    cap = max(lo, min_chunk)
    groups = []
    for b, n in zip(part, n_kv):
        k = -(-n // cap) if n > 0 else 1
        if k <= 1:
            groups.append((n, [(b[0], b[1], 0, -1)]))
            continue
        edges = [n * i // k for i in range(k + 1)]
        groups.append((n / k, [(b[0], b[1], edges[i], edges[i + 1]) for i in range(k)]))
    groups.sort(key=lambda g: -g[0])  # stable: ties keep the head-major order
    return [it for _, its in groups for it in its]


def items_array(items: Sequence[Item]):
    """int32 [n, 4] array of work items for the C ABI."""
    import numpy as np

    return np.asarray(items, dtype=np.int32).reshape(-1, 4)


def choose_splits(nblocks: int, sms: int = 148, target_waves: float = 4.0,
                  max_splits: int = 8) -> int:
    """Split-KV factor so that a launch of `nblocks` query blocks still has
    about `target_waves` work items per SM (1 when the blocks already do).
    Four per SM (two per CTA slot) measured best for one rank's 1/8 share of
    B1 H2 S40000 causal (79 blocks: 8 splits 104 us, 4 splits 112-122 us)."""
    if nblocks <= 0:
        return 1
    want = int(-(-target_waves * sms // nblocks))
    return max(1, min(max_splits, want))
