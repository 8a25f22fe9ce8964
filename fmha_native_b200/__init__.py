"""fmha_native_b200 -- B200 (sm_100a) head-dim-64 BF16 fused attention forward.

Host-side mirror of the poyenc/fmha_native operator surface:

* :class:`FmhaFwdParams` -- the kernel-argument struct
  (reference ``src/runner/params.hpp:18-64``), as a ctypes structure with the
  same field order.
* :data:`ENTRY_POINTS` -- the four entries ``fmha_fwd_d64_bf16_msk{0,1}[_varlen]``
  (reference ``src/fused/kernel.cpp:55-99``), exported by the C-ABI library
  ``libfmha_b200.so`` (see ``include/fmha_fwd.h``).
* :class:`FmhaParams` -- the host workload description
  (reference ``src/runner/fmha_params.hpp:12-44``) and :func:`make_params`
  (reference ``tests/test_params.hpp:31-61``).
* :func:`fmha_fwd` -- a convenience call over torch CUDA tensors that builds
  the params from tensor strides and calls the C ABI.

There is no CPU fallback: every compute call goes through the CUDA library
and raises :class:`FmhaError` if it is missing or fails.
"""
from __future__ import annotations

import ctypes
import dataclasses
import math
import os
from typing import Optional, Sequence

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libfmha_b200.so")

LOG2E = 1.4426950408889634
HEAD_DIM = 64
BLOCK_M = 128          # query rows per tile (one tile per CTA)
BLOCK_N = 128          # keys per KV tile

FMHA_OK = 0
FMHA_ERR_ARG = 1
FMHA_ERR_LAUNCH = 2
FMHA_ERR_TIMEOUT = 3
FMHA_ERR_DEVICE = 4
FMHA_ERR_SCRATCH = 5

ENTRY_POINTS = (
    "fmha_fwd_d64_bf16_msk0",
    "fmha_fwd_d64_bf16_msk1",
    "fmha_fwd_d64_bf16_msk0_varlen",
    "fmha_fwd_d64_bf16_msk1_varlen",
    "fmha_fwd_d64_bf16",
    "fmha_fwd_d64_bf16_tiles",
    "fmha_fwd_d64_bf16_tiles_splitkv",
    "fmha_fwd_d64_splitkv_workspace_bytes",
    "fmha_fwd_d64_bf16_items",
    "fmha_fwd_d64_items_workspace_bytes",
    "fmha_fwd_d64_status",
    "fmha_fwd_d64_set_wait_limit_ns",
    "fmha_fwd_d64_release",
    "fmha_fwd_d64_error_string",
)


class FmhaError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        super().__init__(f"{what}: status {status} ({error_string(status)})" if what else
                         f"status {status} ({error_string(status)})")


class FmhaFwdParams(ctypes.Structure):
    """Kernel argument block; field order follows src/runner/params.hpp:18-64."""

    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("seqlen_q", ctypes.c_int), ("seqlen_k", ctypes.c_int),
        ("nhead_q", ctypes.c_int), ("nhead_k", ctypes.c_int),
        ("scale", ctypes.c_float),
        ("stride_q", ctypes.c_int), ("nhead_stride_q", ctypes.c_int), ("batch_stride_q", ctypes.c_int),
        ("stride_k", ctypes.c_int), ("nhead_stride_k", ctypes.c_int), ("batch_stride_k", ctypes.c_int),
        ("stride_v", ctypes.c_int), ("nhead_stride_v", ctypes.c_int), ("batch_stride_v", ctypes.c_int),
        ("stride_o", ctypes.c_int), ("nhead_stride_o", ctypes.c_int), ("batch_stride_o", ctypes.c_int),
        ("seqstart_q", ctypes.c_void_p), ("seqstart_k", ctypes.c_void_p),
    ]


_lib = None


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the CUDA library (built in-tree).  Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FmhaError(FMHA_ERR_DEVICE, f"CUDA library not built: {path} "
                        "(run `python -m fmha_native_b200.build`)")
    lib = ctypes.CDLL(path)
    P = ctypes.POINTER(FmhaFwdParams)
    for name in ("fmha_fwd_d64_bf16_msk0", "fmha_fwd_d64_bf16_msk1"):
        fn = getattr(lib, name)
        fn.argtypes = [P, ctypes.c_int, ctypes.c_void_p]
        fn.restype = ctypes.c_int
    for name in ("fmha_fwd_d64_bf16_msk0_varlen", "fmha_fwd_d64_bf16_msk1_varlen"):
        fn = getattr(lib, name)
        fn.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        fn.restype = ctypes.c_int
    lib.fmha_fwd_d64_bf16.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_void_p]
    lib.fmha_fwd_d64_bf16.restype = ctypes.c_int
    lib.fmha_fwd_d64_bf16_tiles.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                            ctypes.c_void_p]
    lib.fmha_fwd_d64_bf16_tiles.restype = ctypes.c_int
    lib.fmha_fwd_d64_bf16_tiles_splitkv.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                    ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                                    ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                                    ctypes.c_void_p]
    lib.fmha_fwd_d64_bf16_tiles_splitkv.restype = ctypes.c_int
    lib.fmha_fwd_d64_splitkv_workspace_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
    lib.fmha_fwd_d64_splitkv_workspace_bytes.restype = ctypes.c_size_t
    lib.fmha_fwd_d64_bf16_items.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                            ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.fmha_fwd_d64_bf16_items.restype = ctypes.c_int
    lib.fmha_fwd_d64_items_workspace_bytes.argtypes = [ctypes.c_int]
    lib.fmha_fwd_d64_items_workspace_bytes.restype = ctypes.c_size_t
    lib.fmha_fwd_d64_status.argtypes = [ctypes.c_void_p]
    lib.fmha_fwd_d64_status.restype = ctypes.c_int
    lib.fmha_fwd_d64_set_wait_limit_ns.argtypes = [ctypes.c_ulonglong]
    lib.fmha_fwd_d64_set_wait_limit_ns.restype = None
    lib.fmha_fwd_d64_release.argtypes = []
    lib.fmha_fwd_d64_release.restype = None
    lib.fmha_fwd_d64_error_string.argtypes = [ctypes.c_int]
    lib.fmha_fwd_d64_error_string.restype = ctypes.c_char_p
    lib.fmha_fwd_d64_debug_set_stall.argtypes = [ctypes.c_int]
    lib.fmha_fwd_d64_debug_set_stall.restype = None
    _lib = lib
    return lib


def error_string(status: int) -> str:
    names = {0: "ok", 1: "invalid argument", 2: "CUDA launch or runtime error",
             3: "device pipeline wait exceeded its time limit", 4: "no supported sm_100 device",
             5: "request exceeds the allocation-free scratch"}
    return names.get(status, "unknown status")


@dataclasses.dataclass
class FmhaParams:
    """Host workload description (reference src/runner/fmha_params.hpp:12-44).

    Only the fields the D64 forward path reads are kept; ``scalar()`` is the
    plain softmax scale 1/sqrt(head_dim).
    """

    batch: int = 2
    q_heads: int = 16
    kv_heads: int = 0
    gqa: int = 1
    seq_len: int = 4096
    kv_seq_len: int = 0
    head_dim: int = 64
    mask: int = 0
    lse: int = 0
    varlen_seqs: list = dataclasses.field(default_factory=list)

    def scalar(self) -> float:
        return 1.0 / math.sqrt(float(self.head_dim))


def make_params(b: int, h: int, s: int, d: int = 64, kv_heads: int = 0, kv_seq: int = 0,
                mask: int = 0, lse: int = 0, varlen_seqs: Sequence[int] = ()) -> FmhaParams:
    """Expand a test-case row into FmhaParams (reference tests/test_params.hpp:31-61)."""
    p = FmhaParams(batch=b, q_heads=h, kv_heads=kv_heads, gqa=1, seq_len=s, kv_seq_len=kv_seq,
                   head_dim=d, mask=mask, lse=lse, varlen_seqs=list(varlen_seqs))
    if p.kv_heads == 0:
        p.kv_heads = p.q_heads
    if p.q_heads != p.kv_heads:
        p.gqa = p.q_heads // p.kv_heads
    if p.varlen_seqs:
        p.batch = len(p.varlen_seqs)
        p.seq_len = max(p.varlen_seqs)
        if p.kv_seq_len == 0:
            p.kv_seq_len = p.seq_len
    if p.kv_seq_len == 0:
        p.kv_seq_len = p.seq_len
    return p


def _check(status: int, what: str) -> None:
    if status != FMHA_OK:
        raise FmhaError(status, what)


def call_entry(params: FmhaFwdParams, batch: int, causal: bool, varlen: bool,
               total_q: int = 0, total_k: int = 0, stream: int = 0) -> int:
    """Call one of the four C-ABI entries; returns the raw status."""
    lib = load_library()
    ref = ctypes.byref(params)
    if varlen:
        fn = lib.fmha_fwd_d64_bf16_msk1_varlen if causal else lib.fmha_fwd_d64_bf16_msk0_varlen
        return fn(ref, batch, total_q, total_k, ctypes.c_void_p(stream))
    fn = lib.fmha_fwd_d64_bf16_msk1 if causal else lib.fmha_fwd_d64_bf16_msk0
    return fn(ref, batch, ctypes.c_void_p(stream))


def call_tiles(params: FmhaFwdParams, batch: int, causal: bool, tiles_ptr: int, ntiles: int,
               total_q: int = 0, total_k: int = 0, stream: int = 0) -> int:
    """Call fmha_fwd_d64_bf16_tiles on a device int32 [ntiles, 2] work list."""
    lib = load_library()
    return lib.fmha_fwd_d64_bf16_tiles(ctypes.byref(params), batch, int(causal), total_q, total_k,
                                       ctypes.c_void_p(tiles_ptr), ntiles, ctypes.c_void_p(stream))


def splitkv_workspace_bytes(ntiles: int, num_splits: int) -> int:
    return int(load_library().fmha_fwd_d64_splitkv_workspace_bytes(ntiles, num_splits))


def call_tiles_splitkv(params: FmhaFwdParams, batch: int, causal: bool, tiles_ptr: int,
                       ntiles: int, num_splits: int, workspace_ptr: int, workspace_bytes: int,
                       total_q: int = 0, total_k: int = 0, stream: int = 0) -> int:
    """Call fmha_fwd_d64_bf16_tiles_splitkv (split-KV over a device work list)."""
    lib = load_library()
    return lib.fmha_fwd_d64_bf16_tiles_splitkv(
        ctypes.byref(params), batch, int(causal), total_q, total_k, ctypes.c_void_p(tiles_ptr),
        ntiles, num_splits, ctypes.c_void_p(workspace_ptr), workspace_bytes,
        ctypes.c_void_p(stream))


def items_workspace_bytes(n_items: int) -> int:
    return int(load_library().fmha_fwd_d64_items_workspace_bytes(n_items))


def call_items(params: FmhaFwdParams, batch: int, causal: bool, items_ptr: int, n_items: int,
               workspace_ptr: int, workspace_bytes: int, total_q: int = 0, total_k: int = 0,
               stream: int = 0) -> int:
    """Call fmha_fwd_d64_bf16_items on a device int32 [n_items, 4] item list
    (b*nhead_q + h, query block, kv_begin, kv_end); see shard.plan_items."""
    lib = load_library()
    return lib.fmha_fwd_d64_bf16_items(
        ctypes.byref(params), batch, int(causal), total_q, total_k, ctypes.c_void_p(items_ptr),
        n_items, ctypes.c_void_p(workspace_ptr), workspace_bytes, ctypes.c_void_p(stream))


def status(stream: int = 0) -> int:
    """Synchronise `stream` and read/clear the device error word."""
    return load_library().fmha_fwd_d64_status(ctypes.c_void_p(stream))


def params_from_tensors(q, k, v, o, lse=None, layout: str = "bshd",
                        seqstart_q=None, seqstart_k=None, scale: Optional[float] = None,
                        max_seqlen_q: Optional[int] = None, max_seqlen_k: Optional[int] = None):
    """Build FmhaFwdParams from torch CUDA tensors.

    Dense layouts: "bshd" ([B,S,H,D]) or "bhsd" ([B,H,S,D]).
    Varlen layouts: "thd" ([total,H,D]) or "htd" ([H,total,D]); the longest
    sequence lengths go into seqlen_q/seqlen_k (the reference's varlen
    convention).  Pass max_seqlen_q/max_seqlen_k when known: otherwise they
    are read from the device prefix sums, which synchronises the stream.
    Returns (params, batch, total_q, total_k).
    """
    p = FmhaFwdParams()
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    p.lse = lse.data_ptr() if lse is not None else None
    p.scale = (scale if scale is not None else 1.0 / math.sqrt(HEAD_DIM)) * LOG2E
    if layout in ("bshd", "bhsd"):
        s_ax, h_ax = (1, 2) if layout == "bshd" else (2, 1)
        batch = q.shape[0]
        p.seqlen_q, p.seqlen_k = q.shape[s_ax], k.shape[s_ax]
        p.nhead_q, p.nhead_k = q.shape[h_ax], k.shape[h_ax]
        for name, t in (("q", q), ("k", k), ("v", v), ("o", o)):
            st = t.stride()
            setattr(p, f"stride_{name}", st[s_ax])
            setattr(p, f"nhead_stride_{name}", st[h_ax])
            setattr(p, f"batch_stride_{name}", st[0])
        p.seqstart_q = None
        p.seqstart_k = None
        return p, batch, 0, 0
    if layout in ("thd", "htd"):
        t_ax, h_ax = (0, 1) if layout == "thd" else (1, 0)
        batch = seqstart_q.numel() - 1
        total_q, total_k = q.shape[t_ax], k.shape[t_ax]
        if max_seqlen_q is None or max_seqlen_k is None:
            sq = seqstart_q.to("cpu")
            sk = seqstart_k.to("cpu")
            max_seqlen_q = int((sq[1:] - sq[:-1]).max()) if batch > 0 else 0
            max_seqlen_k = int((sk[1:] - sk[:-1]).max()) if batch > 0 else 0
        p.seqlen_q = int(max_seqlen_q)
        p.seqlen_k = int(max_seqlen_k)
        p.nhead_q, p.nhead_k = q.shape[h_ax], k.shape[h_ax]
        for name, t in (("q", q), ("k", k), ("v", v), ("o", o)):
            st = t.stride()
            setattr(p, f"stride_{name}", st[t_ax])
            setattr(p, f"nhead_stride_{name}", st[h_ax])
            setattr(p, f"batch_stride_{name}", 0)
        p.seqstart_q = seqstart_q.data_ptr()
        p.seqstart_k = seqstart_k.data_ptr()
        return p, batch, total_q, total_k
    raise ValueError(f"unknown layout {layout!r}")


def fmha_fwd(q, k, v, causal: bool = False, return_lse: bool = False, layout: str = "bshd",
             cu_seqlens_q=None, cu_seqlens_k=None, out=None, lse_out=None, stream=None,
             tiles=None, num_splits: int = 1, workspace=None, items=None,
             max_seqlen_q: Optional[int] = None, max_seqlen_k: Optional[int] = None):
    """O = softmax(Q K^T / 8) V on the B200 kernel (head_dim 64, bf16).

    Dense: q [B,Sq,Hq,64] ("bshd") or [B,Hq,Sq,64] ("bhsd"); varlen: q
    [total,Hq,64] ("thd") or [Hq,total,64] ("htd") with int32 cu_seqlens.
    Returns O (and fp32 LSE [B,Hq,Sq] / [Hq,total] when return_lse).
    `tiles`: optional device int32 [n, 2] list of query blocks to compute
    (fmha_native_b200.shard); other rows of `out` are left untouched.
    `num_splits` > 1 (with `tiles`) splits each block's key range (split-KV);
    `workspace` is then a device buffer of splitkv_workspace_bytes() bytes
    (allocated here when omitted).
    `items`: optional device int32 [n, 4] work-item list with per-item KV
    ranges (fmha_native_b200.shard.plan_items); `workspace` then holds
    items_workspace_bytes(n) bytes (allocated here when omitted).
    `max_seqlen_q/k` (varlen): the longest sequence lengths, if known; else
    they are read from cu_seqlens (a stream synchronisation).
    """
    import torch

    for t in (q, k, v):
        if not (t.is_cuda and t.dtype == torch.bfloat16 and t.shape[-1] == HEAD_DIM):
            raise FmhaError(FMHA_ERR_ARG, "q/k/v must be CUDA bf16 tensors with head_dim 64")
    o = out if out is not None else torch.empty_like(q)
    varlen = layout in ("thd", "htd")
    lse = None
    if return_lse:
        if lse_out is not None:
            lse = lse_out
        elif varlen:
            h = q.shape[1] if layout == "thd" else q.shape[0]
            total = q.shape[0] if layout == "thd" else q.shape[1]
            lse = torch.empty(h, total, device=q.device, dtype=torch.float32)
        else:
            s_ax, h_ax = (1, 2) if layout == "bshd" else (2, 1)
            lse = torch.empty(q.shape[0], q.shape[h_ax], q.shape[s_ax], device=q.device,
                              dtype=torch.float32)
    params, batch, tq, tk = params_from_tensors(q, k, v, o, lse, layout, cu_seqlens_q,
                                                cu_seqlens_k, max_seqlen_q=max_seqlen_q,
                                                max_seqlen_k=max_seqlen_k)
    s = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
    if items is not None:
        nbytes = items_workspace_bytes(items.shape[0])
        if workspace is None:
            workspace = torch.empty(max(nbytes, 16) // 4, device=q.device, dtype=torch.float32)
        _check(call_items(params, batch, causal, items.data_ptr(), items.shape[0],
                          workspace.data_ptr(), workspace.numel() * workspace.element_size(),
                          tq, tk, s), "fmha_fwd(items)")
    elif tiles is not None and num_splits > 1:
        nbytes = splitkv_workspace_bytes(tiles.shape[0], num_splits)
        if workspace is None:
            workspace = torch.empty(nbytes // 4, device=q.device, dtype=torch.float32)
        _check(call_tiles_splitkv(params, batch, causal, tiles.data_ptr(), tiles.shape[0],
                                  num_splits, workspace.data_ptr(),
                                  workspace.numel() * workspace.element_size(), tq, tk, s),
               "fmha_fwd(split-KV)")
    elif tiles is not None:
        # device int32 [n, 2] work list (see fmha_native_b200.shard)
        _check(call_tiles(params, batch, causal, tiles.data_ptr(), tiles.shape[0], tq, tk, s),
               "fmha_fwd(tiles)")
    else:
        _check(call_entry(params, batch, causal, varlen, tq, tk, s), "fmha_fwd")
    return (o, lse) if return_lse else o


def fmha_fwd_from_host(q, k, v, causal: bool = False, layout: str = "bshd", out=None,
                       chunks: int = 4, device=None):
    """O = attention(Q, K, V) for dense inputs that live in (pinned) HOST
    memory: the batch is cut into `chunks` slices, and three streams overlap
    the host->device copies of slice i+1, the kernel of slice i and the
    device->host copy of slice i-1's O (PCIe is full duplex, so the two copy
    directions run at the same time).  Returns the host tensor `out`
    (allocated pinned when omitted).  The caller's current stream is ordered
    after the last copy: synchronise it before reading `out`.  Device staging
    buffers are cached per shape and device."""
    import torch

    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if layout not in ("bshd", "bhsd"):
        raise FmhaError(FMHA_ERR_ARG, "fmha_fwd_from_host takes dense layouts")
    B = q.shape[0]
    chunks = max(1, min(chunks, B))
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    key = (tuple(q.shape), tuple(k.shape), dev.index)
    st = _host_state.get(key)
    if st is None:
        st = {"dq": torch.empty(q.shape, dtype=q.dtype, device=dev),
              "dk": torch.empty(k.shape, dtype=k.dtype, device=dev),
              "dv": torch.empty(v.shape, dtype=v.dtype, device=dev),
              "do": torch.empty(q.shape, dtype=q.dtype, device=dev),
              "h2d": torch.cuda.Stream(dev), "comp": torch.cuda.Stream(dev),
              "d2h": torch.cuda.Stream(dev)}
        _host_state[key] = st
    cur = torch.cuda.current_stream(dev)
    h2d, comp, d2h = st["h2d"], st["comp"], st["d2h"]
    for s_ in (h2d, comp, d2h):
        s_.wait_stream(cur)
    bounds = [B * i // chunks for i in range(chunks + 1)]
    for i in range(chunks):
        b0, b1 = bounds[i], bounds[i + 1]
        if b0 == b1:
            continue
        with torch.cuda.stream(h2d):
            for name, h in (("dq", q), ("dk", k), ("dv", v)):
                st[name][b0:b1].copy_(h[b0:b1], non_blocking=True)
            loaded = torch.cuda.Event()
            loaded.record(h2d)
        comp.wait_event(loaded)
        fmha_fwd(st["dq"][b0:b1], st["dk"][b0:b1], st["dv"][b0:b1], causal=causal,
                 layout=layout, out=st["do"][b0:b1], stream=comp.cuda_stream)
        done = torch.cuda.Event()
        done.record(comp)
        d2h.wait_event(done)
        with torch.cuda.stream(d2h):
            out[b0:b1].copy_(st["do"][b0:b1], non_blocking=True)
    cur.wait_stream(d2h)
    cur.wait_stream(comp)
    cur.wait_stream(h2d)
    return out


_host_state: dict = {}
