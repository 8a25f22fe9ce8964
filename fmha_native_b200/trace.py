"""Per-role pipeline timeline of the sm_100a kernel, from its trace build.

``libfmha_b200_trace.so`` is the kernel source compiled with -DFMHA_TRACE:
for a window of consecutive CTAs it stamps ``clock64`` (SM cycles) at the
pipeline events of pass 0, per KV step j:

====  =======================================================  ==========
slot  event                                                     role
====  =======================================================  ==========
0     S(j) complete seen (after the s_full wait)                softmax
1     S(j) in registers, s_free arrived                         softmax
2     exponentials of tile j issued                             softmax
3     P(j-1) consumed seen (pv_done wait passed)                softmax
4     P(j) in TMEM, p_full arrived                              softmax
5     S(j+1) MMAs issued                                        MMA warp
6     PV(j) MMAs issued                                         MMA warp
7     per CTA, by step index: 7 kernel entry, 0 set-up done      --
      (barriers, TMEM), 1 SM id, 5 Q TMA issued, 6 Q landed
      (MMA warp), 2 O complete seen, 3 epilogue stores issued,
      4 CTA past its final barrier
8     K(j+1) landed (seen by the MMA warp)                      MMA warp
9     s_free(j) seen                                            MMA warp
10    V(j) landed                                               MMA warp
11    p_full(j) seen                                            MMA warp
12    S(j) complete (commit observed)                           observer
13    PV(j) complete (commit observed)                          observer
14    K(j) TMA issued                                           producer
15    V(j) TMA issued                                           producer
====  =======================================================  ==========

Softmax stamps come from thread 0 (warp 0); the observer is the otherwise
idle warp 6, polling the commit barriers.  `summarize` turns the stamps into
median segment lengths over the steady-state steps of every traced CTA.

    python -m fmha_native_b200.trace --config c5b [--first-cta 512]
"""
from __future__ import annotations

import argparse
import ctypes
import os
import statistics
from typing import Dict, List

import numpy as np

from .build import TRACE_LIB_PATH

SEGMENTS = [
    # (name, (slot, step offset) end, (slot, step offset) start)
    ("softmax: S(j) TMEM load + s_free", (1, 0), (0, 0)),
    ("softmax: exponential pass issued", (2, 0), (1, 0)),
    ("softmax: pass drains, P(j-1) consumed seen", (3, 0), (2, 0)),
    ("softmax: P(j) store + p_full", (4, 0), (3, 0)),
    ("softmax: p_full(j) -> S(j+1) seen", (0, 1), (4, 0)),
    ("softmax: period (s_free(j) -> s_free(j+1))", (1, 1), (1, 0)),
    ("MMA: s_free(j) seen -> S(j+1) issued", (5, 0), (9, 0)),
    ("MMA: p_full(j) seen -> PV(j) issued", (6, 0), (11, 0)),
    ("MMA: softmax s_free(j) -> MMA sees all arrivals", (9, 0), (1, 0)),
    ("tensor: S(j+1) issue -> complete", (12, 1), (5, 0)),
    ("tensor: PV(j) issue -> complete", (13, 0), (6, 0)),
    ("slack: S(j+1) complete before softmax needs it", (0, 1), (12, 1)),
    ("slack: PV(j-1) complete before softmax needs it", (3, 0), (13, -1)),
    ("TMA: K(j+1) issue -> landed", (8, 0), (14, 1)),
]


# Per-CTA segments: slot-7 stamps (by step index) and the first/last steps.
CTA_SEGMENTS = [
    ("entry -> set-up done (barriers, TMEM alloc)", ("c", 0), ("c", 7)),
    ("set-up done -> Q TMA issued", ("c", 5), ("c", 0)),
    ("Q TMA issued -> Q landed (MMA warp)", ("c", 6), ("c", 5)),
    ("Q landed -> S(0) complete", ("s", 12, 0), ("c", 6)),
    ("S(0) complete -> seen by softmax", ("s", 0, 0), ("s", 12, 0)),
    ("first step (row max) s_free(0) -> s_free(1)", ("s", 1, 1), ("s", 1, 0)),
    ("last p_full -> O complete seen", ("c", 2), ("s", 4, -1)),
    ("O complete -> epilogue stores issued", ("c", 3), ("c", 2)),
    ("epilogue -> CTA past its final barrier", ("c", 4), ("c", 3)),
    ("whole CTA (entry -> final barrier)", ("c", 4), ("c", 7)),
]


def _stamp(T, n, ref):
    if ref[0] == "c":
        return T[ref[1], 7]
    step = ref[2] if ref[2] >= 0 else n + ref[2]
    return T[step, ref[1]]


def summarize_cta(t: np.ndarray) -> Dict[str, object]:
    """Median per-CTA prologue / epilogue segments (cycles) over the traced
    CTAs that ran at least two KV steps, and their median step count."""
    vals: Dict[str, List[float]] = {name: [] for name, _, _ in CTA_SEGMENTS}
    steps = []
    for c in range(t.shape[0]):
        T = t[c]
        n = int((T[:, 4] > 0).sum())
        if n < 2 or T[4, 7] == 0:
            continue
        steps.append(n)
        for name, e, b in CTA_SEGMENTS:
            x, y = _stamp(T, n, e), _stamp(T, n, b)
            if x > 0 and y > 0:
                vals[name].append(float(x - y))
    return {"ctas": len(steps), "steps": statistics.median(steps) if steps else None,
            "segments": {k: (statistics.median(v) if v else None) for k, v in vals.items()}}


def load_trace_library(path: str = TRACE_LIB_PATH) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise RuntimeError(f"trace library not built: {path} "
                           "(fmha_native_b200.build.build_trace_library)")
    lib = ctypes.CDLL(path)
    lib.fmha_fwd_d64_trace_shape.argtypes = [ctypes.POINTER(ctypes.c_int)] * 3
    lib.fmha_fwd_d64_trace_configure.argtypes = [ctypes.c_int]
    lib.fmha_fwd_d64_trace_read.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    return lib


def shape(lib) -> tuple:
    c, s, k = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    if lib.fmha_fwd_d64_trace_shape(ctypes.byref(c), ctypes.byref(s), ctypes.byref(k)) != 0:
        raise RuntimeError("fmha_fwd_d64_trace_shape failed")
    return c.value, s.value, k.value


def read(lib) -> np.ndarray:
    """The stamps as int64 [ctas, steps, slots] (0 = not stamped)."""
    c, s, k = shape(lib)
    buf = np.zeros(c * s * k, dtype=np.uint64)
    if lib.fmha_fwd_d64_trace_read(buf.ctypes.data, buf.size) != 0:
        raise RuntimeError("fmha_fwd_d64_trace_read failed")
    return buf.reshape(c, s, k).astype(np.int64)


def summarize(t: np.ndarray, min_steps: int = 6) -> Dict[str, object]:
    """Median segment lengths (cycles) over steps 2 .. n-3 of every traced CTA
    that ran at least `min_steps` KV steps."""
    vals: Dict[str, List[float]] = {name: [] for name, _, _ in SEGMENTS}
    ctas = 0
    for c in range(t.shape[0]):
        n = int((t[c, :, 4] > 0).sum())
        if n < min_steps:
            continue
        ctas += 1
        for j in range(2, n - 2):
            for name, (se, oe), (ss, os_) in SEGMENTS:
                a, b = t[c, j + oe, se], t[c, j + os_, ss]
                if a > 0 and b > 0:
                    vals[name].append(float(a - b))
    seg = {name: (statistics.median(v) if v else None) for name, v in vals.items()}
    return {"ctas": ctas, "segments": seg}


def capture(workload_key: str, first_cta: int = 512, warmup: int = 2):
    """Run `workload_key` through the trace library on cuda:0; returns
    (stamps, output O)."""
    import torch

    import fmha_native_b200 as fm
    from .synth import WORKLOADS, make_inputs

    lib = load_trace_library()
    # Route the package's launch calls through the trace library for this
    # capture (it exports the same entry points); restored afterwards.
    fm._lib = None
    fm.load_library(TRACE_LIB_PATH)
    fmha_fwd = fm.fmha_fwd
    try:
        w = WORKLOADS[workload_key]
        dev = torch.device("cuda:0")
        q, k, v, cu = make_inputs(w, dev)
        kw = dict(causal=w.causal, return_lse=w.lse, layout=w.layout)
        if cu is not None:
            kw.update(cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=max(w.varlen_seqs),
                      max_seqlen_k=max(w.varlen_seqs))
        for _ in range(warmup):
            fmha_fwd(q, k, v, **kw)
        torch.cuda.synchronize()
        if lib.fmha_fwd_d64_trace_configure(int(first_cta)) != 0:
            raise RuntimeError("fmha_fwd_d64_trace_configure failed")
        out = fmha_fwd(q, k, v, **kw)
        torch.cuda.synchronize()
        return read(lib), (out[0] if isinstance(out, tuple) else out)
    finally:
        fm._lib = None


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--config", default="c5b")
    ap.add_argument("--first-cta", type=int, default=512)
    args = ap.parse_args()
    t, _ = capture(args.config, args.first_cta)
    s = summarize(t)
    print(f"config {args.config}: CTAs {args.first_cta}..{args.first_cta + t.shape[0] - 1}, "
          f"{s['ctas']} traced with >= 6 KV steps; median cycles per KV step")
    for name, v in s["segments"].items():
        print(f"  {name:52s} {v if v is None else round(v):>8}")
    c = summarize_cta(t)
    print(f"per CTA (median over {c['ctas']} CTAs, {c['steps']} KV steps each):")
    for name, v in c["segments"].items():
        print(f"  {name:52s} {v if v is None else round(v):>8}")


if __name__ == "__main__":
    main()
