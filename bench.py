#!/usr/bin/env python3
"""Benchmark of the B200 D64 BF16 FMHA forward (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5b] [--impl native|reference]

One step = one forward pass over the workload.  Default workload is the
largest single-GPU north-star configuration, c5b (B32 H32 S4096 causal).
Multi-GPU (torchrun, one rank per GPU): by default the same problem is split
over the ranks (strong scaling): every rank holds the inputs and computes its
LPT share of the query blocks, no collective on the data path; time = max
over ranks.  `--weak` runs an independent copy per rank instead.

`--impl reference` times the reference's own CPU implementation of the path
(its cpu_ref_verify, compiled from its sources into oracle/_ref) on a bounded
sample of the same workload, on rank 0 only, with every host core.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "d64 bf16 FMHA fwd TFLOP/s per B200 (causal ×0.5), % of BF16 tensor peak"
UNIT = "TFLOP/s"
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n_, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(n_)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def reference_arm(args, workload_key):
    """CPU baseline: the reference's cpu_ref_verify on a bounded sample."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    # torchrun exports OMP_NUM_THREADS=1; the reference's OpenMP runtime reads
    # it when its library loads, so every host core is requested first.
    os.environ["OMP_NUM_THREADS"] = str(host_cores())
    import numpy as np

    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O
    from fmha_native_b200.synth import WORKLOADS

    w = WORKLOADS[workload_key]
    if not O.have_reference():
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/libfmha_ref.so not built (reference tree absent at build)"}))
        return 0
    sample = cpu_sample(w)
    res = time_cpu_reference(O, sample, args.steps, args.warmup)
    line = {
        "metric": METRIC, "value": res["tflops"], "unit": UNIT, "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["ms"], "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16 in / fp32 accumulate (CPU)", "data": "synthetic",
        "config": {"workload": w.name, "sample": sample["desc"]},
        "cpu_baseline": {"value": res["tflops"], "unit": UNIT, "cores": res["threads"],
                         "kind": "reference", "sample": sample["desc"]},
        "e2e": {"value": res["tflops"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def omp_threads() -> int:
    """Threads the OpenMP runtime of this process will use."""
    import ctypes

    try:
        return int(ctypes.CDLL("libgomp.so.1").omp_get_max_threads())
    except Exception:
        return int(os.environ.get("OMP_NUM_THREADS", "1"))


CPU_SAMPLE_MAC = 1.5e10  # multiply-adds per CPU sample: ~1-20 s on the host


def cpu_sample(w):
    """A bounded sample of workload `w` for the reference CPU oracle: every
    (batch, head) pair, the last query rows (full-length rows, the most
    expensive ones), all keys.  The row count is chosen so the sample costs
    about CPU_SAMPLE_MAC multiply-adds (QK^T + PV).  FLOPs are counted with
    the metric's convention on the sample's exact (unmasked) area."""
    if w.varlen_seqs:
        seqs = list(w.varlen_seqs)
        s = max(seqs)
        h = w.heads
        sq = int(min(256, max(16, CPU_SAMPLE_MAC / (h * s * 64 * 2))))
        keys = sum(range(s - sq + 1, s + 1)) if w.causal else sq * s
        return {"desc": f"varlen longest sequence (S={s}), H{h}, its last {sq} query rows",
                "b": 1, "h": h, "sq": sq, "sk": s, "causal": w.causal,
                "flops": 4.0 * h * keys * 64}
    b, h, s = w.batch, w.heads, w.seqlen
    hk = w.heads_k
    sq = int(min(256, s, max(16, CPU_SAMPLE_MAC / (b * h * s * 64 * 2))))
    flops = 4.0 * b * h * sq * s * 64
    if w.causal:
        # rows i = S-sq..S-1 attend i+1 keys
        keys = sum(range(s - sq + 1, s + 1))
        flops = 4.0 * b * h * keys * 64
    kv = f" Hkv{hk}" if hk != h else ""
    return {"desc": f"B{b} H{h}{kv}: last {sq} query rows x {s} keys "
                    f"({'causal' if w.causal else 'non-causal'})",
            "b": b, "h": h, "hk": hk, "sq": sq, "sk": s, "causal": w.causal, "flops": flops}


def time_cpu_reference(O, sample, steps, warmup):
    import numpy as np

    b, h, sq, sk = sample["b"], sample["h"], sample["sq"], sample["sk"]
    hk = sample.get("hk", h)
    rng = np.random.default_rng(0)
    q = O.f32_to_bf16_bits_trunc(rng.standard_normal(b * h * sq * 64).astype(np.float32))
    k = O.f32_to_bf16_bits_trunc(rng.standard_normal(b * hk * sk * 64).astype(np.float32))
    v = O.f32_to_bf16_bits_trunc(rng.standard_normal(b * hk * sk * 64).astype(np.float32))
    o = np.zeros(b * h * sq * 64, np.uint16)
    times = []
    for it in range(warmup + steps):
        t0 = time.perf_counter()
        O.ref_verify(b, h, hk, sq, sk, int(sample["causal"]), [], q, k, v, o)
        dt = time.perf_counter() - t0
        if it >= warmup:
            times.append(dt)
    ms = 1000.0 * sum(times) / len(times)
    # cpu_ref_verify hands out (b,h) pairs in chunks of 16 (cpu_ref.cpp:84),
    # so at most ceil(B*H/16) of the runtime's threads get work.
    threads = min(omp_threads(), max(1, -(-(b * h) // 16)))
    return {"ms": ms, "tflops": sample["flops"] / (ms * 1e-3) / 1e12, "threads": threads}


def load_traffic(workload_key):
    """DRAM bytes per launch of the main kernel on this workload, from the
    committed ncu summary (profiles/ncu_traffic.json), or None."""
    try:
        with open(os.path.join(REPO, "profiles", "ncu_traffic.json")) as f:
            d = json.load(f)
        e = d.get(workload_key)
        return (float(e["dram_bytes_per_launch"]), e.get("how", "")) if e else (None, "")
    except Exception:
        return None, ""


def native_arm(args, workload_key):
    import torch

    import fmha_native_b200 as fm
    from fmha_native_b200.synth import WORKLOADS, make_inputs

    rank, world, local = dist_env()
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    fm.load_library()
    w = WORKLOADS[workload_key]
    # Weak scaling (default): every rank runs its own copy of the workload on
    # its own data.  --shard (strong scaling): one problem, every rank holds
    # the same inputs and computes its share of the query blocks.
    if world > 1 and not args.weak:
        args.shard = True
    # --emulate-world N: one process runs rank `rank`'s share of an N-rank
    # split (profiling a rank's kernels on one GPU); timing is per share.
    part_world = args.emulate_world if args.emulate_world > 0 else world
    q, k, v, cu = make_inputs(w, dev, seed_base=0 if args.shard else 1000 * rank)
    tiles = None
    share = 1.0
    shard_mode = None
    if args.shard:
        from fmha_native_b200 import shard as shd

        if not w.varlen_seqs and w.batch % part_world == 0 and not args.items:
            # (batch, head) partition: every rank owns a contiguous slice of
            # the batch -- its own Q/K/V/O, nothing replicated, equal work.
            shard_mode = "batch"
            per = w.batch // part_world
            sl = slice(rank * per, (rank + 1) * per)
            q, k, v = q[sl], k[sl], v[sl]
            share = 1.0 / part_world
        else:
            # query-tile partition (few heads, long causal sequences, varlen):
            # LPT over all query blocks, K/V replicated on every rank.
            shard_mode = "tiles"
            blocks = shd.plan_blocks(w.batch, w.heads, w.seqlen, w.seqlen, w.causal,
                                     w.varlen_seqs)
            part = shd.partition(blocks, part_world)[rank]
            tiles = torch.from_numpy(shd.tiles_array(part)).to(dev)
            share = sum(b[2] for b in part) / sum(b[2] for b in blocks)
    splits = 1
    workspace = None
    items = None
    if tiles is not None:
        if not args.items:
            # uniform split-KV (every block cut into `splits` equal KV ranges)
            # when this rank's blocks cannot fill the GPU (long causal, few heads)
            splits = args.splits if args.splits > 0 else shd.choose_splits(tiles.shape[0])
            if splits > 1:
                workspace = torch.empty(fm.splitkv_workspace_bytes(tiles.shape[0], splits) // 4,
                                        device=dev, dtype=torch.float32)
        else:
            # per-block split-KV: blocks longer than ~2 items per CTA slot are cut
            plan = shd.plan_items(part)
            if any(it[3] >= 0 for it in plan):
                items = torch.from_numpy(shd.items_array(plan)).to(dev)
                workspace = torch.empty(fm.items_workspace_bytes(items.shape[0]) // 4,
                                        device=dev, dtype=torch.float32)
    layout = w.layout
    o = torch.empty_like(q)
    lse = None
    if w.lse:
        if w.varlen_seqs:
            lse = torch.empty(w.heads, w.tokens(), device=dev, dtype=torch.float32)
        else:
            lse = torch.empty(q.shape[0], w.heads, w.seqlen, device=dev, dtype=torch.float32)
    max_s = max(w.varlen_seqs) if w.varlen_seqs else None
    params, batch, tq, tk = fm.params_from_tensors(q, k, v, o, lse, layout, cu, cu,
                                                   max_seqlen_q=max_s, max_seqlen_k=max_s)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev, dtype=torch.float32)

    def step():
        if items is not None:
            st = fm.call_items(params, batch, w.causal, items.data_ptr(), items.shape[0],
                               workspace.data_ptr(), workspace.numel() * 4, tq, tk, sh)
        elif tiles is not None and splits > 1:
            st = fm.call_tiles_splitkv(params, batch, w.causal, tiles.data_ptr(), tiles.shape[0],
                                       splits, workspace.data_ptr(), workspace.numel() * 4, tq, tk, sh)
        elif tiles is not None:
            st = fm.call_tiles(params, batch, w.causal, tiles.data_ptr(), tiles.shape[0], tq, tk, sh)
        else:
            st = fm.call_entry(params, batch, w.causal, bool(w.varlen_seqs), tq, tk, sh)
        if st != fm.FMHA_OK:
            raise fm.FmhaError(st, "launch")

    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    if fm.status(sh) != fm.FMHA_OK:
        raise RuntimeError("device pipeline timeout during warmup")

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ
                           else local)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    for i in range(args.steps):
        flush.zero_()  # L2 flush between timed launches (outside the events)
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clocks = sampler.stop()
    kern_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(kern_ms)
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
    if fm.status(sh) != fm.FMHA_OK:
        raise RuntimeError("device pipeline timeout during timed steps")
    ms_step = total_ms / args.steps
    flops_rank = w.flops() * share
    flops_job = w.flops() if args.shard else w.flops() * world
    value = flops_job / (ms_step * 1e-3) / 1e12
    peak_tf, peak_hbm, peak_kind = load_peaks()
    achieved = flops_rank / (statistics.mean(kern_ms) * 1e-3) / 1e12

    if args.launch_only:
        if rank == 0:
            print(json.dumps({"launch_only": True, "workload": w.name,
                              "share_tflops": round(achieved, 2), "share": round(share, 4),
                              "unit": UNIT, "ms_per_step": round(ms_step, 5), "splits": splits,
                              "items": int(items.shape[0]) if items is not None else 0}),
                  flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return 0

    # ---- e2e: host buffers through the public API, copies inside the timed region
    e2e = e2e_measure(fm, w, dev, args, tiles, splits, items,
                      batch_slice=(rank, world) if shard_mode == "batch" else None)
    if world > 1:
        t = torch.tensor([e2e["ms"]], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e["ms"] = float(t.item())
    e2e_value = flops_job / (e2e["ms"] * 1e-3) / 1e12

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w)

    traffic, traffic_how = (args.traffic, "--traffic") if args.traffic else load_traffic(
        args.config)
    if traffic is not None and world > 1:
        traffic = traffic * share  # the committed figure is for the whole problem
    if rank == 0:
        alg_bytes = 2 * (q.numel() + k.numel() + v.numel() + o.numel()) + (
            lse.numel() * 4 if lse is not None else 0)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "strong" if args.shard else "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": w.name, "per_gpu_batch": w.batch if not args.shard else None,
                       "global_batch": w.batch if args.shard else w.batch * world,
                       "heads": w.heads, "kv_heads": w.heads_k, "seq_len": w.seqlen, "head_dim": 64, "causal": w.causal,
                       "lse": w.lse,
                       "splitkv": (f"per-block: {items.shape[0]} items, "
                                   f"{int((items[:, 3] >= 0).sum().item())} partial"
                                   if items is not None else splits),
                       "parallelism": parallelism_desc(shard_mode, world),
                       "l2": "flushed (256 MiB write) between steps"},
            "pct_of_bf16_peak": round(100.0 * (value / world) / peak_tf, 2),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak_tf,
                         "unit": UNIT, "frac": round(achieved / peak_tf, 4),
                         "peak_kind": f"{peak_kind} bf16_tflops (burst)",
                         "alg_bytes_per_launch": alg_bytes, "traffic": traffic,
                         "traffic_source": traffic_how},
            "e2e": {"value": round(e2e_value, 3), "unit": UNIT,
                    "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                    "ms_per_step": round(e2e["ms"], 4), "mode": e2e["mode"]},
            "gpu_launches": args.steps * (2 if (splits > 1 or items is not None) else 1),
            "clocks": clocks,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def parallelism_desc(shard_mode, world):
    if shard_mode == "batch":
        return f"(batch, head) shards: contiguous batch slice per GPU over {world} GPU(s), no collective"
    if shard_mode == "tiles":
        return f"LPT query-block shards over {world} GPU(s), K/V replicated, no collective"
    return f"{world} independent replicas (weak scaling), no collective"


def e2e_measure(fm, w, dev, args, tiles=None, splits=1, items=None, batch_slice=None):
    """Public API with pinned host buffers: H2D of Q,K,V (and cu_seqlens),
    the kernel, D2H of O -- all inside CUDA events on the calling stream.
    Dense problems go through fmha_fwd_from_host (batch chunks, copies on one
    stream overlapping the kernel on another); a (batch, head) shard copies
    only its own batch slice."""
    import torch
    from fmha_native_b200.synth import make_inputs

    q, k, v, cu = make_inputs(w, dev, seed_base=77)
    if batch_slice is not None:
        r, n = batch_slice
        per = w.batch // n
        q, k, v = (t[r * per:(r + 1) * per] for t in (q, k, v))
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hcu = cu.cpu().pin_memory() if cu is not None else None
    ho = torch.empty_like(hq).pin_memory()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    do = torch.zeros_like(q)
    dcu = torch.empty_like(cu) if cu is not None else None
    stream = torch.cuda.current_stream(dev)
    h2d = 3 * hq.numel() * 2 + (hcu.numel() * 4 if hcu is not None else 0)
    d2h = ho.numel() * 2
    max_s = max(w.varlen_seqs) if w.varlen_seqs else None
    pipelined = tiles is None and items is None and not w.varlen_seqs

    def one():
        if pipelined:
            fm.fmha_fwd_from_host(hq, hk, hv, causal=w.causal, layout=w.layout, out=ho,
                                  chunks=min(8, q.shape[0]), device=dev)
            return
        dq.copy_(hq, non_blocking=True)
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
        if dcu is not None:
            dcu.copy_(hcu, non_blocking=True)
        o = fm.fmha_fwd(dq, dk, dv, causal=w.causal, return_lse=False, layout=w.layout,
                        cu_seqlens_q=dcu, cu_seqlens_k=dcu, stream=stream.cuda_stream,
                        out=do, tiles=None if items is not None else tiles,
                        num_splits=splits, items=items, max_seqlen_q=max_s,
                        max_seqlen_k=max_s)
        ho.copy_(o, non_blocking=True)

    for _ in range(2):
        one()
    torch.cuda.synchronize()
    n = max(3, min(args.steps, 10))
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(n):
        one()
    e.record(stream)
    torch.cuda.synchronize()
    return {"ms": s.elapsed_time(e) / n, "h2d": h2d, "d2h": d2h,
            "mode": "chunked overlap (fmha_fwd_from_host)" if pipelined else "serial"}


def cpu_baseline(w):
    try:
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import oracle as O

        sample = cpu_sample(w)
        if O.have_reference():
            res = time_cpu_reference(O, sample, steps=2, warmup=0)
            kind = "reference"
        else:
            return {"value": None, "unit": UNIT, "cores": 0, "kind": "reference",
                    "sample": "unavailable: oracle/_ref not built"}
        return {"value": round(res["tflops"], 6), "unit": UNIT, "cores": res["threads"],
                "kind": kind, "sample": sample["desc"], "ms_per_sample": round(res["ms"], 1),
                "host_cpus": os.cpu_count()}
    except Exception as exc:  # reported, never fatal to the GPU number
        return {"value": None, "unit": UNIT, "cores": 0, "kind": "reference",
                "sample": f"failed: {exc}"}


SWEEP_SIZES = [(8, 16, 1024), (4, 16, 2048), (2, 16, 4096), (1, 8, 8192), (1, 16, 8192),
               (1, 8, 16384), (1, 4, 32768), (1, 2, 40000)]  # run-benchmark.sh:12-21
SWEEP_RUNS, SWEEP_DROP = 6, 1                                 # run-benchmark.sh:23-27


def sweep(args):
    """The reference's performance sweep (scripts/run-benchmark.sh of
    poyenc/fmha_native) on the bench_fmha_fwd CLI: its 8 dense configs plus
    the north-star varlen batch, each run SWEEP_RUNS times, the first dropped
    and the rest averaged; with GPU-count, TFLOPS/GPU and %peak columns and the
    reference's CPU oracle (oracle/_ref cpu_ref_verify) timed on a bounded
    sample of each config on this host."""
    import re

    from fmha_native_b200 import build as kbuild
    from fmha_native_b200.synth import varlen_lengths

    cli = kbuild.build_cli()
    peak_tf, _, peak_kind = load_peaks()
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O

    have_ref = O.have_reference() and not args.no_cpu_baseline
    if have_ref:
        os.environ["OMP_NUM_THREADS"] = str(host_cores())
    rows = [("dense", b, h, s, None) for b, h, s in SWEEP_SIZES]
    vl = varlen_lengths()
    rows.append(("varlen", len(vl), 16, max(vl), vl))
    print(f"Sweep: {len(rows)} configs, mask={args.mask}, gpus={args.gpus}, "
          f"runs={SWEEP_RUNS} (drop {SWEEP_DROP}), peak {peak_tf} TFLOP/s ({peak_kind})")
    hdr = (f"{'B':>4} {'H':>3} {'S':>6} {'D':>4} | {'Avg(ms)':>10} {'Min(ms)':>10} {'TFLOPS':>10} | "
           f"{'GPUs':>4} {'TFLOPS/GPU':>10} {'%peak':>6} | {'CPU_ms':>9} {'CPU_threads':>11}")
    print(hdr)
    print("-" * len(hdr))
    results = []
    for kind, b, h, s, seqs in rows:
        cmd = [cli, "-b", str(b), "-h", str(h), "-s", str(s), "-d", "64", "--mask", str(args.mask),
               "--warmup", "5", "--iters", "20", "--gpus", str(args.gpus), "--peak", str(peak_tf)]
        if seqs:
            cmd += ["--varlen-seqs", ",".join(str(x) for x in seqs)]
        vals = {"avg": [], "min": [], "tf": []}
        err = None
        for run in range(SWEEP_RUNS):
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                err = (r.stderr or r.stdout).strip().splitlines()[-1:] or [f"exit {r.returncode}"]
                break
            if run < SWEEP_DROP:
                continue
            vals["avg"].append(float(re.search(r"^Avg: ([0-9.]+)", r.stdout, re.M).group(1)))
            vals["min"].append(float(re.search(r"^min=([0-9.]+)", r.stdout, re.M).group(1)))
            vals["tf"].append(float(re.search(r"^TFLOPS: ([0-9.]+)", r.stdout, re.M).group(1)))
        cpu_ms, cpu_thr = None, None
        if have_ref and err is None:
            from fmha_native_b200.synth import Workload

            w = Workload("sweep", b, h, s, bool(args.mask), False,
                         layout="thd" if seqs else "bshd", varlen_seqs=tuple(seqs) if seqs else None)
            res = time_cpu_reference(O, cpu_sample(w), steps=1, warmup=0)
            cpu_ms, cpu_thr = res["ms"], res["threads"]
        if err is None:
            avg = sum(vals["avg"]) / len(vals["avg"])
            mn = min(vals["min"])
            tf = sum(vals["tf"]) / len(vals["tf"])
            line = (f"{b:>4} {h:>3} {s:>6} {64:>4} | {avg:>10.3f} {mn:>10.3f} {tf:>10.2f} | "
                    f"{args.gpus:>4} {tf / args.gpus:>10.2f} {100 * tf / args.gpus / peak_tf:>6.1f} | "
                    f"{cpu_ms if cpu_ms is None else round(cpu_ms, 1)!s:>9} {cpu_thr!s:>11}")
            results.append({"kind": kind, "b": b, "h": h, "s": s, "mask": args.mask,
                            "avg_ms": round(avg, 4), "min_ms": mn, "tflops": round(tf, 2),
                            "gpus": args.gpus, "pct_peak": round(100 * tf / args.gpus / peak_tf, 2),
                            "cpu_sample_ms": cpu_ms, "cpu_threads": cpu_thr})
        else:
            line = f"{b:>4} {h:>3} {s:>6} {64:>4} | ERROR: {err[0]}"
        print(line, flush=True)
    print(json.dumps({"sweep": results, "peak_tflops": peak_tf, "peak_kind": peak_kind}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c5b",
                    help="north-star workload (fmha_native_b200.synth.WORKLOADS)")
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--splits", type=int, default=0,
                    help="split-KV factor for --shard (0 = automatic)")
    ap.add_argument("--items", action="store_true",
                    help="with --shard: per-block split-KV work items (shard.plan_items) "
                         "instead of uniform splits")
    ap.add_argument("--shard", action="store_true",
                    help="strong scaling: split one problem over the ranks (default for N>1)")
    ap.add_argument("--weak", action="store_true",
                    help="N>1: every rank runs its own copy of the workload (weak scaling)")
    ap.add_argument("--traffic", type=float, default=None,
                    help="ncu dram bytes per launch to report in roofline.traffic")
    ap.add_argument("--launch-only", action="store_true",
                    help="time the kernel launches only (no e2e, no CPU leg): profiling runs")
    ap.add_argument("--emulate-world", type=int, default=0,
                    help="with --shard on one process: run rank 0's share of an N-rank split")
    ap.add_argument("--sweep", action="store_true",
                    help="the reference's 8-config sweep (+ varlen) on the bench_fmha_fwd CLI")
    ap.add_argument("--mask", type=int, default=0, help="--sweep: causal mask 0|1")
    args = ap.parse_args()
    if args.sweep:
        return sweep(args)
    if args.impl == "reference":
        return reference_arm(args, args.config)
    return native_arm(args, args.config)


if __name__ == "__main__":
    sys.exit(main())
