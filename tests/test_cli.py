"""The C++ bench_fmha_fwd CLI (reference command line and output lines)."""
from __future__ import annotations

import os
import re
import subprocess

import pytest

from fmha_native_b200 import build as kbuild


def test_cli_builds_and_prints_usage():
    exe = kbuild.build_cli()
    out = subprocess.run([exe, "--help"], capture_output=True, text=True, timeout=60).stdout
    for flag in ("--batch", "--heads", "--kv-heads", "--seq", "--hdim", "--mask", "--lse",
                 "--varlen-seqs", "--warmup", "--iters", "--gpus", "--peak", "--verify"):
        assert flag in out


def test_cli_rejects_other_head_dims():
    exe = kbuild.build_cli()
    r = subprocess.run([exe, "-d", "128"], capture_output=True, text=True, timeout=60)
    assert r.returncode != 0 and "head_dim 64" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("args", [["-b", "2", "-h", "4", "-s", "1024"],
                                  ["-b", "1", "-h", "8", "--kv-heads", "2", "-s", "2048", "--mask", "1", "--lse", "1"],
                                  ["-h", "4", "--varlen-seqs", "300,1024,17", "--mask", "1"]])
def test_cli_runs_and_reports(cuda_device, args):
    exe = kbuild.build_cli()
    r = subprocess.run([exe, *args, "--warmup", "2", "--iters", "3"], capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert re.search(r"^Avg: [0-9.]+ ms$", r.stdout, re.M)
    assert re.search(r"^min=[0-9.]+ ms$", r.stdout, re.M)
    assert float(re.search(r"^TFLOPS: ([0-9.]+)$", r.stdout, re.M).group(1)) > 0
    assert re.search(r"^GPUS: 1$", r.stdout, re.M)
    assert re.search(r"^TFLOPS/GPU: [0-9.]+$", r.stdout, re.M)
    assert re.search(r"^%peak: [0-9.]+$", r.stdout, re.M)


@pytest.mark.gpu
@pytest.mark.parametrize("args", [["-b", "2", "-h", "4", "-s", "700", "--mask", "1"],
                                  ["-h", "4", "--kv-heads", "2", "--varlen-seqs", "300,1024,17"]])
def test_cli_verify_passes(cuda_device, args):
    """--verify recomputes sampled rows on the host (fp64 softmax, P truncated
    to bf16) and checks the north-star bars; the sharded path (--gpus) is the
    same kernel on each GPU's own list, so one GPU checks the gather logic with
    the full problem."""
    import torch

    exe = kbuild.build_cli()
    gpus = min(2, torch.cuda.device_count())
    r = subprocess.run([exe, *args, "--warmup", "1", "--iters", "2", "--verify", "3",
                        "--gpus", str(gpus)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert re.search(r"^VERIFY: .* PASS$", r.stdout, re.M), r.stdout
    assert re.search(rf"^GPUS: {gpus}$", r.stdout, re.M)
