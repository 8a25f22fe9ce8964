"""The trace build of the kernel (libfmha_b200_trace.so, -DFMHA_TRACE) and
its timeline summary (fmha_native_b200.trace)."""
import ctypes
import os

import numpy as np
import pytest

from fmha_native_b200 import build as kbuild
from fmha_native_b200 import trace

TRACE_SYMBOLS = ("fmha_fwd_d64_trace_shape", "fmha_fwd_d64_trace_configure",
                 "fmha_fwd_d64_trace_read")


def _synthetic(n_steps=10, period=3000):
    """One CTA whose events sit at fixed offsets inside each step."""
    t = np.zeros((2, 64, 16), dtype=np.int64)
    off = {0: -200, 1: 0, 2: 1800, 3: 2100, 4: 2300, 5: 600, 6: 2600, 9: 400, 11: 2450,
           12: -700, 13: 3100, 14: -1900, 8: 250}
    for j in range(n_steps):
        base = 10000 + j * period
        for slot, o in off.items():
            t[0, j, slot] = base + o
    return t


def test_summary_of_a_known_timeline():
    s = trace.summarize(_synthetic())
    seg = s["segments"]
    assert s["ctas"] == 1
    assert seg["softmax: period (s_free(j) -> s_free(j+1))"] == 3000
    assert seg["softmax: S(j) TMEM load + s_free"] == 200
    assert seg["softmax: exponential pass issued"] == 1800
    assert seg["softmax: p_full(j) -> S(j+1) seen"] == 3000 - 200 - 2300
    assert seg["tensor: S(j+1) issue -> complete"] == 3000 - 700 - 600
    assert seg["slack: PV(j-1) complete before softmax needs it"] == 2100 - (3100 - 3000)


def test_short_ctas_are_skipped():
    assert trace.summarize(_synthetic(n_steps=4))["ctas"] == 0


def test_product_library_has_no_trace_hooks():
    lib = ctypes.CDLL(kbuild.build_library())
    for name in TRACE_SYMBOLS:
        assert not hasattr(lib, name), name


def test_trace_library_exports():
    path = kbuild.build_trace_library()
    lib = ctypes.CDLL(path)
    for name in TRACE_SYMBOLS + ("fmha_fwd_d64_bf16_msk0", "fmha_fwd_d64_bf16_tiles"):
        assert hasattr(lib, name), name


@pytest.mark.gpu
def test_trace_capture_matches_product_and_is_ordered(cuda_device):
    """The traced launch gives bit-identical O, and the stamps respect the
    pipeline's dependencies (an MMA completes after it is issued; one
    thread's events are in program order)."""
    import torch

    import fmha_native_b200 as fm
    from fmha_native_b200.synth import WORKLOADS, make_inputs

    t, o_tr = trace.capture("c2", first_cta=0)
    w = WORKLOADS["c2"]
    q, k, v, _ = make_inputs(w, cuda_device)
    o = fm.fmha_fwd(q, k, v, causal=w.causal)
    torch.cuda.synchronize()
    assert torch.equal(o.view(torch.int16), o_tr.view(torch.int16))
    n = 2048 // 128
    traced = 0
    for c in range(t.shape[0]):
        if t[c, 0, 4] == 0:
            continue
        traced += 1
        T = t[c]
        assert (T[:n, 4] > 0).all() and (T[n:, 4] == 0).all()
        for j in range(n):
            assert T[j, 0] <= T[j, 1] <= T[j, 2] <= T[j, 3] <= T[j, 4]
            assert T[j, 6] <= T[j, 13]
            if j + 1 < n:
                assert T[j, 5] <= T[j + 1, 12]
                assert T[j, 4] <= T[j + 1, 0]
    assert traced == t.shape[0]
    s = trace.summarize(t)
    assert s["ctas"] == traced
    per = s["segments"]["softmax: period (s_free(j) -> s_free(j+1))"]
    assert 500 < per < 20000
