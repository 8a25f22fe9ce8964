"""Host-buffer entry (fmha_native_b200.fmha_fwd_from_host): pinned host Q/K/V
in, pinned host O out, the batch in chunks over three streams.  Its result
must be bit-identical to the device entry's on the same inputs, for every
chunking, twice in a row (the staging buffers are reused)."""
from __future__ import annotations

import pytest

import fmha_native_b200 as fm
from fmha_native_b200.synth import Workload, make_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("causal,chunks,layout", [(False, 1, "bshd"), (True, 3, "bshd"),
                                                  (True, 8, "bhsd")])
def test_from_host_matches_device_entry(cuda_device, causal, chunks, layout):
    import torch

    w = Workload("h", 5, 4, 700, causal, False)
    q, k, v, _ = make_inputs(w, cuda_device, seed_base=41)
    if layout == "bhsd":
        q, k, v = (t.transpose(1, 2).contiguous() for t in (q, k, v))
    ref = fm.fmha_fwd(q, k, v, causal=causal, layout=layout)
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    for _ in range(2):
        out = fm.fmha_fwd_from_host(hq, hk, hv, causal=causal, layout=layout, chunks=chunks,
                                    device=cuda_device)
        torch.cuda.current_stream(cuda_device).synchronize()
        assert torch.equal(out.view(torch.int16), ref.cpu().view(torch.int16))
