"""CPU tests: the oracle restatement is pinned to the reference.

* Golden fixtures (tests/golden/*.npz, made by make_golden.py): recomputing
  the C restatement on the stored inputs reproduces the stored O_ref / LSE
  bit for bit, and the stored reference verdict says the reference's own
  cpu_ref_verify agreed with it.
* Where oracle/_ref (the reference's cpu_ref.cpp + buffers.cpp compiled from
  its sources) is present, the checks are re-run live: the generator matches
  FmhaBuffers::fill_random, and cpu_ref_verify accepts the restatement and
  reports the same O_ref at its worst location.
"""
from __future__ import annotations

import glob
import os

import numpy as np
import pytest

import oracle as O
from cases import FULL_CASES

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))
D = 64


def _oracle_for(z):
    B, Hq, Hk, S, Sk, causal = (int(x) for x in z["meta"])
    varlen = tuple(int(x) for x in z["varlen"])
    q, k, v = z["q"], z["k"], z["v"]
    if varlen:
        tot = sum(varlen)
        ss = np.concatenate([[0], np.cumsum(varlen)]).astype(np.int32)
        st = (D, tot * D, 0)
        return O.oracle_fwd(q, k, v, batch=len(varlen), nhead_q=Hq, nhead_k=Hk, seqlen_q=max(varlen),
                            seqlen_k=max(varlen), causal=causal, strides_q=st, strides_k=st,
                            strides_v=st, out_shape=(Hq, tot, D), strides_o=st, seqstart_q=ss,
                            seqstart_k=ss, total_q=tot)
    stq, stk = (D, S * D, Hq * S * D), (D, Sk * D, Hk * Sk * D)
    return O.oracle_fwd(q, k, v, batch=B, nhead_q=Hq, nhead_k=Hk, seqlen_q=S, seqlen_k=Sk,
                        causal=causal, strides_q=stq, strides_k=stk, strides_v=stk,
                        out_shape=(B, Hq, S, D), strides_o=stq)


def test_golden_fixtures_present():
    assert len(GOLDEN) >= 7


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_oracle_reproduces_golden(path):
    z = np.load(path)
    o, lse = _oracle_for(z)
    assert np.array_equal(o.view(np.uint32), z["o_ref"].view(np.uint32))
    assert np.array_equal(lse.view(np.uint32), z["lse_ref"].view(np.uint32))
    # The stored verdict of the reference's own cpu_ref_verify.
    b, h, i, d = (int(x) for x in z["ref_worst"])
    varlen = tuple(int(x) for x in z["varlen"])
    if varlen:
        ss = np.concatenate([[0], np.cumsum(varlen)])
        mine = o[h, ss[b] + i, d]
    else:
        mine = o[b, h, i, d]
    assert np.float32(mine) == z["ref_worst_ref"]
    if "Closed" not in path:
        assert int(z["ref_pass"]) == 1


@pytest.mark.skipif(not O.have_reference(), reason="oracle/_ref not built")
@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_reference_agrees_live(path):
    z = np.load(path)
    B, Hq, Hk, S, Sk, causal = (int(x) for x in z["meta"])
    varlen = [int(x) for x in z["varlen"]]
    o = z["o_ref"]
    u = o.astype(np.float32).view(np.uint32).astype(np.uint64)
    bits = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    rv = O.ref_verify(len(varlen) if varlen else B, Hq, Hk, S, Sk, causal, varlen,
                      z["q"], z["k"], z["v"], bits.ravel())
    assert np.float32(rv.worst_ref) == z["ref_worst_ref"]
    assert rv.max_abs == pytest.approx(float(z["ref_max_abs"]), abs=0)


SMALL = [c for c in FULL_CASES if (c.b * c.h * c.s * max(c.s, c.kv_seq) <= 2 ** 22)]


@pytest.mark.skipif(not O.have_reference(), reason="oracle/_ref not built")
@pytest.mark.parametrize("case", SMALL, ids=[c.name for c in SMALL])
def test_generator_matches_reference(case):
    import fmha_native_b200 as fm

    p = fm.make_params(case.b, case.h, case.s, case.d, case.kv_heads, case.kv_seq, case.mask,
                       case.lse, case.varlen)
    q, k, v = O.ref_fill_random(p.batch, p.q_heads, p.kv_heads, p.seq_len, p.kv_seq_len,
                                list(p.varlen_seqs), 42)
    q2, k2, v2 = O.fill_random(42, q.size, k.size, v.size)
    assert np.array_equal(q, q2) and np.array_equal(k, k2) and np.array_equal(v, v2)


def test_compare_rules():
    ref = np.full((2, 64), 0.5, np.float32)
    ker = ref.copy()
    v = O.compare(ker, ref)
    assert v["ref_pass"] and v["baseline_pass"] and v["max_abs"] == 0
    ker[0, 3] += 2e-3
    v = O.compare(ker, ref)
    assert not v["ref_pass"] and v["mismatch"] == 1 and v["baseline_pass"]
    ker[0, 3] = np.nan
    v = O.compare(ker, ref)
    assert v["nonfinite"] == 1 and not v["baseline_pass"]
    lse = np.array([1.0, -np.inf], np.float32)
    v = O.compare(ref, ref, lse, lse)
    assert v["lse_pass"]
