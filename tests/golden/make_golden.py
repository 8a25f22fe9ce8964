"""Generates the golden parity fixtures in this directory.

Each fixture holds the bf16 input bits of a small case, the oracle output
(O_ref fp32 and LSE fp32 from oracle/fmha_oracle.c) and the verdict of the
REFERENCE's own cpu_ref_verify (src/runner/cpu_ref.cpp, compiled from the
reference sources into oracle/_ref) on the bf16-rounded oracle output:
its pass flag, max_abs, and O_ref value at its worst location, which must
equal the restatement's value there bit for bit.

Run (needs oracle/_ref built, i.e. a container with the reference tree):
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import oracle as O  # noqa: E402

D = 64

# name, B, Hq, Hk, S, Sk, causal, varlen, input kind
CASES = [
    ("D64Smoke2", 1, 1, 1, 256, 256, 0, (), "ref42"),
    ("D64EdgeS33MaskLse", 1, 2, 2, 33, 33, 1, (), "ref42"),
    ("D64AsymSqLtSkvMaskLse_small", 1, 2, 2, 64, 160, 1, (), "ref42"),
    ("D64GqaMask_small", 1, 4, 2, 100, 100, 1, (), "ref42"),
    ("D64VarlenTinyMaskLse", 4, 2, 2, 512, 512, 1, (1, 512, 32, 256), "ref42"),
    ("BaselineC1_B1H2S256_uniform", 1, 2, 2, 256, 256, 0, (), "uniform012"),
    ("CkClosedForm_17x33", 1, 1, 1, 17, 33, 0, (), "closed"),
]


def rne_bits(o):
    u = o.astype(np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def inputs(kind, B, Hq, Hk, S, Sk, varlen):
    if varlen:
        tot = sum(varlen)
        nq, nk = Hq * tot * D, Hk * tot * D
    else:
        nq, nk = B * Hq * S * D, B * Hk * Sk * D
    if kind == "ref42":
        return O.fill_random(42, nq, nk, nk)
    if kind == "uniform012":
        out = []
        for seed, n in ((0, nq), (1, nk), (2, nk)):
            rng = np.random.default_rng(seed)
            out.append(O.f32_to_bf16_bits_trunc((rng.random(n, dtype=np.float32) * 2 - 1)))
        return tuple(out)
    iq, ik = np.arange(nq), np.arange(nk)
    return (O.f32_to_bf16_bits_trunc(((iq % 256) / 256.0).astype(np.float32)),
            O.f32_to_bf16_bits_trunc((((ik + 64) % 256) / 256.0).astype(np.float32)),
            O.f32_to_bf16_bits_trunc(((ik % 256) / 256.0 + 1.0).astype(np.float32)))


def run_case(name, B, Hq, Hk, S, Sk, causal, varlen, kind):
    q, k, v = inputs(kind, B, Hq, Hk, S, Sk, varlen)
    if varlen:
        tot = sum(varlen)
        ss = np.concatenate([[0], np.cumsum(varlen)]).astype(np.int32)
        st = (D, tot * D, 0)
        o, lse = O.oracle_fwd(q, k, v, batch=len(varlen), nhead_q=Hq, nhead_k=Hk, seqlen_q=max(varlen),
                              seqlen_k=max(varlen), causal=causal, strides_q=st, strides_k=st,
                              strides_v=st, out_shape=(Hq, tot, D), strides_o=st, seqstart_q=ss,
                              seqstart_k=ss, total_q=tot)
    else:
        stq, stk = (D, S * D, Hq * S * D), (D, Sk * D, Hk * Sk * D)
        o, lse = O.oracle_fwd(q, k, v, batch=B, nhead_q=Hq, nhead_k=Hk, seqlen_q=S, seqlen_k=Sk,
                              causal=causal, strides_q=stq, strides_k=stk, strides_v=stk,
                              out_shape=(B, Hq, S, D), strides_o=stq)
    return q, k, v, o, lse


def main():
    for name, B, Hq, Hk, S, Sk, causal, varlen, kind in CASES:
        q, k, v, o, lse = run_case(name, B, Hq, Hk, S, Sk, causal, varlen, kind)
        rv = O.ref_verify(len(varlen) if varlen else B, Hq, Hk, S, Sk, causal, list(varlen),
                          q, k, v, rne_bits(o).ravel())
        if varlen:
            ss = np.concatenate([[0], np.cumsum(varlen)])
            mine = o[rv.worst_h, ss[rv.worst_b] + rv.worst_i, rv.worst_d]
        else:
            mine = o[rv.worst_b, rv.worst_h, rv.worst_i, rv.worst_d]
        # O in [1, 2) (closed-form case) has bf16 spacing 2^-7 > the 1e-3 rule,
        # so only the O_ref value itself is compared there.
        assert np.float32(mine) == np.float32(rv.worst_ref), (name, rv.max_abs)
        assert rv.pass_ == 1 or kind == "closed", (name, rv.max_abs)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"), q=q, k=k, v=v, o_ref=o, lse_ref=lse,
            meta=np.array([B, Hq, Hk, S, Sk, causal], np.int64), varlen=np.array(varlen, np.int64),
            ref_pass=np.int64(rv.pass_), ref_max_abs=np.float64(rv.max_abs),
            ref_worst=np.array([rv.worst_b, rv.worst_h, rv.worst_i, rv.worst_d], np.int64),
            ref_worst_ref=np.float32(rv.worst_ref))
        print(f"{name}: reference verdict {rv.pass_}, max_abs {rv.max_abs:.3e}, worst O_ref {rv.worst_ref}")


if __name__ == "__main__":
    main()
