"""Shared GPU-parity harness: run one case through the C ABI and check it
against the oracle (the C restatement) and, where built, the reference's own
cpu_ref_verify.  Mirrors the reference test body
tests/test_fmha_fwd_d64.cpp:500-653 (MatchesGpuRef)."""
from __future__ import annotations

import ctypes

import numpy as np

import fmha_native_b200 as fm
import oracle as O

D = 64


def to_device_bf16(bits: np.ndarray, shape, device):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).reshape(shape))
    return t.to(device).view(torch.bfloat16)


def from_device_bf16(t) -> np.ndarray:
    import torch

    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def run_reference_layout_case(case, device, seed: int = 42, check_reference: bool = True,
                              row_step: int = 1):
    """Reference-layout case (BHSD dense or [H,total,D] varlen), inputs from
    the reference generator.  Returns the verdict dict."""
    import torch

    p = fm.make_params(case.b, case.h, case.s, case.d, case.kv_heads, case.kv_seq, case.mask,
                       case.lse, case.varlen)
    varlen = bool(p.varlen_seqs)
    Hq, Hk = p.q_heads, p.kv_heads
    if varlen:
        total = sum(p.varlen_seqs)
        nq, nk = Hq * total * D, Hk * total * D
        q_shape, k_shape = (Hq, total, D), (Hk, total, D)
        ss = np.concatenate([[0], np.cumsum(p.varlen_seqs)]).astype(np.int32)
    else:
        nq = p.batch * Hq * p.seq_len * D
        nk = p.batch * Hk * p.kv_seq_len * D
        q_shape = (p.batch, Hq, p.seq_len, D)
        k_shape = (p.batch, Hk, p.kv_seq_len, D)
    q, k, v = O.fill_random(seed, nq, nk, nk)

    qd = to_device_bf16(q, q_shape, device)
    kd = to_device_bf16(k, k_shape, device)
    vd = to_device_bf16(v, k_shape, device)
    od = torch.full(q_shape, float("nan"), device=device, dtype=torch.bfloat16)
    lse_d = None
    if case.lse:
        lse_shape = (Hq, total) if varlen else (p.batch, Hq, p.seq_len)
        lse_d = torch.full(lse_shape, float("nan"), device=device, dtype=torch.float32)
    if varlen:
        ss_d = torch.from_numpy(ss).to(device)
        params, batch, tq, tk = fm.params_from_tensors(qd, kd, vd, od, lse_d, "htd", ss_d, ss_d)
    else:
        params, batch, tq, tk = fm.params_from_tensors(qd, kd, vd, od, lse_d, "bhsd")
    st = fm.call_entry(params, batch, bool(case.mask), varlen, tq, tk,
                       torch.cuda.current_stream().cuda_stream)
    assert st == fm.FMHA_OK, f"launch status {st}"
    torch.cuda.synchronize()
    assert fm.status(0) == fm.FMHA_OK
    o_bits = from_device_bf16(od)
    o_k = O.bf16_bits_to_f32(o_bits).reshape(q_shape)

    if varlen:
        st_q = (D, total * D, 0)
        st_k = (D, total * D, 0)
        o_ref, lse_ref = O.oracle_fwd(q, k, v, batch=p.batch, nhead_q=Hq, nhead_k=Hk,
                                      seqlen_q=p.seq_len, seqlen_k=p.kv_seq_len, causal=p.mask,
                                      strides_q=st_q, strides_k=st_k, strides_v=st_k,
                                      out_shape=q_shape, strides_o=st_q, seqstart_q=ss,
                                      seqstart_k=ss, total_q=total, with_lse=bool(case.lse),
                                      row_step=row_step)
    else:
        st_q = (D, p.seq_len * D, Hq * p.seq_len * D)
        st_k = (D, p.kv_seq_len * D, Hk * p.kv_seq_len * D)
        o_ref, lse_ref = O.oracle_fwd(q, k, v, batch=p.batch, nhead_q=Hq, nhead_k=Hk,
                                      seqlen_q=p.seq_len, seqlen_k=p.kv_seq_len, causal=p.mask,
                                      strides_q=st_q, strides_k=st_k, strides_v=st_k,
                                      out_shape=q_shape, strides_o=st_q, with_lse=bool(case.lse),
                                      row_step=row_step)
    lse_k = lse_d.cpu().numpy() if lse_d is not None else None
    verdict = O.compare(o_k, o_ref, lse_k, lse_ref)
    if check_reference and O.have_reference() and row_step == 1:
        rv = O.ref_verify(p.batch, Hq, Hk, p.seq_len, p.kv_seq_len, p.mask, p.varlen_seqs,
                          q, k, v, o_bits.ravel())
        verdict["reference_cpu_ref_verify"] = bool(rv.pass_)
        verdict["reference_max_abs"] = rv.max_abs
    return verdict
