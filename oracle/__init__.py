"""TEST INFRASTRUCTURE ONLY -- parity checkers for the B200 FMHA forward.

Importable only from tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg.  Nothing in the product package imports this module.

* :func:`fill_random` / :func:`oracle_fwd` bind ``liboracle.so``, the C
  restatement of the reference oracle (``fmha_oracle.c``, which cites the
  reference lines it follows).
* :func:`ref_fill_random` / :func:`ref_verify` bind ``_ref/libfmha_ref.so``,
  the reference's own ``cpu_ref_verify`` and ``FmhaBuffers::fill_random``
  compiled from its sources (present when built in a container that mounts
  the reference tree; the built ``.so`` travels with the repository).
* :func:`compare` computes the verdicts: the reference's own pass rule
  (src/runner/cpu_ref.cpp:26-28, 246-247: every |dO| <= 1e-3, max relative
  error <= 0.05 over |ref| >= 0.01, per-row cosine >= 0.99995, no non-finite)
  and the north-star rule (max-abs <= 2e-2, rel-L2 <= 5e-3; LSE |d| <= 1e-3).
"""
from __future__ import annotations

import contextlib
import ctypes
import os
from typing import Optional, Sequence

import numpy as np

ORACLE_DIR = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(ORACLE_DIR, "liboracle.so")
REF_LIB = os.path.join(ORACLE_DIR, "_ref", "libfmha_ref.so")

# Tolerances.
REF_TOL_ABS = 1e-3        # cpu_ref.cpp:26
REF_TOL_REL = 0.05        # cpu_ref.cpp:27 (|ref| >= 0.01)
REF_TOL_COS = 0.99995     # cpu_ref.cpp:28
LSE_TOL_ABS = 1e-3        # tests/test_fmha_fwd_d64.cpp:634
BASE_TOL_MAX_ABS = 2e-2
BASE_TOL_REL_L2 = 5e-3


class OracleProblem(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int), ("nhead_q", ctypes.c_int), ("nhead_k", ctypes.c_int),
        ("seqlen_q", ctypes.c_int), ("seqlen_k", ctypes.c_int), ("causal", ctypes.c_int),
        ("stride_q", ctypes.c_longlong), ("nhead_stride_q", ctypes.c_longlong),
        ("batch_stride_q", ctypes.c_longlong),
        ("stride_k", ctypes.c_longlong), ("nhead_stride_k", ctypes.c_longlong),
        ("batch_stride_k", ctypes.c_longlong),
        ("stride_v", ctypes.c_longlong), ("nhead_stride_v", ctypes.c_longlong),
        ("batch_stride_v", ctypes.c_longlong),
        ("stride_o", ctypes.c_longlong), ("nhead_stride_o", ctypes.c_longlong),
        ("batch_stride_o", ctypes.c_longlong),
        ("seqstart_q", ctypes.c_void_p), ("seqstart_k", ctypes.c_void_p),
        ("total_q", ctypes.c_int),
        ("row_step", ctypes.c_int), ("row_phase", ctypes.c_int),
    ]


class RefVerdict(ctypes.Structure):
    _fields_ = [
        ("pass_", ctypes.c_int),
        ("max_abs", ctypes.c_double), ("max_rel", ctypes.c_double),
        ("min_cos", ctypes.c_double), ("mean_cos", ctypes.c_double),
        ("mismatch", ctypes.c_ulonglong), ("nonfinite", ctypes.c_ulonglong),
        ("total_elems", ctypes.c_ulonglong), ("cos_fail", ctypes.c_ulonglong),
        ("cos_rows", ctypes.c_ulonglong),
        ("worst_b", ctypes.c_int), ("worst_h", ctypes.c_int), ("worst_i", ctypes.c_int),
        ("worst_d", ctypes.c_int),
        ("worst_ref", ctypes.c_float), ("worst_kern", ctypes.c_float),
    ]


_olib = None
_rlib = None


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def oracle_lib() -> ctypes.CDLL:
    global _olib
    if _olib is None:
        if not os.path.exists(ORACLE_LIB):
            from . import build as _b  # noqa: F401  (oracle/build.py)
            _b.build_oracle()
        _olib = ctypes.CDLL(ORACLE_LIB)
        _olib.oracle_fill_random.argtypes = [ctypes.c_uint] + [ctypes.c_void_p, ctypes.c_size_t] * 3
        _olib.oracle_fill_random.restype = None
        _olib.oracle_srand.argtypes = [ctypes.c_uint]
        _olib.oracle_fill_rand_bf16.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        _olib.oracle_fmha_fwd.argtypes = [ctypes.POINTER(OracleProblem)] + [ctypes.c_void_p] * 5
        _olib.oracle_fmha_fwd.restype = None
    return _olib


def have_reference() -> bool:
    return os.path.exists(REF_LIB)


def ref_lib() -> ctypes.CDLL:
    global _rlib
    if _rlib is None:
        if not have_reference():
            raise FileNotFoundError(REF_LIB)
        _rlib = ctypes.CDLL(REF_LIB)
        I = ctypes.c_int
        _rlib.ref_sizes.argtypes = [I, I, I, I, I, ctypes.c_void_p, I, ctypes.c_void_p]
        _rlib.ref_fill_random.argtypes = [I, I, I, I, I, ctypes.c_void_p, I, ctypes.c_uint,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _rlib.ref_verify.argtypes = [I, I, I, I, I, I, ctypes.c_void_p, I] + [ctypes.c_void_p] * 4 + \
            [ctypes.POINTER(RefVerdict)]
        _rlib.ref_verify.restype = I
    return _rlib


@contextlib.contextmanager
def quiet_stdout():
    """Silence C-level stdout (the reference oracle prints its report)."""
    import sys
    sys.stdout.flush()
    fd = os.dup(1)
    devnull = os.open(os.devnull, os.O_WRONLY)
    os.dup2(devnull, 1)
    try:
        yield
    finally:
        os.dup2(fd, 1)
        os.close(fd)
        os.close(devnull)


# ----------------------------------------------------------------- inputs

def fill_random(seed: int, nq: int, nk: int, nv: int):
    """Reference input generator restated (buffers.cpp:99-127): Q, K, V bf16
    bit patterns from glibc srand(seed)/rand()."""
    lib = oracle_lib()
    q = np.empty(nq, np.uint16)
    k = np.empty(nk, np.uint16)
    v = np.empty(nv, np.uint16)
    lib.oracle_fill_random(seed, _ptr(q), nq, _ptr(k), nk, _ptr(v), nv)
    return q, k, v


def rand_bf16_stream(seed: int, counts: Sequence[int]):
    """One srand(seed), then consecutive glibc-rand bf16 fills of each count
    (the reference smoke tests' inline generator, test_fmha_fwd_d64.cpp:212-215)."""
    lib = oracle_lib()
    lib.oracle_srand(seed)
    out = []
    for n in counts:
        a = np.empty(n, np.uint16)
        lib.oracle_fill_rand_bf16(_ptr(a), n)
        out.append(a)
    return out


def ref_fill_random(batch, q_heads, kv_heads, seq_len, kv_seq_len, varlen_seqs, seed):
    """The reference's own FmhaBuffers::fill_random (needs _ref)."""
    lib = ref_lib()
    vl = np.asarray(varlen_seqs, np.int32) if varlen_seqs else np.zeros(1, np.int32)
    n = len(varlen_seqs) if varlen_seqs else 0
    sizes = np.zeros(3, np.uint64)
    lib.ref_sizes(batch, q_heads, kv_heads, seq_len, kv_seq_len, _ptr(vl), n, _ptr(sizes))
    q = np.empty(int(sizes[0]), np.uint16)
    k = np.empty(int(sizes[1]), np.uint16)
    v = np.empty(int(sizes[1]), np.uint16)
    lib.ref_fill_random(batch, q_heads, kv_heads, seq_len, kv_seq_len, _ptr(vl), n, seed,
                        _ptr(q), _ptr(k), _ptr(v))
    return q, k, v


def ref_verify(batch, q_heads, kv_heads, seq_len, kv_seq_len, mask, varlen_seqs, q, k, v, o,
               quiet: bool = True) -> RefVerdict:
    """Run the reference's own cpu_ref_verify on bf16 output `o` (reference
    layouts: BHSD dense, [H,total,D] varlen)."""
    lib = ref_lib()
    vl = np.asarray(varlen_seqs, np.int32) if varlen_seqs else np.zeros(1, np.int32)
    n = len(varlen_seqs) if varlen_seqs else 0
    res = RefVerdict()
    args = [np.ascontiguousarray(x, dtype=np.uint16) for x in (q, k, v, o)]
    ctx = quiet_stdout() if quiet else contextlib.nullcontext()
    with ctx:
        lib.ref_verify(batch, q_heads, kv_heads, seq_len, kv_seq_len, mask, _ptr(vl), n,
                       *[_ptr(a) for a in args], ctypes.byref(res))
    return res


# ----------------------------------------------------------------- oracle

def oracle_fwd(q: np.ndarray, k: np.ndarray, v: np.ndarray, *, batch: int, nhead_q: int,
               nhead_k: int, seqlen_q: int, seqlen_k: int, causal: bool,
               strides_q, strides_k, strides_v, out_shape, strides_o,
               seqstart_q: Optional[np.ndarray] = None, seqstart_k: Optional[np.ndarray] = None,
               total_q: int = 0, with_lse: bool = True, row_step: int = 1, row_phase: int = 0,
               lse_shape=None):
    """C restatement of cpu_ref.cpp:86-144 (+ gpu_ref.cpp:116-125 LSE).

    q/k/v: flat uint16 bf16 arrays addressed by (row, head, batch) element
    strides.  Returns (o_ref float32 array of `out_shape` addressed with
    `strides_o`, lse float32 or None).  Rows skipped by row_step are NaN.
    """
    lib = oracle_lib()
    p = OracleProblem()
    p.batch, p.nhead_q, p.nhead_k = batch, nhead_q, nhead_k
    p.seqlen_q, p.seqlen_k, p.causal = seqlen_q, seqlen_k, int(causal)
    p.stride_q, p.nhead_stride_q, p.batch_stride_q = strides_q
    p.stride_k, p.nhead_stride_k, p.batch_stride_k = strides_k
    p.stride_v, p.nhead_stride_v, p.batch_stride_v = strides_v
    p.stride_o, p.nhead_stride_o, p.batch_stride_o = strides_o
    sq = sk = None
    if seqstart_q is not None:
        sq = np.ascontiguousarray(seqstart_q, np.int32)
        sk = np.ascontiguousarray(seqstart_k, np.int32)
        p.seqstart_q, p.seqstart_k = sq.ctypes.data, sk.ctypes.data
    p.total_q = total_q
    p.row_step, p.row_phase = row_step, row_phase
    o = np.full(out_shape, np.nan, np.float32)
    lse = None
    if with_lse:
        if lse_shape is None:
            lse_shape = (nhead_q, total_q) if seqstart_q is not None else (batch, nhead_q, seqlen_q)
        lse = np.full(lse_shape, np.nan, np.float32)
    qa, ka, va = (np.ascontiguousarray(x, np.uint16) for x in (q, k, v))
    lib.oracle_fmha_fwd(ctypes.byref(p), _ptr(qa), _ptr(ka), _ptr(va), _ptr(o),
                        _ptr(lse) if lse is not None else None)
    return o, lse


# ----------------------------------------------------------------- verdicts

def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits_trunc(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def compare(o_kern: np.ndarray, o_ref: np.ndarray, lse_kern=None, lse_ref=None) -> dict:
    """Verdicts of kernel O (float32 values of bf16) against oracle O_ref.
    Rows where o_ref is NaN (not computed) are skipped.  Arrays are
    [..., 64] with the last axis the head dimension."""
    ok_rows = ~np.isnan(o_ref).any(axis=-1)
    ref = o_ref[ok_rows].astype(np.float64)
    ker = o_kern[ok_rows].astype(np.float64)
    out = {"rows": int(ok_rows.sum())}
    diff = np.abs(ker - ref)
    nonfinite = int((~np.isfinite(ker)).sum())
    diff = np.where(np.isfinite(diff), diff, np.inf)
    out["nonfinite"] = nonfinite
    out["max_abs"] = float(diff.max()) if diff.size else 0.0
    out["mismatch"] = int((diff > REF_TOL_ABS).sum())
    big = np.abs(ref) >= 0.01
    out["max_rel"] = float((diff[big] / np.abs(ref[big])).max()) if big.any() else 0.0
    num = (ker * ref).sum(-1)
    den = np.sqrt((ref * ref).sum(-1)) * np.sqrt((ker * ker).sum(-1))
    valid = den > 0
    cos = num[valid] / den[valid]
    out["min_cos"] = float(cos.min()) if cos.size else 1.0
    out["cos_fail"] = int((cos < REF_TOL_COS).sum())
    nref = np.sqrt((ref * ref).sum())
    out["rel_l2"] = float(np.sqrt(((ker - ref) ** 2).sum()) / nref) if nref > 0 else float(
        np.sqrt(((ker - ref) ** 2).sum()))
    out["ref_pass"] = (out["mismatch"] == 0 and nonfinite == 0 and out["cos_fail"] == 0 and
                       (not big.any() or out["max_rel"] <= REF_TOL_REL))
    out["baseline_pass"] = (nonfinite == 0 and out["max_abs"] <= BASE_TOL_MAX_ABS and
                            out["rel_l2"] <= BASE_TOL_REL_L2)
    if lse_kern is not None and lse_ref is not None:
        lk = np.asarray(lse_kern, np.float64)
        lr = np.asarray(lse_ref, np.float64)
        sel = ~np.isnan(lr)
        lk, lr = lk[sel], lr[sel]
        both_ninf = np.isneginf(lk) & np.isneginf(lr)
        with np.errstate(invalid="ignore"):
            d = np.abs(lk - lr)
        d[both_ninf] = 0.0
        d = np.where(np.isnan(d), np.inf, d)
        out["lse_max_abs"] = float(d.max()) if d.size else 0.0
        out["lse_mismatch"] = int((d > LSE_TOL_ABS).sum())
        out["lse_pass"] = out["lse_mismatch"] == 0
    return out


# ----------------------------------------------------------------- device oracle

GPU_REF_LIB = os.path.join(ORACLE_DIR, "libgpu_ref.so")
_glib = None


def gpu_ref_lib() -> ctypes.CDLL:
    global _glib
    if _glib is None:
        if not os.path.exists(GPU_REF_LIB):
            raise FileNotFoundError(f"{GPU_REF_LIB} not built (python oracle/build.py)")
        _glib = ctypes.CDLL(GPU_REF_LIB)
        L, I, P = ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p
        _glib.gpu_ref_fmha_fwd.argtypes = [P, P, P, P, P, ctypes.POINTER(L), I, I, I, I, I, I,
                                           P, P, I, ctypes.c_float, P]
        _glib.gpu_ref_fmha_fwd.restype = I
    return _glib


def gpu_ref_fwd(q, k, v, *, layout: str, causal: bool, seqstart_q=None, seqstart_k=None,
                with_lse: bool = True, stream: int = 0):
    """Device oracle (gpu_ref.cu, restating gpu_ref.cpp:12-126) on torch CUDA
    bf16 tensors.  Layouts as fmha_native_b200.params_from_tensors: "bshd",
    "bhsd" (dense), "thd", "htd" (varlen, int32 seqstart on the device).
    Returns (O fp32 with q's shape, LSE fp32 [B,H,Sq] / [H,total] or None)."""
    import torch

    lib = gpu_ref_lib()
    o = torch.zeros(q.shape, device=q.device, dtype=torch.float32)
    if layout in ("bshd", "bhsd"):
        s_ax, h_ax = (1, 2) if layout == "bshd" else (2, 1)
        batch, sq, sk = q.shape[0], q.shape[s_ax], k.shape[s_ax]
        hq, hk = q.shape[h_ax], k.shape[h_ax]
        strides = []
        for t in (q, k, v, o):
            st = t.stride()
            strides += [st[s_ax], st[h_ax], st[0]]
        lse = torch.full((batch, hq, sq), float("nan"), device=q.device,
                         dtype=torch.float32) if with_lse else None
        total_q = 0
        ssq = ssk = None
    else:
        t_ax, h_ax = (0, 1) if layout == "thd" else (1, 0)
        batch = seqstart_q.numel() - 1
        hq, hk = q.shape[h_ax], k.shape[h_ax]
        total_q = q.shape[t_ax]
        lens_q = (seqstart_q[1:] - seqstart_q[:-1]).max().item() if batch > 0 else 0
        lens_k = (seqstart_k[1:] - seqstart_k[:-1]).max().item() if batch > 0 else 0
        sq, sk = int(lens_q), int(lens_k)
        strides = []
        for t in (q, k, v, o):
            st = t.stride()
            strides += [st[t_ax], st[h_ax], 0]
        lse = torch.full((hq, total_q), float("nan"), device=q.device,
                         dtype=torch.float32) if with_lse else None
        ssq, ssk = seqstart_q.data_ptr(), seqstart_k.data_ptr()
    arr = (ctypes.c_longlong * 12)(*[int(x) for x in strides])
    rc = lib.gpu_ref_fmha_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                              lse.data_ptr() if lse is not None else None, arr, batch, hq, hk,
                              sq, sk, int(causal), ssq, ssk, total_q, 1.0 / 8.0,
                              ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"gpu_ref launch failed: CUDA error {rc}")
    return o, lse


def compare_device(o_kern, o_ref, lse_kern=None, lse_ref=None) -> dict:
    """North-star verdict on device tensors (no host copy of the data):
    max-abs and rel-L2 of O (kernel bf16 vs oracle fp32), LSE max |d| with
    -inf == -inf; rows where the oracle is NaN are skipped."""
    import torch

    ref = o_ref.double()
    ker = o_kern.double()
    ok = ~torch.isnan(ref)
    d = torch.where(ok, (ker - ref).abs(), torch.zeros_like(ref))
    nonfinite = int((~torch.isfinite(ker) & ok).sum().item())
    out = {"nonfinite": nonfinite, "max_abs": float(d.max().item())}
    num = torch.sqrt((d * d).sum()).item()
    den = torch.sqrt(torch.where(ok, ref * ref, torch.zeros_like(ref)).sum()).item()
    out["rel_l2"] = num / den if den > 0 else num
    out["baseline_pass"] = (nonfinite == 0 and out["max_abs"] <= BASE_TOL_MAX_ABS and
                            out["rel_l2"] <= BASE_TOL_REL_L2)
    if lse_kern is not None and lse_ref is not None:
        lr = lse_ref.double()
        lk = lse_kern.double()
        sel = ~torch.isnan(lr)
        both = torch.isneginf(lk) & torch.isneginf(lr)
        dl = (lk - lr).abs()
        dl = torch.where(both, torch.zeros_like(dl), dl)
        dl = torch.where(torch.isnan(dl), torch.full_like(dl, float("inf")), dl)
        dl = torch.where(sel, dl, torch.zeros_like(dl))
        out["lse_max_abs"] = float(dl.max().item())
        out["lse_pass"] = out["lse_max_abs"] <= LSE_TOL_ABS
    return out
