"""Device helpers of the kernel checked against CUDA's own functions (GPU).

* exp2_poly2 (fmha_native_b200/csrc/sm100_ptx.cuh): the degree-3 polynomial
  exp2 that takes a share of the softmax exponentials off MUFU.  Its stated
  bound is a relative error of 7.5e-5 (coefficients fitted by
  csrc/fit_exp2_poly.py) over the inputs it gets, x in [-120, 0] (scores
  minus the running max, scaled; the kernel's lazy reference lets x reach
  +8, also covered).  Checked against exp2f on a dense grid plus random
  points, and against the MUFU ex2.approx it replaces.
* The bf16 packers: truncation (P before P.V, as the reference's
  op_gemm.hpp:272-273) and round-to-nearest-even (O) against bit arithmetic.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "native", "libfmha_unit.so")
POLY_REL_BOUND = 7.5e-5


def _lib():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} not built (fmha_native_b200.build.build_test_lib)")
    lib = ctypes.CDLL(LIB)
    P = ctypes.c_void_p
    lib.unit_exp2.argtypes = [P, P, P, P, ctypes.c_int]
    lib.unit_pack_bf16.argtypes = [P, P, P, ctypes.c_int]
    return lib


def test_exp2_poly_within_bound(cuda_device):
    import torch

    lib = _lib()
    grid = np.linspace(-120.0, 8.0, 1 << 20, dtype=np.float32)
    rnd = np.random.default_rng(5).uniform(-120.0, 8.0, 1 << 18).astype(np.float32)
    x = torch.from_numpy(np.concatenate([grid, rnd])).to(cuda_device)
    yp, ym, yr = (torch.empty_like(x) for _ in range(3))
    assert lib.unit_exp2(x.data_ptr(), yp.data_ptr(), ym.data_ptr(), yr.data_ptr(), x.numel()) == 0
    torch.cuda.synchronize()
    rel = ((yp.double() - yr.double()).abs() / yr.double()).max().item()
    assert rel <= POLY_REL_BOUND, rel
    # exact against an independent fp64 exp2 too (exp2f itself is within 2 ulp)
    ref64 = torch.exp2(x.double())
    assert ((yp.double() - ref64).abs() / ref64).max().item() <= POLY_REL_BOUND + 2.4e-7
    # The MUFU path it replaces is of the same order (ftz: tiny results -> 0).
    big = yr > 1e-30
    rel_m = ((ym.double() - yr.double()).abs() / yr.double())[big].max().item()
    assert rel_m <= 1e-5, rel_m


def test_bf16_packers(cuda_device):
    import torch

    lib = _lib()
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(1 << 16).astype(np.float32) * 3,
                        np.array([0.0, -0.0, 1.0, 1.00390625, 1.01171875, 65504.0, 1e-30, -7.5],
                                 np.float32)])
    xd = torch.from_numpy(x).to(cuda_device)
    n = x.size // 2
    tr = torch.empty(n, dtype=torch.int32, device=cuda_device)
    rn = torch.empty(n, dtype=torch.int32, device=cuda_device)
    assert lib.unit_pack_bf16(xd.data_ptr(), tr.data_ptr(), rn.data_ptr(), n) == 0
    torch.cuda.synchronize()
    u = x[: 2 * n].view(np.uint32)
    want_tr = (u[0::2] >> 16) | ((u[1::2] >> 16) << 16)
    # round to nearest even on the upper 16 bits (finite inputs only here)
    def rne(a):
        return ((a + 0x7FFF + ((a >> 16) & 1)) >> 16) & 0xFFFF
    want_rn = rne(u[0::2].astype(np.uint64)) | (rne(u[1::2].astype(np.uint64)) << 16)
    assert np.array_equal(tr.cpu().numpy().view(np.uint32), want_tr.astype(np.uint32))
    assert np.array_equal(rn.cpu().numpy().view(np.uint32), want_rn.astype(np.uint32))
