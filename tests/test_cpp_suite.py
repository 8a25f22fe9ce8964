"""The C++ gtest-format suite (tests/cpp/test_fmha_fwd_d64.cpp), graded the
way the reference's gate grades its gtest binaries (scripts/run-gates.sh:
80-113 of poyenc/fmha_native): exit code 0, no "[  FAILED  ]" or
"[  SKIPPED ]" line, and a "[  PASSED  ] N tests." summary with every test."""
from __future__ import annotations

import os
import re
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXPECTED = 67  # 2 smoke + 63 matrix + 2 closed-form, as the reference's fused suite


def _binary():
    from fmha_native_b200 import build

    return build.build_cpp_tests()


def test_cpp_suite_builds_and_lists_every_case():
    exe = _binary()
    out = subprocess.run([exe, "--gtest_list_tests"], capture_output=True, text=True,
                         check=True).stdout.split()
    assert len(out) == EXPECTED
    assert "Full/FmhaFwdD64Test.MatchesGpuRef/D64KitchenSink" in out
    sub = subprocess.run([exe, "--gtest_list_tests", "--gtest_filter=FmhaGoldenCK.*"],
                         capture_output=True, text=True, check=True).stdout.split()
    assert sub == ["FmhaGoldenCK.FullTile", "FmhaGoldenCK.PartialTile"]


@pytest.mark.gpu
def test_cpp_suite_passes_on_gpu(cuda_device):
    exe = _binary()
    r = subprocess.run([exe], capture_output=True, text=True, timeout=1200)
    out = r.stdout
    assert r.returncode == 0, out[-3000:]
    assert "[  FAILED  ]" not in out and "[  SKIPPED ]" not in out, out[-3000:]
    m = re.findall(r"\[  PASSED  \] (\d+) tests\.", out)
    assert m and int(m[-1]) == EXPECTED, out[-3000:]
