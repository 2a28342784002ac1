"""The error budgets of the certified int8 SiLU epilogue hold on this GPU.

The fast path evaluates exp and the reciprocal with ex2.approx.ftz.f32 and
rcp.approx.ftz.f32 and certifies each int8 result against a bound built from
their largest relative errors (kEx2RelErr, kRcpRelErr in
dragonwing_edge_rs_b200/csrc/dw_device.cuh).  This test measures those errors
exhaustively -- every float input of the ranges the fast path uses -- with a
small CUDA program (tests/cuda/fast_math_err.cu) and checks they are within the
budgets; a GPU whose approximations were less accurate would fail here before
any int8 result could go wrong unnoticed.
"""
import os
import re
import shutil
import subprocess

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _budgets():
    src = open(os.path.join(ROOT, "dragonwing_edge_rs_b200", "csrc", "dw_device.cuh")).read()
    get = lambda name: float(re.search(rf"constexpr float {name} = ([0-9.e+-]+)f;", src).group(1))
    return get("kEx2RelErr"), get("kRcpRelErr")


def test_ex2_rcp_approx_errors_within_the_silu_budgets(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = str(tmp_path / "fast_math_err")
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-o", exe,
                    os.path.join(HERE, "cuda", "fast_math_err.cu")], check=True, capture_output=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True, timeout=300).stdout
    got = {line.split()[0]: float(line.split()[1]) for line in out.strip().splitlines()}
    ex2_budget, rcp_budget = _budgets()
    print(f"\nex2.approx max rel err {max(got['ex2_neg'], got['ex2_pos']):.4e} (budget {ex2_budget:.1e}); "
          f"rcp.approx {got['rcp']:.4e} (budget {rcp_budget:.1e})")
    assert 0.0 < got["ex2_neg"] <= ex2_budget
    assert 0.0 < got["ex2_pos"] <= ex2_budget
    assert 0.0 < got["rcp"] <= rcp_budget
