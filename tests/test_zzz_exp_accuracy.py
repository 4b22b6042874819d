"""The kernels' own exp (Tang's table-driven method, ACM TOMS 15(2), 1989;
so3lr_b200/csrc/common.cuh exp_tang) and the SiLU / SiLU' built on it with a
Newton-refined reciprocal, checked against CUDA's exp and IEEE division
(tests/exp_check/exp_check.cu): exp within 2 ulp, SiLU within 8 ulp, SiLU'
within 4e-15 (1 + |x|), on dense grids of [-40, 40], [-700, 700] and
[-1e-3, 1e-3]. The CPU part only compiles the checker."""
import shutil
import subprocess

import pytest

from conftest import ROOT

SRC = ROOT / "tests" / "exp_check" / "exp_check.cu"


def _compile(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not shutil.which(nvcc):
        pytest.skip("nvcc not available")
    exe = tmp_path / "exp_check"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", str(SRC), "-o",
                    str(exe)], check=True, capture_output=True, text=True, timeout=600)
    return exe


def test_exp_checker_compiles(tmp_path):
    assert _compile(tmp_path).exists()


@pytest.mark.gpu
def test_exp_and_silu_against_cuda(tmp_path):
    exe = _compile(tmp_path)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0 and "EXP CHECK OK" in res.stdout, res.stdout + res.stderr
