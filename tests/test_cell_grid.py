"""Host-side planning of the neighbour-search cell grid
(so3lr_b200/csrc/cell_grid.cpp, plain C++): cells never smaller than the
short-range cutoff, bounded cell counts for periodic and open systems (dense,
sparse, one atom far away), every open-system atom inside its grid, and
refusals of oversized boxes and non-finite positions."""
import shutil
import subprocess

import pytest

from conftest import ROOT


def test_cell_grid_planning(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    csrc = ROOT / "so3lr_b200" / "csrc"
    exe = tmp_path / "cell_grid_check"
    subprocess.run([gxx, "-std=c++17", "-O1", "-I", str(csrc), str(csrc / "cell_grid.cpp"),
                    str(ROOT / "tests" / "cell_grid" / "cell_grid_check.cpp"), "-o", str(exe)],
                   check=True, capture_output=True, text=True, timeout=300)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0 and "CELL GRID OK" in res.stdout, res.stdout + res.stderr
