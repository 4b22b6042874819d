"""The LAMMPS pair style so3lr/b200 (so3lr_b200/lammps/) compiled against a
minimal mock of the LAMMPS Pair API (tests/lammps_mock/): pair_style and
pair_coeff parsing and refusals mirror the reference style
(plugins/lammps/pair_so3lr_native_mpi.cpp:1097-1192); on a GPU one compute()
must return what the C ABI returns for the same atoms.
"""
import json
import pathlib
import shutil
import subprocess

import numpy as np
import pytest

from conftest import MODEL, ROOT


def _build(tmp_path: pathlib.Path) -> pathlib.Path:
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    from so3lr_b200.runtime import LIB_PATH
    if not LIB_PATH.exists():
        pytest.skip("library not built")
    exe = tmp_path / "test_pair_shim"
    cmd = [gxx, "-std=c++17", "-O1", "-I", str(ROOT / "tests" / "lammps_mock"), "-I",
           str(ROOT / "so3lr_b200" / "lammps"), "-I", str(ROOT / "include"),
           str(ROOT / "so3lr_b200" / "lammps" / "pair_so3lr_b200.cpp"),
           str(ROOT / "tests" / "lammps_mock" / "test_pair_shim.cpp"), "-L", str(LIB_PATH.parent),
           "-lso3lr_b200", f"-Wl,-rpath,{LIB_PATH.parent}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_pair_style_parsing_and_refusals(tmp_path):
    exe = _build(tmp_path)
    res = subprocess.run([str(exe), "parse", str(MODEL)], capture_output=True, text=True, timeout=300)
    assert "PARSE OK" in res.stdout, res.stdout + res.stderr
    assert res.returncode == 0


@pytest.mark.gpu
def test_pair_style_compute_matches_c_abi(tmp_path, gpu_model):
    from so3lr_b200.systems import water_box
    exe = _build(tmp_path)
    w = water_box(64, seed=21)
    inp = tmp_path / "box.txt"
    lines = [f"{float(w.cell[0])!r} {len(w.z)}"]
    for zi, p in zip(w.z, w.pos):
        lines.append(f"{1 if zi == 8 else 2} {float(p[0])!r} {float(p[1])!r} {float(p[2])!r}")
    inp.write_text("\n".join(lines) + "\n")
    res = subprocess.run([str(exe), "run", str(MODEL), str(inp)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    out = json.loads(res.stdout.strip().splitlines()[-1])
    ref = gpu_model.compute(w.pos, w.z, cell=w.cell, boxlo=w.boxlo)
    ref_va = gpu_model.virial_atom(len(w.z))
    assert np.array_equal(np.array(out["vatom"]), ref_va)
    assert out["energy"] == ref["energy"]
    assert np.array_equal(np.array(out["forces"]), ref["forces"])
    assert np.allclose(out["virial"], ref["virial"], rtol=0, atol=1e-12)
    assert abs(out["eatom_sum"] - ref["energy"]) < 1e-8
    assert "SO3LR_B200_FORCE_PATH=PASS" in out["log"]
