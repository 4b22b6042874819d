"""The boundary seen from C: tests/c_abi/c_abi_check.c includes
include/so3lr_b200.h, compiles as strict C99 and links libso3lr_b200.so the way
a C host (a LAMMPS plugin, a cgo or FFI binding) would. On the CPU it runs the
host-only entry points; on a GPU one compute must equal the Python binding's.
"""
import re
import shutil
import subprocess

import numpy as np
import pytest

from conftest import MODEL, ROOT


def _build(tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    from so3lr_b200.runtime import LIB_PATH
    if not LIB_PATH.exists():
        pytest.skip("library not built")
    exe = tmp_path / "c_abi_check"
    subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "c_abi" / "c_abi_check.c"), "-L", str(LIB_PATH.parent), "-lso3lr_b200",
                    f"-Wl,-rpath,{LIB_PATH.parent}", "-lm", "-o", str(exe)], check=True, capture_output=True,
                   text=True)
    return exe


def test_c_consumer_host_entry_points(tmp_path):
    exe = _build(tmp_path)
    res = subprocess.run([str(exe), "host", str(MODEL)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0 and "C ABI OK" in res.stdout, res.stdout + res.stderr


@pytest.mark.gpu
def test_c_consumer_compute_matches_python_binding(tmp_path, gpu_model):
    exe = _build(tmp_path)
    res = subprocess.run([str(exe), "gpu", str(MODEL)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0 and "C ABI OK" in res.stdout, res.stdout + res.stderr
    m = re.search(r"energy (\S+) force0 (\S+) (\S+) (\S+)", res.stdout)
    x, z = [], []
    for i in range(2):
        for j in range(2):
            for k in range(2):
                o = np.array([3.1 * i + 0.5, 3.1 * j + 0.5, 3.1 * k + 0.5])
                x += [o, o + [0.9572, 0, 0], o + [-0.24, 0.9266, 0]]
                z += [8, 1, 1]
    ref = gpu_model.compute(np.array(x), np.array(z), cell=np.array([6.2] * 3), boxlo=np.zeros(3))
    assert float(m.group(1)) == ref["energy"]
    assert np.array_equal(np.array([float(m.group(k)) for k in (2, 3, 4)]), ref["forces"][0])
