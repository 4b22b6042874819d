"""Build libso3lr_b200.so in-tree with nvcc for sm_100a.

    python -m so3lr_b200.build [--force]

Every translation unit is compiled with
``-gencode arch=compute_100a,code=sm_100a -O3 -lineinfo`` and linked into
``so3lr_b200/libso3lr_b200.so``. nvcc cross-compiles without a GPU. The
translation units whose code depends on the model width are compiled once per
supported width (``-DSO3LR_FEATURES=128`` and ``=256``; the mixed-precision
filter kernels exist for F = 128 only). Object files are cached under
``so3lr_b200/_build`` and rebuilt when a source or header is newer.
"""
from __future__ import annotations

import concurrent.futures
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libso3lr_b200.so"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-lineinfo", "-I", str(INCLUDE), "-I", str(CSRC)]
CU_FLAGS = ARCH + COMMON + ["--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libso3lr_b200")
    return path


# width-dependent translation units and the widths each is compiled for
SHAPED = {"attention.cu": (128, 256), "filter.cu": (128, 256), "node.cu": (128, 256),
          "evaluator.cu": (128, 256), "local_frame.cu": (128, 256),
          "filter_mixed.cu": (128,), "filter_tc.cu": (128,)}


def sources():
    """(source, model width or None) for every object of the library"""
    out = []
    for src in sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp"))):
        for width in SHAPED.get(src.name, (None,)):
            out.append((src, width))
    return out


def headers():
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + list(INCLUDE.glob("*.h")))


def _compile(unit, newest_header: float, force: bool, verbose: bool) -> pathlib.Path:
    src, width = unit
    obj = BUILD / (src.name + (f".f{width}" if width else "") + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header):
        return obj
    cmd = [nvcc(), "-c", str(src), "-o", str(obj)] + CU_FLAGS
    if src.suffix == ".cpp":
        cmd = [nvcc(), "-x", "cu", "-c", str(src), "-o", str(obj)] + CU_FLAGS
    if width:
        cmd += [f"-DSO3LR_FEATURES={width}"]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name} (width {width}):\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    BUILD.mkdir(exist_ok=True)
    newest_header = max([h.stat().st_mtime for h in headers()] + [pathlib.Path(__file__).stat().st_mtime])
    srcs = sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as pool:
        objs = list(pool.map(lambda s: _compile(s, newest_header, force, verbose), srcs))
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), "-shared", "-o", str(LIB)] + ARCH + [str(o) for o in objs] + ["-lcudart", "-ldl", "-Xlinker", "-rpath=/usr/local/cuda/lib64"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    lib = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(lib)
