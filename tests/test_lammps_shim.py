"""The LAMMPS pair styles so3lr/b200 and so3lr/b200/turbo (so3lr_b200/lammps/)
compiled against a minimal mock of the LAMMPS Pair API (tests/lammps_mock/):
pair_style and pair_coeff parsing and refusals mirror the reference styles
(plugins/lammps/pair_so3lr_native_mpi.cpp:1097-1192,
pair_so3lr_turbo.cpp:110-223); on a GPU one compute() must return what the C
ABI returns for the same atoms. The turbo style's partitions run as threads
acting as the ranks of a LAMMPS universe (tests/lammps_mock/mpi.h); on the CPU a
stand-in of the C ABI (tests/lammps_mock/fake_so3lr_b200.cpp) checks that every
partition gets back exactly its own image.
"""
import json
import pathlib
import shutil
import subprocess

import numpy as np
import pytest

from conftest import MODEL, ROOT


def _build(tmp_path: pathlib.Path, fake: bool = False) -> pathlib.Path:
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    from so3lr_b200.runtime import LIB_PATH
    if not fake and not LIB_PATH.exists():
        pytest.skip("library not built")
    mock = ROOT / "tests" / "lammps_mock"
    shim = ROOT / "so3lr_b200" / "lammps"
    exe = tmp_path / ("test_pair_fake" if fake else "test_pair_shim")
    cmd = [gxx, "-std=c++17", "-O1", "-pthread", "-I", str(mock), "-I", str(shim), "-I", str(ROOT / "include"),
           str(shim / "pair_so3lr_b200.cpp"), str(shim / "pair_so3lr_b200_turbo.cpp"),
           str(shim / "so3lrb200plugin.cpp"), str(mock / "test_pair_shim.cpp")]
    if fake:
        cmd += [str(mock / "fake_so3lr_b200.cpp")]
    else:
        cmd += ["-L", str(LIB_PATH.parent), "-lso3lr_b200", f"-Wl,-rpath,{LIB_PATH.parent}"]
    subprocess.run(cmd + ["-o", str(exe)], check=True, capture_output=True, text=True)
    return exe


def _write_images(path: pathlib.Path, pos, z, off, q, m) -> None:
    lines = [str(len(off) - 1)]
    for k in range(len(off) - 1):
        lines.append(f"{int(off[k + 1] - off[k])} {float(q[k])!r} {float(m[k])!r}")
        for i in range(off[k], off[k + 1]):
            lines.append(f"{1 if z[i] == 8 else 2} {float(pos[i, 0])!r} {float(pos[i, 1])!r} {float(pos[i, 2])!r}")
    path.write_text("\n".join(lines) + "\n")


def _json_lines(res, expected: int):
    """The JSON records a driver mode printed (one per image or rank); other
    lines (library or NCCL log output) are skipped."""
    assert res.returncode == 0, res.stdout + res.stderr
    out = [json.loads(line) for line in res.stdout.splitlines() if line.startswith("{")]
    assert len(out) == expected, res.stdout + res.stderr
    return out


def _run_images(exe, model, inp, nimg):
    res = subprocess.run([str(exe), "turbo-run", str(model), str(inp)], capture_output=True, text=True, timeout=600)
    return _json_lines(res, nimg)


def _fdotr(x, f):
    """LAMMPS's virial_fdotr_compute: sum over atoms of x (x) f, order xx yy zz xy xz yz."""
    return np.array([(f[:, 0] * x[:, 0]).sum(), (f[:, 1] * x[:, 1]).sum(), (f[:, 2] * x[:, 2]).sum(),
                     (f[:, 1] * x[:, 0]).sum(), (f[:, 2] * x[:, 0]).sum(), (f[:, 2] * x[:, 1]).sum()])


def test_pair_style_parsing_and_refusals(tmp_path):
    exe = _build(tmp_path)
    res = subprocess.run([str(exe), "parse", str(MODEL)], capture_output=True, text=True, timeout=300)
    assert "PARSE OK" in res.stdout, res.stdout + res.stderr
    assert res.returncode == 0
    res = subprocess.run([str(exe), "turbo-parse", str(MODEL)], capture_output=True, text=True, timeout=300)
    assert "TURBO PARSE OK" in res.stdout, res.stdout + res.stderr
    assert res.returncode == 0


def test_debug_dump_in_the_reference_schema(tmp_path, monkeypatch):
    """SO3LR_NATIVE_DEBUG_DUMP (pair_so3lr_native_mpi.cpp:1811-1862): one JSON
    object with schema so3lr-native-debug-v1, the long-range totals and, per
    local atom, its tag, type and terms (here from the CPU stand-in of the
    library, whose row k carries charge 0.01 k, so the tag mapping shows)."""
    exe = _build(tmp_path, fake=True)
    pos = np.array([[0.0, 0.0, 0.0], [0.96, 0.0, 0.0], [-0.24, 0.93, 0.0], [3.0, 3.0, 3.0]])
    types = [1, 2, 2, 1]
    inp = tmp_path / "atoms.txt"
    inp.write_text("10.0 4\n" + "".join(f"{t} {float(p[0])!r} {float(p[1])!r} {float(p[2])!r}\n"
                                          for t, p in zip(types, pos)))
    dump = tmp_path / "dump.json"
    monkeypatch.setenv("SO3LR_NATIVE_DEBUG_DUMP", str(dump))
    res = subprocess.run([str(exe), "run-reversed-tags", "fake", str(inp)], capture_output=True, text=True,
                         timeout=120)
    out = _json_lines(res, 1)[0]
    assert "SO3LR: total charge 0, spin multiplicity 1" in out["log"]
    assert "SO3LR_B200_FORCE_PATH=PASS" in out["log"]
    d = json.loads(dump.read_text())
    assert d["schema"] == "so3lr-native-debug-v1" and d["natoms"] == 4
    assert d["tag"] == [4, 3, 2, 1] and d["type"] == [1, 2, 2, 1]
    z = np.array([8, 1, 1, 8])
    assert np.allclose(d["learned_energy"], 0.25 * z)
    assert np.allclose(d["zbl_energy"], 0.125)
    assert np.allclose(d["physical_energy"], 0.25 * z - 0.125)
    assert np.allclose(d["partial_charges"], [0.03, 0.02, 0.01, 0.0])  # row = tag - 1
    assert np.allclose(d["hirshfeld_ratios"], 1.0 + 0.001 * z)
    assert abs(d["electrostatic_total"] - 0.5 * (0.25 * z - 0.125).sum()) < 1e-12
    assert abs(d["dispersion_total"] - d["electrostatic_total"]) < 1e-12


def test_profile_lines(tmp_path, monkeypatch):
    """SO3LR_B200_PROFILE / SO3LR_B200_PROFILE_EVERY: every N-th compute logs
    the pair-filter kernel times since the previous line (the counterpart of
    the reference's SO3_NATIVE_MPI_PROFILE lines)."""
    exe = _build(tmp_path, fake=True)
    inp = tmp_path / "atoms.txt"
    inp.write_text("10.0 3\n1 0.0 0.0 0.0\n2 0.96 0.0 0.0\n2 -0.24 0.93 0.0\n")
    monkeypatch.setenv("SO3LR_B200_PROFILE", "1")
    monkeypatch.setenv("SO3LR_B200_PROFILE_EVERY", "2")
    res = subprocess.run([str(exe), "repeat", "fake", str(inp)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("SO3LR_B200_PROFILE ")]
    assert len(lines) == 2, res.stdout
    assert "calls=2 filter_forward_ms=2.0000 launches=2 tflops=1.00" in lines[0]
    assert "calls=4 " in lines[1] and "filter_reverse_ms=2.0000 launches=2" in lines[1]


def test_charge_log_line_and_periodic_charge_warning(tmp_path):
    """init_style logs the total charge and multiplicity once and warns about a
    net charge in a periodic cell (pair_so3lr_native_mpi.cpp:1225-1234)."""
    exe = _build(tmp_path, fake=True)
    inp = tmp_path / "atoms.txt"
    inp.write_text("10.0 3\n1 0.0 0.0 0.0\n2 0.96 0.0 0.0\n2 -0.24 0.93 0.0\n")
    res = subprocess.run([str(exe), "repeat", "fake", str(inp), "1", "2"], capture_output=True, text=True,
                         timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "SO3LR: total charge 1, spin multiplicity 2" in res.stdout
    warn = [ln for ln in res.stdout.splitlines() if ln.startswith("WARNING:")]
    assert len(warn) == 1 and "net charge 1 in a periodic cell" in warn[0], res.stdout
    res = subprocess.run([str(exe), "repeat", "fake", str(inp)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "SO3LR: total charge 0, spin multiplicity 1" in res.stdout and "WARNING" not in res.stdout


def _water_input(tmp_path, nmol=8, seed=5):
    from so3lr_b200.systems import water_box
    w = water_box(nmol, seed=seed)
    inp = tmp_path / "box.txt"
    lines = [f"{float(w.cell[0])!r} {len(w.z)}"]
    for zi, p in zip(w.z, w.pos):
        lines.append(f"{1 if zi == 8 else 2} {float(p[0])!r} {float(p[1])!r} {float(p[2])!r}")
    inp.write_text("\n".join(lines) + "\n")
    return w, inp


def test_multirank_routing_with_the_cpu_stand_in(tmp_path, monkeypatch):
    """so3lr/b200 on three ranks (threads) with atoms dealt out of order: every
    rank passes only its own atoms (so3lr_compute_local) and gets back exactly
    their forces and per-atom energies (the stand-in returns f = -x and
    eatom = z / 2 per atom), and only rank 0 reports the global energy (the
    stand-in's natoms + 0.5)."""
    exe = _build(tmp_path, fake=True)
    monkeypatch.delenv("FAKE_SO3LR_FAIL_RANK", raising=False)
    w, inp = _water_input(tmp_path)
    res = subprocess.run([str(exe), "multirank", "fake", str(inp), "3"], capture_output=True, text=True, timeout=120)
    out = _json_lines(res, 3)
    seen = []
    for o in out:
        rows = np.array(o["tags"]) - 1
        seen += list(rows)
        assert np.array_equal(np.array(o["forces"]), -w.pos[rows])
        assert np.array_equal(np.array(o["eatom"]), 0.5 * w.z[rows])
        assert o["energy"] == (len(w.z) + 0.5 if o["rank"] == 0 else 0.0)
    assert sorted(seen) == list(range(len(w.z)))


def test_evaluation_failure_on_one_rank_aborts_from_that_rank(tmp_path, monkeypatch):
    """A library failure on one of several ranks is reported with error->one
    from the failing rank (which aborts the job), not error->all, whose barrier
    would wait for ranks that may be blocked in the library's collectives."""
    exe = _build(tmp_path, fake=True)
    monkeypatch.setenv("FAKE_SO3LR_FAIL_RANK", "1")
    _, inp = _water_input(tmp_path)
    res = subprocess.run([str(exe), "multirank", "fake", str(inp), "2"], capture_output=True, text=True, timeout=120)
    assert res.returncode == 1, res.stdout + res.stderr
    assert "ERROR rank 1: ERROR on proc: SO3LR evaluation failed: injected failure" in res.stdout, res.stdout


def test_duplicate_atom_tags_are_refused(tmp_path):
    exe = _build(tmp_path, fake=True)
    _, inp = _water_input(tmp_path, nmol=2)
    res = subprocess.run([str(exe), "run-duplicate-tag", "fake", str(inp)], capture_output=True, text=True,
                         timeout=120)
    assert res.returncode != 0 and "atom tags must be unique" in res.stdout + res.stderr, res.stdout + res.stderr


def test_precision_environment_variable(tmp_path, monkeypatch):
    """SO3LR_B200_PRECISION=mixed switches the style's handle to the mixed
    precision mode; any value other than float64 or mixed is refused when the
    pair style is set up."""
    exe = _build(tmp_path, fake=True)
    _, inp = _water_input(tmp_path, nmol=2)
    monkeypatch.setenv("SO3LR_B200_PRECISION", "bf16")
    res = subprocess.run([str(exe), "run", "fake", str(inp)], capture_output=True, text=True, timeout=120)
    assert res.returncode != 0 and "must be 'float64' or 'mixed'" in res.stdout + res.stderr, res.stdout + res.stderr
    monkeypatch.setenv("SO3LR_B200_PRECISION", "mixed")
    res = subprocess.run([str(exe), "run", "fake", str(inp)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr


def test_model_failure_on_one_rank_stops_every_rank(tmp_path):
    """so3lr/b200 on two ranks (threads) where only one cannot load the model:
    that rank reports the loader's message, the other learns of it in the same
    collective instead of waiting (the reference's allreduced error flags,
    pair_so3lr_native_mpi.cpp:1293, 1388)."""
    exe = _build(tmp_path, fake=True)
    res = subprocess.run([str(exe), "rank-failure", "fake"], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0 and "RANK FAILURE OK" in res.stdout, res.stdout + res.stderr


def test_plugin_registers_both_styles(tmp_path):
    """`plugin load` entry point (lammpsplugin_init): both pair styles are
    registered under their names and their creators construct the styles."""
    exe = _build(tmp_path, fake=True)
    res = subprocess.run([str(exe), "plugin"], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0 and "PLUGIN OK" in res.stdout, res.stdout + res.stderr
    assert "pair so3lr/b200 constructed" in res.stdout and "pair so3lr/b200/turbo constructed" in res.stdout


def test_turbo_routes_each_image_back_to_its_partition(tmp_path):
    """Four partitions of different sizes and charges: the coordinator packs
    them, and each partition gets back its own forces, per-atom energies and
    virials, its image energy, and the F dot r virial of its atoms; a second
    step where only image 0 asks for per-atom virials repeats the first."""
    from so3lr_b200.systems import turbo_batch
    exe = _build(tmp_path, fake=True)
    pos, z, off, q, m = turbo_batch(4, seed=7)
    inp = tmp_path / "images.txt"
    _write_images(inp, pos, z, off, q, m)
    out = _run_images(exe, "fake", inp, 4)
    for k, o in enumerate(out):
        sl = slice(off[k], off[k + 1])
        x = pos[sl]
        f = np.array(o["forces"])
        assert o["image"] == k
        assert np.array_equal(f, (k + 1) * x)
        assert o["energy"] == float((z[sl] + 1000 * k).sum())
        assert o["eatom_sum"] == o["energy"]
        assert np.array_equal(np.array(o["vatom"]), x[:, [0, 1, 2, 0, 1, 2]] + k)
        assert np.allclose(o["virial"], _fdotr(x, f), rtol=1e-14, atol=0)
        assert o["repeat_equal"] and o["evaluations"] == 2
        assert f"SO3LR_TURBO_LIVE image={k} universe_rank={k} coordinator={int(k == 0)} images=4" in o["log"]
        assert f"SO3LR turbo image {k}: total charge {q[k]:g}" in o["log"]


def test_turbo_gpu_groups_keep_each_image_in_its_group(tmp_path, monkeypatch):
    """SO3LR_B200_TURBO_GPUS=2 over four partitions: two groups of two
    consecutive partitions, each with its own coordinator (universe ranks 0 and
    2) and its own pack. The stand-in encodes an image's index inside the pack
    it was evaluated in, so each partition's results show that its image went
    to its own group's pack, at index k mod 2, and came back to it."""
    from so3lr_b200.systems import turbo_batch
    monkeypatch.setenv("SO3LR_B200_TURBO_GPUS", "2")
    exe = _build(tmp_path, fake=True)
    pos, z, off, q, m = turbo_batch(4, seed=7)
    inp = tmp_path / "images.txt"
    _write_images(inp, pos, z, off, q, m)
    out = _run_images(exe, "fake", inp, 4)
    for k, o in enumerate(out):
        j = k % 2  # index of the image in its group's pack
        sl = slice(off[k], off[k + 1])
        x = pos[sl]
        f = np.array(o["forces"])
        assert o["image"] == k
        assert np.array_equal(f, (j + 1) * x)
        assert o["energy"] == float((z[sl] + 1000 * j).sum())
        assert np.array_equal(np.array(o["vatom"]), x[:, [0, 1, 2, 0, 1, 2]] + j)
        assert o["repeat_equal"] and o["evaluations"] == 2
        assert (f"SO3LR_TURBO_LIVE image={k} universe_rank={k} coordinator={int(j == 0)} images=2" in o["log"]
                and f"gpu_group={k // 2} of 2" in o["log"]), o["log"]


def test_turbo_refusal_on_one_partition_stops_all(tmp_path):
    """A periodic image and an impossible multiplicity on two partitions: each
    reports its own problem and the others stop too, instead of waiting."""
    from so3lr_b200.systems import turbo_batch
    exe = _build(tmp_path, fake=True)
    pos, z, off, q, m = turbo_batch(3, seed=7)
    inp = tmp_path / "images.txt"
    _write_images(inp, pos, z, off, q, m)
    res = subprocess.run([str(exe), "turbo-refuse", "fake", str(inp)], capture_output=True, text=True, timeout=300)
    assert "TURBO REFUSE OK" in res.stdout, res.stdout + res.stderr


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
    out = _json_lines(res, 1)[0]
    ref = gpu_model.compute(w.pos, w.z, cell=w.cell, boxlo=w.boxlo)
    ref_va = gpu_model.virial_atom(len(w.z))
    assert np.array_equal(np.array(out["vatom"]), ref_va)
    assert out["energy"] == ref["energy"]
    assert np.array_equal(np.array(out["forces"]), ref["forces"])
    assert np.allclose(out["virial"], ref["virial"], rtol=0, atol=1e-12)
    assert abs(out["eatom_sum"] - ref["energy"]) < 1e-8
    assert "SO3LR_B200_FORCE_PATH=PASS" in out["log"]


@pytest.mark.gpu
def test_pair_style_on_two_ranks_matches_one_gpu(tmp_path, gpu_model):
    """so3lr/b200 on two MPI ranks (threads of the mock universe, one GPU
    each, atoms dealt to the ranks out of order): every rank's forces,
    per-atom energies and virials equal the single-GPU result for its atoms'
    tags, and rank 0 alone reports the global energy and virial."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from so3lr_b200.systems import water_box
    exe = _build(tmp_path)
    w = water_box(216, seed=23)
    inp = tmp_path / "box.txt"
    lines = [f"{float(w.cell[0])!r} {len(w.z)}"]
    for zi, p in zip(w.z, w.pos):
        lines.append(f"{1 if zi == 8 else 2} {float(p[0])!r} {float(p[1])!r} {float(p[2])!r}")
    inp.write_text("\n".join(lines) + "\n")
    res = subprocess.run([str(exe), "multirank", str(MODEL), str(inp), "2"], capture_output=True, text=True,
                         timeout=600)
    out = _json_lines(res, 2)
    ref = gpu_model.compute(w.pos, w.z, cell=w.cell, boxlo=w.boxlo)
    ref_va = gpu_model.virial_atom(len(w.z))
    seen = []
    for o in out:
        rows = np.array(o["tags"]) - 1
        seen += list(rows)
        assert np.array_equal(np.array(o["forces"]), ref["forces"][rows])
        assert np.array_equal(np.array(o["vatom"]), ref_va[rows])
        assert np.array_equal(np.array(o["eatom"]), ref["eatom"][rows])
        if o["rank"] == 0:
            assert o["energy"] == ref["energy"]
            assert np.array_equal(np.array(o["virial"]), ref["virial"])
        else:
            assert o["energy"] == 0.0 and not any(o["virial"])
    assert sorted(seen) == list(range(len(w.z)))


@pytest.mark.gpu
def test_turbo_pair_style_matches_c_abi(tmp_path, gpu_model):
    """so3lr/b200/turbo over five partitions returns, per image, what
    so3lr_compute_batch returns for the same pack (bit for bit), per-atom
    virials equal to so3lr_virial_atom, and an F dot r virial equal to the
    image's own pair virial (so3lr_compute on the lone image); refusals on one
    partition stop all of them."""
    from so3lr_b200.systems import turbo_batch
    exe = _build(tmp_path)
    pos, z, off, q, m = turbo_batch(5, seed=11)
    inp = tmp_path / "images.txt"
    _write_images(inp, pos, z, off, q, m)
    out = _run_images(exe, MODEL, inp, 5)
    ref = gpu_model.compute_batch(pos, z, off, q, m)
    ref_va = gpu_model.virial_atom(len(z))
    for k, o in enumerate(out):
        sl = slice(off[k], off[k + 1])
        assert np.array_equal(np.array(o["forces"]), ref["forces"][sl])
        assert o["energy"] == ref["image_energy"][k]
        assert abs(o["eatom_sum"] - ref["image_energy"][k]) <= 1e-9
        assert np.array_equal(np.array(o["vatom"]), ref_va[sl])
        assert o["repeat_equal"] and o["evaluations"] == 2
        single = gpu_model.compute(pos[sl], z[sl], charge=q[k], multiplicity=m[k])
        assert np.allclose(o["virial"], single["virial"], rtol=0, atol=1e-8)
    res = subprocess.run([str(exe), "turbo-refuse", str(MODEL), str(inp)], capture_output=True, text=True,
                         timeout=600)
    assert "TURBO REFUSE OK" in res.stdout, res.stdout + res.stderr


@pytest.mark.gpu
def test_turbo_pair_style_on_two_gpus_matches_c_abi(tmp_path, gpu_model, monkeypatch):
    """so3lr/b200/turbo with SO3LR_B200_TURBO_GPUS=2 over six partitions: two
    coordinators, each with its own GPU (devices 0 and 1) and its own pack of
    three images, no communication between them; every image's forces, energy
    and per-atom virials equal so3lr_compute_batch of its group's pack bit for
    bit."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from so3lr_b200.systems import turbo_batch
    monkeypatch.setenv("SO3LR_B200_TURBO_GPUS", "2")
    exe = _build(tmp_path)
    pos, z, off, q, m = turbo_batch(6, seed=13)
    inp = tmp_path / "images.txt"
    _write_images(inp, pos, z, off, q, m)
    out = _run_images(exe, MODEL, inp, 6)
    for g in range(2):
        ks = list(range(3 * g, 3 * g + 3))
        a, b = off[ks[0]], off[ks[-1] + 1]
        sub_off = off[ks[0]:ks[-1] + 2] - a
        ref = gpu_model.compute_batch(pos[a:b], z[a:b], sub_off, q[ks], m[ks])
        ref_va = gpu_model.virial_atom(b - a)
        for j, k in enumerate(ks):
            o = out[k]
            sl = slice(sub_off[j], sub_off[j + 1])
            assert np.array_equal(np.array(o["forces"]), ref["forces"][sl]), k
            assert o["energy"] == ref["image_energy"][j], k
            assert np.array_equal(np.array(o["vatom"]), ref_va[sl]), k
            assert f"gpu_group={g} of 2" in o["log"]
