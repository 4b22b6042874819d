"""Optional operators of other checkpoints (reference src/so3lr_capabilities.cpp:46-80):
RMSNorm without scale, no second block norm, query/key normalisation,
residual scalars, the NLH repulsion, ratio heads with fewer keys and the C6
ratio head. Synthetic model files
(tests/model_variants.py) switch each one on. CPU: the native loader accepts
them and refuses what the reference refuses; the oracle's restatement reduces to
the base model where it must. GPU: each variant against the oracle.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import MODEL
from model_variants import make_l_variant, make_variant
from so3lr_b200.model_file import write_model

RESID = ([0.9, 1.1, 0.8], [0.1, -0.2, 0.3])

VARIANTS = {
    "rms_norm": dict(rms_norm=True),
    "no_second_norm": dict(second_norm=False, attention_norm_factor=20.0),
    "qk_norm": dict(qk_norm=True, attention_norm_factor=20.0),
    "residual_scalars": dict(residual_scalars=RESID),
    "nlh": dict(nlh_capacity=10, seed=1),
    "c6_head": dict(c6_keys=64, seed=3),
    "a0_c6_one_key": dict(hirshfeld_keys=1, c6_keys=1, seed=4),
    "all": dict(rms_norm=True, qk_norm=True, residual_scalars=RESID, nlh_capacity=9, hirshfeld_keys=1, c6_keys=1,
                seed=2, attention_norm_factor=20.0),
    # F = 256, 8 heads, 64 radial functions, degrees [1,1,2,2,3,3,4,4]
    "l_size": dict(l_size=True, seed=7),
}


@pytest.fixture(scope="module")
def variant_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("variants")


def _variant(variant_dir, name):
    path = variant_dir / f"{name}.so3lr"
    if not path.exists():
        kw = dict(VARIANTS[name])
        if kw.pop("l_size", False):
            make_l_variant(MODEL, path, **kw)
        else:
            make_variant(MODEL, path, **kw)
    return path


def _inspect(path):
    from so3lr_b200.runtime import LIB_PATH, ArchInfo
    lib = C.CDLL(str(LIB_PATH))
    info = ArchInfo()
    err = C.create_string_buffer(4096)
    rc = lib.so3lr_inspect_model(str(path).encode(), C.byref(info), err, 4096)
    return rc, err.value.decode(), info


def test_writer_round_trips_the_shipped_model(variant_dir):
    """Rewriting every tensor unchanged keeps each one's shape (0-d included),
    dtype and bytes."""
    from oracle.model_io import load_model
    base = load_model(str(MODEL))
    path = write_model(variant_dir / "copy.so3lr", base.manifest,
                       [(r, base.tensors[r["state_key"]]) for r in base.manifest["tensors"]])
    copy = load_model(str(path))
    for r in base.manifest["tensors"]:
        a, b = base.tensors[r["state_key"]], copy.tensors[r["state_key"]]
        assert a.shape == b.shape and a.dtype == b.dtype and a.tobytes() == b.tobytes(), r["state_key"]
    assert _inspect(path)[0] == 0


def test_model_file_tool(variant_dir, capsys):
    """python -m so3lr_b200.model_file: PASS and the summary for the shipped
    model, FAIL with the loader's message for a corrupted copy; its tensor
    reader agrees with the oracle's."""
    from oracle.model_io import load_model
    from so3lr_b200 import model_file
    assert model_file.main([str(MODEL), "--manifest", str(variant_dir / "manifest.json")]) == 0
    out = capsys.readouterr().out
    assert "native_model_check=PASS" in out and "tensor_count=213" in out and "long_range_cutoff=12.0" in out
    assert '"model_family": "SO3LR"' in (variant_dir / "manifest.json").read_text()
    data = bytearray(MODEL.read_bytes())
    data[-3] ^= 0x40
    bad = variant_dir / "corrupt.so3lr"
    bad.write_bytes(bytes(data))
    assert model_file.main([str(bad)]) == 1
    assert "SHA-256" in capsys.readouterr().out
    ref = load_model(str(MODEL)).tensors
    mine = model_file.tensors(MODEL)
    assert ref.keys() == mine.keys()
    for k in ref:
        assert ref[k].shape == mine[k].shape and np.array_equal(ref[k], mine[k]), k


@pytest.mark.parametrize("name", sorted(VARIANTS))
def test_native_loader_accepts_variant(name, variant_dir):
    rc, err, info = _inspect(_variant(variant_dir, name))
    assert rc == 0, err
    assert ("repulsion=nlh" in info.summary.decode()) == ("nlh_capacity" in VARIANTS[name])
    if "l_size" in VARIANTS[name]:
        assert (info.features, info.heads, info.rbf, info.ev_width, info.degrees) == (256, 8, 64, 48, 4)
        assert "degrees=[1,1,2,2,3,3,4,4]" in info.summary.decode()


def test_native_loader_refuses_other_widths(variant_dir):
    """Shapes outside the two compiled widths are refused with the loader's
    reason: F = 256 with the F = 128 degree list, and a 256-wide model that
    declares 32 radial functions."""
    from oracle.model_io import load_model
    base = load_model(str(_variant(variant_dir, "l_size")))
    cases = [("l_degrees", "model.euclidean_transformers.0.euclidean_attention_block.degree_repeats",
              np.array([3, 5, 7, 9, 3, 5, 7, 9], dtype=np.int64), None, "degree_repeats must be [3,3,5,5,7,7,9,9]"),
             ("l_rbf32", None, None, dict(radial_basis_features=32), "radial_basis_features must be 64")]
    for tag, key, value, arch, needle in cases:
        import copy as _copy
        man = _copy.deepcopy(base.manifest)
        if arch:
            man["architecture"].update(arch)
        tensors = [(r, value if r["state_key"] == key else base.tensors[r["state_key"]]) for r in man["tensors"]]
        rc, err, _ = _inspect(write_model(variant_dir / f"bad_{tag}.so3lr", man, tensors))
        assert rc != 0 and needle in err, (tag, err)


def test_oracle_l_size_is_rotation_invariant(variant_dir):
    """The duplicated-degree layout keeps the model equivariant: rotating a
    molecule leaves the energy and charges unchanged and rotates the forces
    (a slot fed harmonics of another degree would break this)."""
    from oracle.so3lr_oracle import OracleModel, System, evaluate
    from so3lr_b200.systems import turbo_batch
    m = OracleModel.load(str(_variant(variant_dir, "l_size")))
    pos, z, off, q, mult = turbo_batch(3, seed=13)
    sl = slice(off[2], off[3])
    p0 = pos[sl] - pos[sl].mean(axis=0)
    rot, _ = np.linalg.qr(np.random.default_rng(3).standard_normal((3, 3)))
    a = evaluate(m, System(pos=p0, z=z[sl], charge=q[2], multiplicity=mult[2]))
    b = evaluate(m, System(pos=p0 @ rot.T, z=z[sl], charge=q[2], multiplicity=mult[2]))
    assert abs(a["energy"] - b["energy"]) <= 1e-9 * abs(a["energy"])
    assert np.abs(a["forces"] @ rot.T - b["forces"]).max() <= 1e-9 * (1 + np.abs(a["forces"]).max())
    assert np.abs(a["partial_charges"] - b["partial_charges"]).max() <= 1e-12


def _mutated(variant_dir, tag, mutate_manifest=None, drop=(), add=()):
    from oracle.model_io import load_model
    base = load_model(str(MODEL))
    man = base.manifest
    if mutate_manifest:
        mutate_manifest(man["architecture"])
    tensors = [(r, base.tensors[r["state_key"]]) for r in man["tensors"] if r["state_key"] not in drop]
    tensors += list(add)
    return write_model(variant_dir / f"bad_{tag}.so3lr", man, tensors)


def test_native_loader_refuses_what_the_reference_refuses(variant_dir):
    cases = [
        ("norm1_off", lambda a: a.update(layer_normalization_1=False), (), (), "first block norm"),
        ("repulsion_none", lambda a: a.update(repulsion_type="none"), (), (), "repulsion_type 'none'"),
        ("resid_missing", lambda a: a.update(use_residual_scalars=True), (), (), "model.resid_lambdas"),
        ("nlh_missing", lambda a: a.update(repulsion_type="nlh"), (), (), "physical.nlh_a"),
        ("nlh_shape", lambda a: a.update(repulsion_type="nlh"), (),
         [({"name": k, "state_key": k, "dtype": "float64", "role": "physical_constant"}, np.ones((4, 4, 2)))
          for k in ("physical.nlh_a", "physical.nlh_b")], "[cap, cap, 3]"),
        ("qk_nonlin", lambda a: a.update(qk_nonlinearity="silu"), (), (), "qk_nonlinearity"),
        ("mlp2", lambda a: a.update(residual_mlp_2=True), (), (), "residual_mlp_1"),
    ]
    for tag, mut, drop, add, needle in cases:
        rc, err, _ = _inspect(_mutated(variant_dir, tag, mut, drop, add))
        assert rc != 0 and needle in err, (tag, err)


def test_oracle_identity_residual_scalars_equal_base_model(variant_dir, oracle_model):
    """resid = 1, x0 = 0 before every block is the plain stack."""
    from oracle.so3lr_oracle import OracleModel, System, evaluate
    from so3lr_b200.systems import water_box
    path = make_variant(MODEL, variant_dir / "resid_identity.so3lr", residual_scalars=([1.0] * 3, [0.0] * 3))
    w = water_box(8, seed=5)
    a = evaluate(oracle_model, System(pos=w.pos, z=w.z, cell=w.cell))
    b = evaluate(OracleModel.load(str(path)), System(pos=w.pos, z=w.z, cell=w.cell))
    assert a["energy"] == b["energy"]
    assert np.array_equal(a["forces"], b["forces"])


def test_oracle_nlh_repulsion_matches_the_pair_formula(variant_dir):
    """NLH energy of one O-H pair: 0.5 * 2 * switch(r) * ke Z_O Z_H phi(r) / r *
    sum_k a_k exp(-b_k r), tables indexed (min Z, max Z) (physical_zbl.cpp:81-178)."""
    import math
    from oracle.so3lr_oracle import OracleModel, System, evaluate
    path = _variant(variant_dir, "nlh")
    m = OracleModel.load(str(path))
    r = 0.93
    o = evaluate(m, System(pos=np.array([[0.0, 0.0, 0.0], [r, 0.0, 0.0]]), z=np.array([8, 1]), multiplicity=2.0))
    a = m.file.arch
    ta, tb = m.file.t("physical.nlh_a"), m.file.t("physical.nlh_b")
    y = sum(ta[0, 7, k] * math.exp(-tb[0, 7, k] * r) for k in range(3))
    x = r / m.r_sr
    phi = 1 - 10 * x ** 3 + 15 * x ** 4 - 6 * x ** 5
    c = r / float(a["zbl_switch_off_angstrom"])
    sl, sr = math.exp(-1 / (1 - c)), math.exp(-1 / c)
    sw = sl / (sl + sr + 1e-12)
    e = sw * float(a["zbl_ke"]) * phi * 8.0 / r * y
    assert abs(o["zbl_energy"].sum() - e) <= 1e-12 * abs(e)


def _cases():
    from so3lr_b200.systems import turbo_batch, water_box
    w = water_box(27, seed=9)
    pos, z, off, q, m = turbo_batch(3, seed=13)
    k = 2  # one charged cluster, open boundaries
    sl = slice(off[k], off[k + 1])
    return [("box27", w.pos, w.z, w.cell, w.boxlo, 0.0, 1.0), ("cluster", pos[sl], z[sl], None, None, q[k], m[k])]


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(VARIANTS))
def test_gpu_variant_matches_oracle(name, variant_dir):
    """Energy per atom <= 1e-9 eV, forces <= 1e-9 (1 + max|F|) eV/A, virial <=
    1e-8 (1 + max|W|) eV: the float64 bar of the shipped model."""
    from oracle.so3lr_oracle import OracleModel, System, evaluate
    from so3lr_b200 import So3lrB200
    path = _variant(variant_dir, name)
    om = OracleModel.load(str(path))
    g = So3lrB200(path, 0)
    try:
        for case, pos, z, cell, lo, q, mult in _cases():
            o = evaluate(om, System(pos=pos, z=z, cell=cell, charge=q, multiplicity=mult))
            r = g.compute(pos, z, cell=cell, boxlo=lo, charge=q, multiplicity=mult)
            fmax = np.abs(o["forces"]).max()
            assert abs(r["energy"] - o["energy"]) / len(z) <= 1e-9, (case, r["energy"], o["energy"])
            assert np.abs(r["forces"] - o["forces"]).max() <= 1e-9 * (1 + fmax), case
            assert np.abs(r["virial"] - o["virial"]).max() <= 1e-8 * (1 + np.abs(o["virial"]).max()), case
            assert np.abs(r["charges"] - o["partial_charges"]).max() <= 1e-10, case
            assert np.abs(r["ratios"] - o["hirshfeld_ratios"]).max() <= 1e-10, case
    finally:
        g.close()


@pytest.mark.gpu
def test_gpu_l_size_refuses_mixed_precision(variant_dir):
    """The mixed-precision filter kernels exist for F = 128 only: an F = 256
    handle refuses SO3LR_PRECISION_MIXED with the reason and keeps float64."""
    from so3lr_b200 import So3lrB200
    from so3lr_b200.runtime import So3lrError
    g = So3lrB200(_variant(variant_dir, "l_size"), 0)
    try:
        with pytest.raises(So3lrError, match="F = 128 models only"):
            g.set_precision("mixed")
        g.set_precision("float64")
    finally:
        g.close()
