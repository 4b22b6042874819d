"""The seeded synthetic inputs against the shapes and distributions the
benchmark configurations specify: water at 0.997 g/cm^3 (30.0 A^3 per
molecule), rigid O-H 0.9572 A and H-O-H 104.52 deg geometry, lattice jitter
with every O-O distance >= 2.5 A under the minimum image (also for the
weak-scaled multi-GPU boxes), Maxwell-Boltzmann velocities with zero net
momentum, and turbo packs of 4-16 water clusters with about half neutral, a
quarter OH- and a quarter H3O+ (all singlets)."""
import math

import numpy as np
import pytest

from so3lr_b200.systems import maxwell_boltzmann, min_oo_distance, turbo_batch, water_box


def _geometry(pos):
    o, h1, h2 = pos[0::3], pos[1::3], pos[2::3]
    r1 = np.linalg.norm(h1 - o, axis=1)
    r2 = np.linalg.norm(h2 - o, axis=1)
    cosang = ((h1 - o) * (h2 - o)).sum(1) / (r1 * r2)
    return r1, r2, np.degrees(np.arccos(cosang))


@pytest.mark.parametrize("nmol", [64, 1000, 8000, 16000])
def test_water_box_spec(nmol):
    w = water_box(nmol, seed=2026)
    assert len(w.z) == 3 * nmol and list(w.z[:3]) == [8, 1, 1]
    L = w.cell[0]
    assert abs(L ** 3 / nmol - 30.005) < 0.01  # A^3 per molecule at 0.997 g/cm^3
    r1, r2, ang = _geometry(w.pos)
    assert np.allclose(r1, 0.9572, atol=1e-12) and np.allclose(r2, 0.9572, atol=1e-12)
    assert np.allclose(ang, 104.52, atol=1e-9)
    assert min_oo_distance(w.pos[0::3], L, nmol) >= 2.5


def test_headline_box_is_the_measured_one():
    """Config 3's box (8,000 H2O, seed 2026) keeps its first jitter draw, so
    the positions of the measured runs do not change."""
    w = water_box(8000, seed=2026)
    assert abs(w.cell[0] - 62.14784361731874) < 1e-12
    assert min_oo_distance(w.pos[0::3], w.cell[0], 8000) >= 2.5


def test_maxwell_boltzmann_temperature_and_momentum():
    w = water_box(1000, seed=3)
    v = maxwell_boltzmann(w.mass, 300.0, seed=1)
    assert np.abs((v * w.mass[:, None]).sum(0)).max() < 1e-9
    kb, mvv2e = 8.617333262e-5, 1.0364269e-4
    t = (w.mass[:, None] * v ** 2).sum() * mvv2e / (3 * len(w.z) * kb)
    assert abs(t - 300.0) < 15.0


def test_turbo_pack_spec():
    pos, z, off, q, m = turbo_batch(1024, seed=7)
    sizes = np.diff(off)
    nmol = np.round(sizes / 3).astype(int)
    assert nmol.min() >= 4 and nmol.max() <= 16
    assert np.all(m == 1.0)
    frac = {c: float(np.mean(q == c)) for c in (0.0, -1.0, 1.0)}
    assert abs(frac[0.0] - 0.5) < 0.05 and abs(frac[-1.0] - 0.25) < 0.05 and abs(frac[1.0] - 0.25) < 0.05
    for k in range(len(sizes)):
        zk = z[off[k]:off[k + 1]]
        n_o, n_h = int((zk == 8).sum()), int((zk == 1).sum())
        assert n_h - 2 * n_o == int(q[k])  # OH- lacks one H, H3O+ has one more
        # every cluster is an isolated sphere at liquid density: atoms within ~ (3 V / 4 pi)^(1/3) + 1.5 A
        c = pos[off[k]:off[k + 1]]
        radius = (3 * n_o * 30.0 / (4 * math.pi)) ** (1 / 3)
        assert np.linalg.norm(c, axis=1).max() <= radius + 1.5


@pytest.mark.parametrize("kind, dq", [("neutral", 0), ("hydroxide", -1), ("hydronium", 1)])
def test_cluster_kinds(kind, dq):
    """Every cluster kind keeps whole O-H bonds of 0.9572 A; OH- lacks one H,
    H3O+ carries one more H on one oxygen, and O-O distances are >= 2.6 A."""
    from so3lr_b200.systems import water_cluster
    rng = np.random.default_rng(11)
    pos, z, q = water_cluster(8, rng, kind)
    assert q == dq and int((z == 8).sum()) == 8 and int((z == 1).sum()) == 16 + dq
    o = pos[z == 8]
    d = np.linalg.norm(o[:, None] - o[None, :], axis=-1) + np.eye(8) * 1e9
    assert d.min() >= 2.6
    for h in pos[z == 1]:  # every hydrogen sits on an oxygen at the O-H bond length
        assert abs(np.linalg.norm(o - h, axis=1).min() - 0.9572) < 1e-9
