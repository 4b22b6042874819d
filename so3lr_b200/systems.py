"""Seeded synthetic inputs with the shapes of the benchmark configurations.

Water boxes follow the recipe of the reference's scaling inputs
(examples/scaling/generate_water_boxes.py:53-102: rigid H2O on a cubic lattice
with random-quaternion orientations) with the benchmark's additions: O-H
0.9572 A, H-O-H 104.52 deg, lattice jitter, a minimum O-O distance of 2.5 A and
a density of 0.997 g/cm^3. Clusters are open-boundary spheres of 4..16 waters
at liquid density, 50 % neutral, 25 % OH- (one H removed) and 25 % H3O+ (one H
added), all singlets. There is no public dataset for this path; these seeded
systems stand in for the reference's generated boxes.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

R_OH = 0.9572
THETA = math.radians(104.52)
MASS = {1: 1.008, 8: 15.999}
WATER_MASS_AMU = 2 * 1.008 + 15.999
AVOGADRO = 6.02214076e23


def molecule_frame() -> np.ndarray:
    """O at the origin, the two H in the xy plane (3 x 3)."""
    h = 0.5 * THETA
    return np.array([[0.0, 0.0, 0.0],
                     [R_OH * math.sin(h), R_OH * math.cos(h), 0.0],
                     [-R_OH * math.sin(h), R_OH * math.cos(h), 0.0]])


def random_rotation(rng: np.random.Generator) -> np.ndarray:
    u1, u2, u3 = rng.random(3)
    w = math.sqrt(1 - u1) * math.sin(2 * math.pi * u2)
    x = math.sqrt(1 - u1) * math.cos(2 * math.pi * u2)
    y = math.sqrt(u1) * math.sin(2 * math.pi * u3)
    z = math.sqrt(u1) * math.cos(2 * math.pi * u3)
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
                     [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
                     [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]])


def box_length(n_molecules: int, density_g_cm3: float = 0.997) -> float:
    volume_cm3 = n_molecules * WATER_MASS_AMU / (AVOGADRO * density_g_cm3)
    return (volume_cm3 * 1e24) ** (1.0 / 3.0)


@dataclass
class WaterSystem:
    pos: np.ndarray          # N x 3, Angstrom
    z: np.ndarray            # N, int32
    cell: np.ndarray | None  # box lengths or None
    boxlo: np.ndarray
    mass: np.ndarray         # g/mol
    charge: float = 0.0
    multiplicity: float = 1.0


def min_oo_distance(centers: np.ndarray, L: float, n_molecules: int) -> float:
    """Smallest minimum-image distance between the molecule centres (the O
    atoms): a dense comparison for small boxes, a periodic k-d tree for large
    ones."""
    if n_molecules < 2:
        return math.inf
    if n_molecules <= 4000:
        d = centers[:, None, :] - centers[None, :, :]
        d -= L * np.round(d / L)
        return float((np.sqrt((d * d).sum(-1)) + np.eye(n_molecules) * 1e9).min())
    from scipy.spatial import cKDTree
    x = np.mod(centers, L)
    dist, _ = cKDTree(x, boxsize=L).query(x, k=2)
    return float(dist[:, 1].min())


def close_molecules(centers: np.ndarray, L: float, min_oo: float) -> np.ndarray:
    """One molecule (the first) of every pair closer than min_oo under the
    minimum image, from a periodic k-d tree."""
    from scipy.spatial import cKDTree
    x = np.mod(centers, L)
    pairs = cKDTree(x, boxsize=L).query_pairs(min_oo, output_type="ndarray")
    return np.unique(pairs[:, 0]) if len(pairs) else np.zeros(0, dtype=np.int64)


def water_box(n_molecules: int, seed: int, density: float = 0.997, jitter: float = 0.1,
              min_oo: float = 2.5) -> WaterSystem:
    """Periodic cubic water box."""
    rng = np.random.default_rng(seed)
    L = box_length(n_molecules, density)
    ng = int(math.ceil(n_molecules ** (1.0 / 3.0)))
    spacing = L / ng
    sites = np.array([[i, j, k] for i in range(ng) for j in range(ng) for k in range(ng)], dtype=np.float64)
    order = rng.permutation(len(sites))[:n_molecules]
    centers = (sites[np.sort(order)] + 0.5) * spacing
    base = molecule_frame()
    # jitter the lattice, keeping O-O >= min_oo under the minimum image
    if n_molecules <= 4000:
        # small boxes: redraw the whole jitter (fixes the boxes the tests use)
        for attempt in range(50):
            trial = centers + rng.uniform(-jitter, jitter, centers.shape) * spacing
            if min_oo_distance(trial, L, n_molecules) >= min_oo:
                break
        else:
            trial = centers
    else:
        # large boxes: some pair is almost always too close, so only the
        # molecules of close pairs get a new jitter, until none is left
        trial = centers + rng.uniform(-jitter, jitter, centers.shape) * spacing
        for attempt in range(200):
            close = close_molecules(trial, L, min_oo)
            if len(close) == 0:
                break
            trial[close] = centers[close] + rng.uniform(-jitter, jitter, (len(close), 3)) * spacing
        else:
            trial = centers
    centers = trial
    pos = np.empty((3 * n_molecules, 3))
    for m in range(n_molecules):
        rot = random_rotation(rng)
        pos[3 * m:3 * m + 3] = centers[m] + base @ rot.T
    z = np.tile(np.array([8, 1, 1], dtype=np.int32), n_molecules)
    mass = np.array([MASS[int(q)] for q in z])
    return WaterSystem(pos=pos, z=z, cell=np.array([L, L, L]), boxlo=np.zeros(3), mass=mass)


def maxwell_boltzmann(mass: np.ndarray, temperature: float, seed: int) -> np.ndarray:
    """Velocities in A/ps (LAMMPS metal) at `temperature` K, zero net momentum."""
    rng = np.random.default_rng(seed)
    kb = 8.617333262e-5          # eV/K
    mvv2e = 1.0364269e-4         # (g/mol) A^2/ps^2 -> eV
    sigma = np.sqrt(kb * temperature / (mass * mvv2e))
    v = rng.normal(size=(len(mass), 3)) * sigma[:, None]
    p = (v * mass[:, None]).sum(0) / mass.sum()
    return v - p


def water_cluster(n_molecules: int, rng: np.random.Generator, kind: str = "neutral"):
    """Open-boundary water cluster inside a sphere at liquid density (config 5).

    kind: 'neutral' (Q=0), 'hydroxide' (one H removed, Q=-1) or 'hydronium'
    (one H added to a random O, Q=+1). All singlets."""
    volume = n_molecules * 30.0
    radius = (3 * volume / (4 * math.pi)) ** (1 / 3)
    centers = []
    while len(centers) < n_molecules:
        c = rng.uniform(-radius, radius, 3)
        if np.linalg.norm(c) > radius:
            continue
        if all(np.linalg.norm(c - o) >= 2.6 for o in centers):
            centers.append(c)
    base = molecule_frame()
    pos, z = [], []
    for c in centers:
        pos.append(c + base @ random_rotation(rng).T)
        z.append([8, 1, 1])
    pos = np.concatenate(pos)
    z = np.concatenate(z).astype(np.int32)
    charge = 0.0
    if kind == "hydroxide":
        m = rng.integers(n_molecules)
        drop = 3 * m + 1 + rng.integers(2)
        pos = np.delete(pos, drop, axis=0)
        z = np.delete(z, drop)
        charge = -1.0
    elif kind == "hydronium":
        m = rng.integers(n_molecules)
        o = pos[3 * m]
        h1, h2 = pos[3 * m + 1] - o, pos[3 * m + 2] - o
        bis = -(h1 + h2)
        bis /= np.linalg.norm(bis)
        normal = np.cross(h1, h2)
        normal /= np.linalg.norm(normal)
        new_h = o + R_OH * (0.35 * bis + 0.94 * normal) / np.linalg.norm(0.35 * bis + 0.94 * normal)
        pos = np.insert(pos, 3 * m + 3, new_h, axis=0)
        z = np.insert(z, 3 * m + 3, 1)
        charge = 1.0
    return pos, z, charge


def turbo_batch(n_clusters: int, seed: int, min_mol: int = 4, max_mol: int = 16):
    """Packed clusters (config 5). Returns positions, Z, image offsets, per-image Q and M."""
    rng = np.random.default_rng(seed)
    pos, z, offsets, charges = [], [], [0], []
    for k in range(n_clusters):
        n = int(rng.integers(min_mol, max_mol + 1))
        u = rng.random()
        kind = "neutral" if u < 0.5 else ("hydroxide" if u < 0.75 else "hydronium")
        p, zz, q = water_cluster(n, rng, kind)
        pos.append(p + np.array([0.0, 0.0, 0.0]))
        z.append(zz)
        offsets.append(offsets[-1] + len(zz))
        charges.append(q)
    return (np.concatenate(pos), np.concatenate(z).astype(np.int32), np.array(offsets, dtype=np.int64),
            np.array(charges), np.ones(n_clusters))
