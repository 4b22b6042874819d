"""Periodic multi-image neighbour lists for the CPU oracle (test infrastructure).

ORACLE — test infrastructure; see oracle/__init__.py for who may import it.

The reference receives LAMMPS neighbour lists and keeps, every step, the
candidates with ``0 < r^2 < rc^2`` (pair_so3lr_native_mpi.cpp:258-291,
``count_active_device_edges``): a FULL list at the 4.5 A short-range cutoff and a
HALF list (newton on) at the 12 A long-range cutoff
(pair_so3lr_native_mpi.cpp:1174-1192). LAMMPS supplies periodic images as ghost
atoms, so a box shorter than twice a cutoff yields several images of the same
atom; this module reproduces that by explicit image shifts.

Conventions (shared with the CUDA path): an edge is ``(receiver r, sender s,
shift S)`` and its vector is ``v = x_r - (x_s + S)``, the receiver-minus-sender
vector the reference stores (learned_energy_forces.cpp:217-219).
"""
from __future__ import annotations

import numpy as np
from scipy.spatial import cKDTree


def _image_range(length: float, periodic: bool, cutoff: float) -> int:
    if not periodic:
        return 0
    return int(np.ceil(cutoff / length))


def directed_pairs(pos: np.ndarray, cell: np.ndarray | None, cutoff: float,
                   pbc=(True, True, True)):
    """All directed (receiver, sender, shift) with 0 < r^2 < cutoff^2.

    ``cell`` holds the three orthorhombic box lengths, or None for an open
    system. Returns int64 receivers, senders and float64 shifts (E x 3),
    sorted by receiver, then sender, then shift.
    """
    pos = np.asarray(pos, dtype=np.float64)
    n = len(pos)
    if n == 0:
        return (np.zeros(0, np.int64), np.zeros(0, np.int64), np.zeros((0, 3)))
    if cell is None:
        shifts = np.zeros((1, 3))
    else:
        cell = np.asarray(cell, dtype=np.float64)
        ranges = [range(-_image_range(cell[d], pbc[d], cutoff),
                        _image_range(cell[d], pbc[d], cutoff) + 1) for d in range(3)]
        shifts = np.array([[a, b, c] for a in ranges[0] for b in ranges[1] for c in ranges[2]],
                          dtype=np.float64) * cell[None, :]
    images = (pos[None, :, :] + shifts[:, None, :]).reshape(-1, 3)
    tree_base = cKDTree(pos)
    tree_img = cKDTree(images)
    # generous radius; the exact strict cutoff is applied below on the vectors
    sparse = tree_base.sparse_distance_matrix(tree_img, cutoff * (1 + 1e-9) + 1e-9,
                                              output_type="ndarray")
    recv = sparse["i"].astype(np.int64)
    img = sparse["j"].astype(np.int64)
    send = img % n
    shift = shifts[img // n]
    vec = pos[recv] - (pos[send] + shift)
    r2 = np.einsum("ij,ij->i", vec, vec)
    keep = (r2 > 0.0) & (r2 < cutoff * cutoff)
    recv, send, shift = recv[keep], send[keep], shift[keep]
    order = np.lexsort((shift[:, 2], shift[:, 1], shift[:, 0], send, recv))
    return recv[order], send[order], shift[order]


def half_pairs(pos, cell, cutoff, pbc=(True, True, True)):
    """Unordered pairs, each once: keep (i, j, S) with i < j, or i == j and S > 0
    lexicographically. Matches a LAMMPS newton-on half list up to orientation."""
    recv, send, shift = directed_pairs(pos, cell, cutoff, pbc)
    lex_pos = (shift[:, 0] > 0) | ((shift[:, 0] == 0) & ((shift[:, 1] > 0) |
                                                         ((shift[:, 1] == 0) & (shift[:, 2] > 0))))
    keep = (recv < send) | ((recv == send) & lex_pos)
    return recv[keep], send[keep], shift[keep]
