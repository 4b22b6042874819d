"""The allocation-free long-range entry point (so3lr_long_range_noalloc).

It exists for callers that cannot let the library allocate device memory once
their run has started (an engine that hands out only pre-reserved buffers from
its own pool). Every output it writes is checked:

* per-atom total, electrostatic and dispersion energies against the ordinary,
  allocating entry point (so3lr_compute) on the same system, to 1e-12 eV;
* dE/dq and dE/d(ratio) to 1e-10, the direct long-range force to 1e-9 eV/A and
  the per-atom virial to 1e-9 eV, against the CPU oracle's long-range term
  evaluated alone for the same charges and ratios (oracle.long_range_only).

Two calls in a row are checked, because every call reuses the same fixed
scratch array. The 3,000-atom droplet is the size at which the allocating path
switches to its open-boundary cell grid, while this entry point always scans
the single image: the two sum in different orders and must still agree.

This file is named so that pytest collects it last: a run that stops at the
first failure has run every other test before reaching it.
"""
import numpy as np
import pytest

from conftest import golden_system, load_golden

pytestmark = pytest.mark.gpu

TOL = {"e_lr": 1e-12, "e_elec": 1e-12, "e_disp": 1e-12, "dq": 1e-10, "dh": 1e-10, "f": 1e-9, "w": 1e-9}


def _device(a, dtype):
    import torch
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device="cuda:0")


def _system(case):
    from so3lr_b200.systems import water_cluster
    if case == "alanine_cation":
        s = golden_system(load_golden("alanine_cation"))
        return s.pos, s.z, s.charge, s.multiplicity
    if case == "h3o_cluster":
        pos, z, q = water_cluster(16, np.random.default_rng(3), "hydronium")
        return pos, z, q, 1.0
    pos, z, q = water_cluster(1000, np.random.default_rng(5), "neutral")
    return pos, z, q, 1.0


@pytest.mark.parametrize("case", ["alanine_cation", "h3o_cluster", "droplet_3000"])
def test_noalloc_long_range_every_output(case, gpu_model, oracle_model):
    import torch
    from oracle.so3lr_oracle import long_range_only
    pos, z, charge, mult = _system(case)
    ref = gpu_model.compute(pos, z, charge=charge, multiplicity=mult)
    lr = long_range_only(oracle_model, pos, z, ref["charges"], ref["ratios"])
    expect = {"e_lr": ref["e_lr"], "e_elec": ref["e_elec"], "e_disp": ref["e_disp"], "dq": lr["dq"],
              "dh": lr["dh"], "f": lr["f"].reshape(-1), "w": lr["virial_atom"].reshape(-1)}
    # the oracle's energies and the allocating path's agree as well
    for k in ("e_lr", "e_elec", "e_disp"):
        assert np.abs(lr[k] - ref[k]).max() <= 1e-12, (case, k)
    n = len(z)
    x_d = _device(pos, torch.float64)
    q_d = _device(ref["charges"], torch.float64)
    h_d = _device(ref["ratios"], torch.float64)
    z_d = _device(z, torch.int32)
    for call in range(2):
        outs = {k: torch.full((n * w,), float("nan"), dtype=torch.float64, device="cuda:0")
                for k, w in (("e_lr", 1), ("e_elec", 1), ("e_disp", 1), ("dq", 1), ("dh", 1), ("f", 3), ("w", 6))}
        gpu_model.long_range_noalloc(n, x_d.data_ptr(), q_d.data_ptr(), h_d.data_ptr(), z_d.data_ptr(),
                                     outs["e_lr"].data_ptr(), outs["e_elec"].data_ptr(), outs["e_disp"].data_ptr(),
                                     outs["dq"].data_ptr(), outs["dh"].data_ptr(), outs["f"].data_ptr(),
                                     outs["w"].data_ptr())
        torch.cuda.synchronize()
        for k, tol in TOL.items():
            got = outs[k].cpu().numpy()
            assert np.isfinite(got).all(), (case, call, k)
            err = np.abs(got - expect[k]).max()
            assert err <= tol, (case, call, k, err)
        # the rows sum to the long-range part of the global virial; dE/dq is not all zero
        assert np.abs(outs["dq"].cpu().numpy()).max() > 0.0


def test_noalloc_rejects_oversized_systems(gpu_model):
    import torch
    from so3lr_b200 import So3lrError
    buf = torch.zeros(64, dtype=torch.float64, device="cuda:0")
    zb = torch.ones(64, dtype=torch.int32, device="cuda:0")
    p = buf.data_ptr()
    with pytest.raises(So3lrError, match="outside 1..16384"):
        gpu_model.long_range_noalloc(16385, p, p, p, zb.data_ptr(), p, p, p, p, p, p, p)
