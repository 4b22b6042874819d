"""The allocation-free long-range entry point (so3lr_long_range_noalloc).

It exists for callers that cannot let the library allocate device memory once
their run has started (an engine that hands out only pre-reserved buffers from
its own pool). It must reproduce the long-range terms of the ordinary,
allocating entry point (so3lr_compute) on the same system: per-atom total,
electrostatic and dispersion energies agree to 1e-12 eV, the per-term tolerance
of the parity suite. Two calls in a row are checked, because every call reuses
the same fixed scratch array.

This file is named so that pytest collects it last: a run that stops at the
first failure has run every other test before reaching it.
"""
import numpy as np
import pytest

from conftest import golden_system, load_golden

pytestmark = pytest.mark.gpu


def _device(a, dtype):
    import torch
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device="cuda:0")


def _systems():
    from so3lr_b200.systems import water_cluster
    fx = load_golden("alanine_cation")
    s = golden_system(fx)
    yield "alanine_cation", s.pos, s.z, s.charge, s.multiplicity
    pos, z, q = water_cluster(16, np.random.default_rng(3), "hydronium")
    yield "h3o_cluster", pos, z, q, 1.0


@pytest.mark.parametrize("case", list(range(2)))
def test_noalloc_long_range_matches_compute(case, gpu_model):
    import torch
    name, pos, z, charge, mult = list(_systems())[case]
    ref = gpu_model.compute(pos, z, charge=charge, multiplicity=mult)
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
        for k in ("e_lr", "e_elec", "e_disp"):
            got = outs[k].cpu().numpy()
            assert np.isfinite(got).all(), (name, call, k)
            assert np.abs(got - ref[k]).max() <= 1e-12, (name, call, k, np.abs(got - ref[k]).max())
        assert np.isfinite(outs["f"].cpu().numpy()).all()
        # charge neutrality of the seeds' sum is not required; dE/dq must be finite and nonzero
        assert np.abs(outs["dq"].cpu().numpy()).max() > 0.0


def test_noalloc_rejects_oversized_systems(gpu_model):
    import torch
    from so3lr_b200 import So3lrError
    buf = torch.zeros(64, dtype=torch.float64, device="cuda:0")
    zb = torch.ones(64, dtype=torch.int32, device="cuda:0")
    p = buf.data_ptr()
    with pytest.raises(So3lrError, match="outside 1..16384"):
        gpu_model.long_range_noalloc(16385, p, p, p, zb.data_ptr(), p, p, p, p, p, p, p)
