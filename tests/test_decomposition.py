"""Spatial decomposition across GPUs.

CPU part (gloo, world size 2): every rank computes the brick partition of the
same positions and gets the same owners; every atom has exactly one owner and
the bricks are balanced. GPU part (2 GPUs, skipped with fewer): one process per
GPU joins an NCCL group through the C ABI, evaluates the same periodic box, and
the energy, forces and virial are bit-identical to the single-GPU result (the
north-star requirement, reference VALIDATION.md:49-57).
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import MODEL


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _partition_worker(rank, world, port, result_q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from so3lr_b200.runtime import partition
    from so3lr_b200.systems import water_box
    w = water_box(512, seed=3)
    owners = {}
    for nr in (2, 4, 8):
        o = torch.from_numpy(partition(w.pos, w.boxlo, w.cell, nr).astype(np.int64))
        gathered = [torch.empty_like(o) for _ in range(world)]
        dist.all_gather(gathered, o)
        owners[nr] = [g.numpy() for g in gathered]
    dist.barrier()
    dist.destroy_process_group()
    result_q.put((rank, owners))


def test_partition_consistent_across_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_partition_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for nr, per_rank in results[0].items():
        a, b = per_rank
        assert np.array_equal(a, b)
        counts = np.bincount(a, minlength=nr)
        assert counts.sum() == len(a) and (counts > 0).all()
        assert counts.max() <= 1.35 * counts.mean(), counts


def _gpu_worker(rank, world, uid, nmol, seed, result_q, model=MODEL):
    try:
        from so3lr_b200 import So3lrB200
        from so3lr_b200.systems import water_box
        m = So3lrB200(model, rank)
        m.comm_init(world, rank, uid)
        w = water_box(nmol, seed=seed)
        out = m.compute(w.pos, w.z, cell=w.cell, boxlo=w.boxlo)
        va = m.virial_atom(len(w.z))
        result_q.put((rank, out["energy"], out["forces"], out["virial"], out["charges"], m.owned_atoms(), va, None))
        m.close()
    except Exception as exc:  # report to the parent instead of hanging it
        result_q.put((rank, None, None, None, None, 0, None, repr(exc)))


def _nvt_worker(rank, world, uid, nmol, seed, steps, result_q):
    try:
        from so3lr_b200 import So3lrB200
        from so3lr_b200.systems import maxwell_boltzmann, water_box
        m = So3lrB200(MODEL, rank)
        if world > 1:
            m.comm_init(world, rank, uid)
        w = water_box(nmol, seed=seed)
        v = maxwell_boltzmann(w.mass, 300.0, seed=seed)
        m.md_init(w.pos, w.z, w.cell, w.boxlo, v, w.mass)
        m.md_thermostat(300.0, 0.05, 3)
        m.md_run(steps, 0.0005)
        st = m.md_state(len(w.z))
        result_q.put((rank, st["x"], st["v"], st["energy"], m.md_thermostat_energy(), None))
        m.close()
    except Exception as exc:  # report to the parent instead of hanging it
        result_q.put((rank, None, None, None, None, repr(exc)))


@pytest.mark.gpu
def test_multi_gpu_nvt_trajectory_bit_identical():
    """A Nose-Hoover (NVT) trajectory on 2 GPUs equals the single-GPU one bit
    for bit: the chain's kinetic energy is an exact sum and every rank updates
    the chain identically."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from so3lr_b200 import So3lrB200
    ctx = mp.get_context("spawn")
    nmol, seed, steps = 1000, 23, 10
    q1 = ctx.Queue()
    p1 = ctx.Process(target=_nvt_worker, args=(0, 1, None, nmol, seed, steps, q1))
    p1.start()
    ref = q1.get(timeout=300)
    p1.join(timeout=120)
    assert ref[5] is None, ref[5]
    uid = So3lrB200.nccl_unique_id()
    q = ctx.Queue()
    procs = [ctx.Process(target=_nvt_worker, args=(r, 2, uid, nmol, seed, steps, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, x, v, e, ech, err in res:
        assert err is None, err
        assert np.array_equal(x, ref[1]) and np.array_equal(v, ref[2])
        assert e == ref[3] and ech == ref[4]


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_gpu_bit_identical(world, gpu_model):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from so3lr_b200 import So3lrB200
    from so3lr_b200.systems import water_box
    nmol, seed = 1000, 17
    w = water_box(nmol, seed=seed)
    ref = gpu_model.compute(w.pos, w.z, cell=w.cell, boxlo=w.boxlo)
    ref_va = gpu_model.virial_atom(len(w.z))
    uid = So3lrB200.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gpu_worker, args=(r, world, uid, nmol, seed, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, e, f, vir, chg, owned, va, err in res:
        assert err is None, err
        assert 0 < owned < len(w.z)
        assert e == ref["energy"], (e, ref["energy"])
        assert np.array_equal(f, ref["forces"]), np.abs(f - ref["forces"]).max()
        assert np.array_equal(vir, ref["virial"])
        assert np.array_equal(chg, ref["charges"])
        assert np.array_equal(va, ref_va)


def _local_worker(rank, world, uid, nmol, seed, steps, result_q):
    """Rank `rank` passes only its share of the atoms (a random split, not the
    library's bricks) to so3lr_compute_local, for `steps` positions."""
    try:
        from so3lr_b200 import So3lrB200
        from so3lr_b200.systems import water_box
        m = So3lrB200(MODEL, rank)
        m.comm_init(world, rank, uid)
        w = water_box(nmol, seed=seed)
        n = len(w.z)
        mine = np.nonzero(np.random.default_rng(seed).integers(0, world, n) == rank)[0]
        out = []
        for k in range(steps):
            pos = w.pos + 0.01 * k * np.sin(np.arange(3 * n).reshape(n, 3))
            r = m.compute_local(n, mine + 1, pos[mine], w.z[mine], cell=w.cell, boxlo=w.boxlo, vatom=True)
            out.append((r["energy"], r["virial"], r["forces"], r["eatom"], r["vatom"]))
        result_q.put((rank, mine, out, None))
        m.close()
    except Exception as exc:  # report to the parent instead of hanging it
        result_q.put((rank, None, None, repr(exc)))


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_gpu_local_frames_bit_identical(world, gpu_model):
    """Every rank passes only its own atoms (as a LAMMPS rank does) through
    so3lr_compute_local: each gets its atoms' forces, energies and per-atom
    virials, bit-identical to the single-GPU evaluation of the whole system,
    on a first call and on two later positions."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from so3lr_b200 import So3lrB200
    from so3lr_b200.systems import water_box
    nmol, seed, steps = 1000, 29, 3
    w = water_box(nmol, seed=seed)
    n = len(w.z)
    refs = []
    for k in range(steps):
        pos = w.pos + 0.01 * k * np.sin(np.arange(3 * n).reshape(n, 3))
        r = gpu_model.compute(pos, w.z, cell=w.cell, boxlo=w.boxlo)
        refs.append((r, gpu_model.virial_atom(n)))
    uid = So3lrB200.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_local_worker, args=(r, world, uid, nmol, seed, steps, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    seen = np.zeros(n, dtype=int)
    for rank, mine, out, err in res:
        assert err is None, err
        seen[mine] += 1
        for k, (e, vir, f, ea, va) in enumerate(out):
            ref, ref_va = refs[k]
            assert e == ref["energy"], (rank, k)
            assert np.array_equal(vir, ref["virial"]), (rank, k)
            assert np.array_equal(f, ref["forces"][mine]), (rank, k)
            assert np.array_equal(ea, ref["eatom"][mine]), (rank, k)
            assert np.array_equal(va, ref_va[mine]), (rank, k)
    assert (seen == 1).all()


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["optional_operators", "l_size"])
def test_multi_gpu_bit_identical_other_models(kind, tmp_path):
    """2 GPUs give the single-GPU bits for (a) a model with RMSNorm,
    query/key normalisation (also on the halo rows each GPU projects itself),
    residual scalars, NLH repulsion and a C6 ratio head (its ratios
    all-gathered like the Hirshfeld ratios), and (b) the F = 256 width with
    duplicated degrees (the halo rows carry 256 features and 48 equivariant
    channels)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from model_variants import make_l_variant, make_variant
    from so3lr_b200 import So3lrB200
    from so3lr_b200.systems import water_box
    if kind == "l_size":
        path = make_l_variant(MODEL, tmp_path / "l.so3lr", seed=7)
    else:
        path = make_variant(MODEL, tmp_path / "all.so3lr", rms_norm=True, qk_norm=True,
                            residual_scalars=([0.9, 1.1, 0.8], [0.1, -0.2, 0.3]), nlh_capacity=9,
                            hirshfeld_keys=1, c6_keys=1, seed=2, attention_norm_factor=20.0)
    nmol, seed = 1000, 19
    w = water_box(nmol, seed=seed)
    single = So3lrB200(path, 0)
    ref = single.compute(w.pos, w.z, cell=w.cell, boxlo=w.boxlo)
    ref_va = single.virial_atom(len(w.z))
    single.close()
    uid = So3lrB200.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gpu_worker, args=(r, 2, uid, nmol, seed, q, path)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, e, f, vir, chg, owned, va, err in res:
        assert err is None, err
        assert e == ref["energy"], (e, ref["energy"])
        assert np.array_equal(f, ref["forces"]), np.abs(f - ref["forces"]).max()
        assert np.array_equal(vir, ref["virial"])
        assert np.array_equal(chg, ref["charges"])
        assert np.array_equal(va, ref_va)


@pytest.mark.gpu
def test_two_devices_in_one_process():
    """One process, one handle per GPU (how turbo packs are spread over GPUs):
    each device gets its own kernel configuration, and the same pack gives the
    same bits on both."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from so3lr_b200 import So3lrB200
    from so3lr_b200.systems import turbo_batch
    pos, z, off, q, m = turbo_batch(16, seed=31)
    a = So3lrB200(MODEL, 0)
    b = So3lrB200(MODEL, 1)
    ra = a.compute_batch(pos, z, off, q, m)
    rb = b.compute_batch(pos, z, off, q, m)
    assert np.array_equal(ra["forces"], rb["forces"])
    assert np.array_equal(ra["image_energy"], rb["image_energy"])
    a.close()
    b.close()
