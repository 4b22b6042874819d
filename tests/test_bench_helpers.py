"""Host-side helpers of bench.py: the long-range pair count of the whole-step
roofline against a brute-force minimum-image count, and the FLOP formula."""
import importlib.util

import numpy as np

from conftest import ROOT


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_lr_pair_count_matches_brute_force():
    from so3lr_b200.systems import water_box
    b = _bench()
    w = water_box(300, seed=4)  # 900 atoms, box 20.8 A > 2 x 10 A
    cut = 10.0
    d = w.pos[:, None, :] - w.pos[None, :, :]
    d -= np.round(d / w.cell) * w.cell
    r2 = (d * d).sum(-1)
    brute = int((np.triu(r2 < cut * cut, k=1)).sum())
    assert b.count_lr_pairs(w.pos, w.boxlo, w.cell, cut) == brute


def test_step_flops_formula():
    b = _bench()
    r = b.step_roofline(24000, 946822, 473411, 8651195, 1 / 0.02125, 35.4, 1)
    assert abs(r["reference_flop_per_step"] - (3 * 946822 * 203.6e3 + 3 * 24000 * 288e3 + 24000 * 181e3
                                               + 250 * 8651195)) < 1.0
    assert r["executed_flop_per_step"] < r["reference_flop_per_step"]
    assert abs(r["frac_executed"] - r["executed_tflops"] / 35.4) < 1e-12
    two = b.step_roofline(24000, 946822, 473411, 8651195, 1 / 0.02125, 35.4, 2)
    assert abs(two["executed_tflops"] - 2 * r["executed_tflops"]) < 1e-9


def test_clock_summary_reads_nvidia_smi_rows():
    """The clocks record of the bench line: median SM clock under sampling, the
    maximum, and every throttle reason that was Active in any sample (the
    rejection rule looks for hw_slowdown and the thermal reasons)."""
    b = _bench()
    text = "\n".join([
        "0, 1965, 1965, 650.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1875, 1965, 998.7, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1830, 1965, 1003.2, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "garbage line",
    ])
    c = b.summarize_clocks(text)
    assert c["sm_mhz"] == 1875.0 and c["sm_max_mhz"] == 1965.0 and c["samples"] == 3
    assert c["reasons"] == ["sw_power_cap"]
    hot = b.summarize_clocks("0, 1500, 1965, 900.0, 0x48, Active, Not Active, Active, Not Active")
    assert hot["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]
    assert b.summarize_clocks("")["reasons"] == ["no samples"]


def test_turbo_clusters_dealt_once_and_balanced():
    """Config 5 under N ranks: every cluster on exactly one rank, atom counts
    within one largest cluster of each other."""
    from so3lr_b200.systems import turbo_batch
    b = _bench()
    _, _, off, _, _ = turbo_batch(512, seed=7)
    sizes = np.diff(off)
    for world in (1, 2, 4, 8):
        parts = [b.deal_clusters(sizes, r, world) for r in range(world)]
        allk = np.sort(np.concatenate(parts))
        assert np.array_equal(allk, np.arange(len(sizes)))
        atoms = [int(sizes[p].sum()) for p in parts]
        assert max(atoms) - min(atoms) <= sizes.max(), (world, atoms)


def test_clock_sampler_keeps_only_rows_after_start(tmp_path, monkeypatch):
    """ClockSampler.start returns after nvidia-smi's first row; stop() keeps
    the rows written after that, i.e. those of the timed region (here a
    stand-in nvidia-smi on PATH writes one row every 50 ms, the first with a
    clock of 100 MHz)."""
    fake = tmp_path / "nvidia-smi"
    fake.write_text("#!/bin/sh\n"
                    "echo '0, 100, 1965, 100.0, 0x0, Not Active, Not Active, Not Active, Not Active'\n"
                    "while true; do sleep 0.05; "
                    "echo '0, 1900, 1965, 900.0, 0x4, Not Active, Not Active, Not Active, Active'; done\n")
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}:{__import__('os').environ['PATH']}")
    import time
    b = _bench()
    s = b.ClockSampler(0)
    s.start()
    assert s.skip >= 1
    time.sleep(0.5)
    c = s.stop()
    assert c["samples"] >= 3 and c["sm_mhz"] == 1900.0 and c["reasons"] == ["sw_power_cap"], c


def test_reference_arm_line_keeps_the_contract():
    """`bench.py --impl reference` (the CPU restatement timed on the host) prints
    one JSON line with the keys the driver reads, on the same metric, workload
    and `config` record as the GPU arm (config 1 here, to keep the test short;
    the default config 3 evaluates the same 24,000-atom box as the GPU arm)."""
    import json
    import subprocess
    import sys
    sys.path.insert(0, str(ROOT))
    import bench
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--config", "1"], capture_output=True, text=True, timeout=600,
                         cwd=str(ROOT))
    assert res.returncode == 0, res.stderr
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["metric"] == "atom-steps/s" and d["unit"] == "atom-steps/s"
    assert d["steps"] == 1 and d["warmup"] == 3  # at least 3 warm-up steps, whatever is asked
    assert d["value"] > 0 and d["higher_is_better"] is True and d["dtype"] == "f64"
    assert d["config"]["workload"].startswith("config1")
    assert d["config"] == bench.workload(1, 1)[1]  # the GPU arm's config record
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert cb["sample_atoms"] == 192 and "same 192-atom box" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "atom-steps/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only():
    """Under torchrun the reference arm's rank 0 alone works and prints; the
    other ranks exit 0 at once."""
    import os
    import subprocess
    import sys
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1"],
                         capture_output=True, text=True, timeout=300, cwd=str(ROOT), env=env)
    assert res.returncode == 0 and not [ln for ln in res.stdout.splitlines() if ln.startswith("{")], res.stdout
