"""The benchmark's command-line contract, checked on CPU.

`bench.py --impl reference` (the arm the harness runs beside this build's) prints one
JSON line with the contract's keys and the reference-arm additions, at N = 1 and, under
torch.distributed.run with two CPU ranks, from rank 0 only.  The sweep's tables are
well formed (every configuration of the five, the GPU counts each runs at, a rank grid
for every count).
"""
import json
import os
import socket
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)

KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def json_lines(out: str):
    return [json.loads(x) for x in out.splitlines() if x.startswith("{")]


def check_reference_line(d, n_gpus):
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["n_gpus"] == n_gpus and d["steps"] == 1 and d["warmup"] == 1
    assert d["metric"] == "atom-steps/s (E+F+virial)" and d["unit"] == "atom-steps/s" and d["higher_is_better"]
    assert d["config"]["workload"] == "c1_water_12288" and d["value"] > 0
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


@pytest.mark.slow
def test_reference_arm_one_rank():
    env = dict(os.environ, OMP_NUM_THREADS=str(os.cpu_count() or 1))
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1
    check_reference_line(lines[0], 1)


@pytest.mark.slow
def test_reference_arm_two_ranks_prints_once():
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
                        os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "1",
                        "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1
    check_reference_line(lines[0], 2)


def test_sweep_tables():
    import bench

    table = bench.sweep_table()
    labels = [row[0] for row in table]
    assert len(labels) == len(set(labels))
    for prefix in ("c0_", "c1_", "c2_", "c3_", "c4_"):
        assert any(x.startswith(prefix) for x in labels), prefix
    sizes = {row[0]: row[1]().natoms for row in table if not row[0].endswith(("786k", "3.1M", "786k-slab"))}
    assert sizes["c0_water_192"] == 192 and sizes["c1_water_12288"] == 12288
    assert sizes["c2_cu_131072"] == 131072 and sizes["c3_bcc_524288"] == 524288
    for label, _, kind, precisions, md_cfg, gpus in table:
        assert kind in bench.MASSES and set(precisions) <= {"fp64", "mixed"} and 1 in gpus
        if md_cfg:
            assert md_cfg[0] in ("nvt", "npt") and md_cfg[1] > 0 and md_cfg[2] > 0
        for n in gpus:
            grid = bench.sweep_grid(label, n)
            assert grid[0] * grid[1] * grid[2] == n
            if "slab" in label:
                assert grid[2] == 1  # the vacuum half is never split off
