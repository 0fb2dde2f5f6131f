"""Spatial domain decomposition (multi-GPU row) checked on CPU ranks.

Each rank owns the atoms of its sub-box, builds its ghost shell by the staged
x/y/z halo exchange, runs the force call in ghost mode and folds ghost forces
back to their owners.  Energy, virial and every atom's force must equal one
periodic evaluation of the whole box by the CPU oracle; only the summation
order differs, so the bar is 1e-10 relative.  World sizes 2 (slab) and 4
(2x2x1) run as gloo process groups on 127.0.0.1.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import domain
import oracle
import systems

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def reference(model, mol):
    s = systems.water(*mol, seed=3)
    return s, oracle.Oracle(model).compute(s.coord, s.atype, s.box, atomic=False)


def check(s, ref, parts, rel=1e-10):
    f = np.full((s.natoms, 3), np.nan)
    for p in parts:
        f[p["ids"]] = p["force"]
    assert not np.isnan(f).any(), "every atom has exactly one owner"
    assert sum(len(p["ids"]) for p in parts) == s.natoms
    scale = np.abs(ref["force"]).max()
    np.testing.assert_allclose(f, ref["force"], atol=rel * scale, rtol=0)
    for p in parts:
        assert abs(float(p["energy"][0]) - ref["energy"]) <= rel * abs(ref["energy"])
        np.testing.assert_allclose(p["virial"].reshape(3, 3), ref["virial"], atol=rel * np.abs(ref["virial"]).max())


def run_ranks(tmp_path, model, mol, grid, halo, extra=()):
    world = int(np.prod(grid))
    port = free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                   OMP_NUM_THREADS="1")
        cmd = [sys.executable, os.path.join(HERE, "dd_worker.py"), "--model", model, "--mol", *map(str, mol),
               "--grid", *map(str, grid), "--halo", str(halo), "--out", str(tmp_path / f"r{r}.npz"), *extra]
        procs.append(subprocess.Popen(cmd, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        outs.append(out.decode(errors="replace"))
    for p, o in zip(procs, outs):
        assert p.returncode == 0, o[-3000:]
    return [dict(np.load(tmp_path / f"r{r}.npz")) for r in range(world)]


@pytest.mark.parametrize("grid,mol", [((2, 1, 1), (8, 4, 4)), ((2, 2, 1), (8, 8, 4))])
def test_peer_mode_orchestration_on_cpu_ranks(tmp_path, model_dir, grid, mol):
    """The peer mode's step (publish, barrier, gather of ghost positions from the
    owners' buffers with the recorded shifts, force call with ghost rows added
    into the owners' buffers, all-reduce, finish) on gloo ranks with shared
    memory standing in for the GPUs' peer memory: equal to one periodic
    evaluation, over two replayed steps."""
    model = str(model_dir / "water.b2dp")
    s, ref = reference(model, mol)
    parts = run_ranks(tmp_path, model, mol, grid, 6.0, extra=("--fold",))
    check(s, ref, parts)
    check_origins(parts)


def test_single_rank_self_exchange_equals_periodic(model_dir):
    """grid 1x1x1: the ghost shell is the periodic images, made by self-exchange."""
    model = str(model_dir / "water.b2dp")
    mol = (4, 4, 4)
    s, ref = reference(model, mol)
    import torch

    dd = domain.Decomposition(s.box, (1, 1, 1), 0, 6.0)
    x, t, ids = domain.distribute(s.coord, s.atype, dd)
    o = oracle.Oracle(model)

    def compute(x_all, t_all, nloc, nghost, region, e, f, v):
        r = o.compute(x_all.numpy(), t_all.numpy(), None, nloc=nloc, atomic=False)
        e.copy_(torch.tensor([r["energy"]], dtype=torch.float64))
        f.copy_(torch.from_numpy(r["force"]))
        v.copy_(torch.from_numpy(r["virial"].reshape(9)))

    ddp = domain.DistributedDeepPot(compute, s.box, (1, 1, 1), 0, 6.0, x, t, ids)
    e, f, v = ddp.step()
    assert ddp.nghost > 0
    check(s, ref, [dict(ids=ids, force=f.numpy(), energy=e.numpy(), virial=v.numpy())])


def test_decomposition_geometry():
    box = np.diag([40.0, 20.0, 30.0])
    grid = (2, 2, 2)
    owners = np.zeros(1000, int)
    rng = np.random.default_rng(0)
    pts = rng.uniform(-50, 90, size=(1000, 3))
    for r in range(8):
        dd = domain.Decomposition(box, grid, r, 6.0)
        owners += dd.owns(pts)
        assert dd.rank_of(dd.cell) == r
        for dim in range(3):
            assert dd.neighbour(dim, +1) != r and dd.neighbour(dim, -1) != r
    assert (owners == 1).all()
    with pytest.raises(ValueError):
        domain.Decomposition(box, (4, 1, 1), 0, 12.0)  # halo wider than a 10 A sub-box
    with pytest.raises(ValueError):
        domain.Decomposition(np.array([[10, 0, 0], [1, 10, 0], [0, 0, 10.0]]), grid, 0, 3.0)
    w = domain.wrap(np.array([[-1e-17, 40.0, 5.0]]), np.array([40.0, 40.0, 40.0]))
    assert (w >= 0).all() and (w < 40).all()


def check_origins(parts):
    """Every ghost row's recorded origin (owner rank, owner's row) is the atom it
    copies, and the owner's position plus the recorded shift is the ghost's
    position bit for bit (what the peer gather computes)."""
    for p in parts:
        o = p["origin"]
        assert o.shape == (int(p["nghost"]), 2)
        owner_ids = np.array([parts[r]["ids"][k] for r, k in o])
        np.testing.assert_array_equal(owner_ids, p["ghost_ids"])
        xo = np.array([parts[r]["x_owned"][k] for r, k in o])
        np.testing.assert_array_equal(xo + p["shift"], p["x_ghost"])


@pytest.mark.parametrize("grid,mol,halo", [((2, 1, 1), (8, 4, 4), 6.0), ((2, 1, 1), (8, 4, 4), 6.2),
                                           ((2, 2, 1), (8, 8, 4), 6.0)])
def test_gloo_ranks_equal_periodic(tmp_path, model_dir, grid, mol, halo):
    model = str(model_dir / "water.b2dp")
    s, ref = reference(model, mol)
    parts = run_ranks(tmp_path, model, mol, grid, halo)
    assert all(int(p["nghost"]) > 0 for p in parts)
    check(s, ref, parts)
    check_origins(parts)
