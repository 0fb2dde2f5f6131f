"""The C++ decomposed driver (b200dp_dd_*) on GPUs.

One rank on one GPU (NCCL group of one, every ghost a periodic image of an
owned atom): the decomposed force call equals the periodic engine call, and
NVT MD with atom migration and ghost-plan rebuilds every 5 steps follows the
single-GPU MD driver's trajectory.  Two ranks on two GPUs (skipped with
fewer): the same checks with the atoms split over the ranks, each rank in its
own process on its own GPU.  fp64 throughout: force call within 1e-10
relative, trajectories within fp64 round-off of the single-GPU run (the
decomposed sums of kinetic energy and virial run in another order).
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import b200dp
import systems

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
MASS = [15.9994, 15.9994]


def periodic(model, s):
    dp = b200dp.DeepPot(model, precision=b200dp.FP64)
    r = dp.compute(s.coord, s.atype, s.box)
    dp.close()
    return r


def md_setup(s, system, ensemble):
    """Masses, seeded velocities and integrator settings of the comparison runs."""
    rng = np.random.default_rng(3)
    if system == "water":
        masses, temp = [15.9994, 15.9994], 300.0
    else:
        masses, temp = [63.546], 800.0
    m = np.array([masses[t] for t in s.atype])
    v = rng.normal(size=s.coord.shape) * np.sqrt(8.617343e-5 * temp / (m[:, None] * 1.0364269e-4))
    v -= (m[:, None] * v).sum(0) / m.sum()
    kw = dict(dt=0.0005 if system == "water" else 0.001, t_target=temp,
              t_damp=0.025 if system == "water" else 0.1)
    if ensemble == "npt":
        kw.update(ensemble=b200dp.NPT, p_target=1.0, p_damp=0.2)
    else:
        kw.update(ensemble=b200dp.NVT)
    return masses, v, kw


def reference_md(model, s, system, ensemble, nsteps):
    masses, vel, kw = md_setup(s, system, ensemble)
    dp = b200dp.DeepPot(model, precision=b200dp.FP64)
    md = b200dp.MD(dp, s.coord, s.atype, s.box, masses, vel=vel, rebuild_every=0, **kw)
    md.run(nsteps)
    x, v, f = md.state()
    th = md.thermo()
    md.close()
    dp.close()
    return x, v, th


def check_force(ref, parts, natoms):
    e = parts[0]["energy"]
    for p in parts:
        assert p["energy"] == e  # the rendezvous gives every rank the same bits
    assert abs(e - ref["energy"]) <= 1e-10 * abs(ref["energy"])
    assert np.abs(parts[0]["virial"] - ref["virial"]).max() <= 1e-10 * np.abs(ref["virial"]).max()
    f = np.full((natoms, 3), np.nan)
    for p in parts:
        f[p["ids"]] = p["force"]
    assert np.isfinite(f).all()
    assert np.abs(f - ref["force"]).max() <= 1e-10 * np.abs(ref["force"]).max()


def unwrap_to(x, ref, L):
    return x - np.round((x - ref) / L) * L


def check_md(model, s, parts, nsteps, system="water", ensemble="nvt"):
    xr, vr, thr = reference_md(model, s, system, ensemble, nsteps)
    th = dict(zip(b200dp.MD.THERMO, parts[0]["thermo"]))
    L = np.diag(s.box) * np.cbrt(thr["volume"] / np.prod(np.diag(s.box)))
    x = np.full_like(xr, np.nan)
    v = np.full_like(vr, np.nan)
    for p in parts:
        x[p["md_ids"]] = p["md_x"]
        v[p["md_ids"]] = p["md_v"]
    assert np.isfinite(x).all()
    assert np.abs(unwrap_to(x, xr, L) - xr).max() < 1e-8  # migration wraps positions into the box
    assert np.abs(v - vr).max() < 1e-7 * np.abs(vr).max()
    assert th["step"] == nsteps
    assert abs(th["pe"] - thr["pe"]) < 1e-9 * abs(thr["pe"])
    assert abs(th["temp"] - thr["temp"]) < 1e-7 * thr["temp"]
    assert abs(th["conserved"] - thr["conserved"]) < 1e-7 * abs(thr["conserved"])
    assert abs(th["volume"] - thr["volume"]) < 1e-10 * thr["volume"]


def test_one_rank_force_and_md(model_dir):
    model = str(model_dir / "water.b2dp")
    s = systems.water(6)  # 648 atoms, 18.63 A cube
    ref = periodic(model, s)
    dp = b200dp.DeepPot(model, precision=b200dp.FP64)
    dd = b200dp.DD(dp, b200dp.dd_unique_id(), 1, 0, s.coord, s.atype, s.box, (1, 1, 1), halo=8.0)
    assert dd.counts()[0] == s.natoms
    for _ in range(2):
        dd.force()
    e, v = dd.result()
    ids, _, _, f = dd.owned()
    check_force(ref, [dict(energy=e, virial=v, ids=ids, force=f)], s.natoms)
    nsteps = 30
    masses, vel, kw = md_setup(s, "water", "nvt")
    dd.md_start(masses, vel=vel, rebuild_every=5, **kw)
    dd.md_run(nsteps)
    th = dd.thermo()
    ids, x, vv, f = dd.owned()
    check_md(model, s, [dict(md_ids=ids, md_x=x, md_v=vv, thermo=np.array([th[k] for k in dd.THERMO]))], nsteps)
    dd.close()
    dp.close()


def test_one_rank_npt(model_dir):
    """Cu NPT (fix npt iso order, 1 bar, 800 K) over the decomposition against the single-GPU driver:
    the box and the ghost shifts scale with the barostat between plan rebuilds."""
    model = str(model_dir / "cu.b2dp")
    s = systems.fcc(4)  # 256 atoms, 14.46 A cube
    dp = b200dp.DeepPot(model, precision=b200dp.FP64)
    dd = b200dp.DD(dp, b200dp.dd_unique_id(), 1, 0, s.coord, s.atype, s.box, (1, 1, 1), halo=8.0)
    nsteps = 20
    masses, vel, kw = md_setup(s, "cu", "npt")
    dd.md_start(masses, vel=vel, rebuild_every=5, **kw)
    dd.md_run(nsteps)
    th = dd.thermo()
    ids, x, vv, f = dd.owned()
    check_md(model, s, [dict(md_ids=ids, md_x=x, md_v=vv, thermo=np.array([th[k] for k in dd.THERMO]))], nsteps,
             "cu", "npt")
    dd.close()
    dp.close()


def run_two_ranks(tmp_path, model, system, mol, ensemble, nsteps, grid=(2, 1, 1)):
    idfile = str(tmp_path / f"uid_{system}_{ensemble}")
    procs = []
    for r in range(2):
        cmd = [sys.executable, os.path.join(HERE, "dd_cpp_worker.py"), "--rank", str(r), "--nranks", "2", "--grid",
               *map(str, grid), "--model", model, "--mol", *map(str, mol), "--system", system, "--ensemble", ensemble,
               "--idfile", idfile, "--out", str(tmp_path / f"{system}_{ensemble}_r{r}.npz"), "--md-steps",
               str(nsteps), "--rebuild-every", "5"]
        env = dict(os.environ, NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen(cmd, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=300)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        outs.append(out)
    for p, out in zip(procs, outs):
        assert p.returncode == 0, out[-3000:]
    return [dict(np.load(tmp_path / f"{system}_{ensemble}_r{r}.npz")) for r in range(2)]


def test_two_ranks_two_gpus(tmp_path, model_dir):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    model = str(model_dir / "water.b2dp")
    mol = (12, 6, 6)  # 1,296 atoms, 37.26 x 18.63 x 18.63 A, split along x
    s = systems.water(*mol)
    parts = run_two_ranks(tmp_path, model, "water", mol, "nvt", 30)
    check_force(periodic(model, s), parts, s.natoms)
    check_md(model, s, parts, 30)
    # copper NPT on two GPUs (configuration 2's ensemble, on a small box)
    model = str(model_dir / "cu.b2dp")
    s = systems.fcc(6)  # 864 atoms, 21.69 A cube: 10.8 A sub-boxes
    parts = run_two_ranks(tmp_path, model, "cu", (6, 6, 6), "npt", 20)
    check_force(periodic(model, s), parts, s.natoms)
    check_md(model, s, parts, 20, "cu", "npt")
