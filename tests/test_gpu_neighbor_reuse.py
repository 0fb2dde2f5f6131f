"""Neighbour reuse (skin candidates kept between calls) against fresh builds.

Candidates within rcut + skin are built on one call and the rows of the next
calls are formed from them with the new positions; within skin / 2 of the
build positions every call must give the rows, energies and forces of a fresh
build (fp64: rows identical, r_ij and results to 1e-12 relative), including
after an atom crosses the periodic boundary (unwrapped positions, as the MD
driver keeps them).  A larger move triggers a rebuild on the device inside
the same call (counted, same results as a fresh build), and the MD driver's
default (skin 2 A, rebuild every 10 steps) and a skin small enough to trigger
rebuilds both reproduce its every-step trajectory.
"""
import numpy as np
import pytest

import b200dp
import systems

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(np.asarray(b)).max(), 1e-300))


def test_reuse_matches_fresh_builds(model_dir):
    s = systems.config0()
    path = str(model_dir / "water.b2dp")
    fresh = b200dp.DeepPot(path, precision=b200dp.FP64)
    reuse = b200dp.DeepPot(path, precision=b200dp.FP64)
    reuse.set_neighbor_reuse(2.0, 5)
    rng = np.random.default_rng(7)
    x = s.coord.copy()
    # an atom next to the upper x face that crosses it during the sequence
    L = np.diag(s.box)
    k = int(np.argmax(x[:, 0] - np.floor(x[:, 0] / L[0]) * L[0]))
    x[k, 0] = (np.floor(x[k, 0] / L[0]) + 1) * L[0] - 0.05
    for call in range(12):  # rebuilds at calls 0, 5, 10
        d = rng.normal(0.0, 0.05, size=x.shape)
        d[k] = [0.03, 0.0, 0.0]
        x = x + d
        a = fresh.compute(x, s.atype, s.box, atomic=True)
        b = reuse.compute(x, s.atype, s.box, atomic=True)
        reuse.check()
        assert abs(a["energy"] - b["energy"]) <= 1e-12 * abs(a["energy"])
        assert rel(b["force"], a["force"]) <= 1e-12
        assert rel(b["virial"], a["virial"]) <= 1e-12
        assert rel(b["atom_virial"], a["atom_virial"]) <= 1e-12
        na, nb = fresh.last_nlist(s.natoms), reuse.last_nlist(s.natoms)
        np.testing.assert_array_equal(na["nlist"], nb["nlist"])
        assert np.abs(na["rij"] - nb["rij"]).max() <= 1e-12
    assert reuse.neighbor_stats() == {"scheduled": 3, "triggered": 0}
    fresh.close()
    reuse.close()


def test_large_move_triggers_rebuild_on_device(model_dir):
    s = systems.config0()
    dp = b200dp.DeepPot(str(model_dir / "water.b2dp"), precision=b200dp.FP64)
    f = b200dp.DeepPot(str(model_dir / "water.b2dp"), precision=b200dp.FP64)
    dp.set_neighbor_reuse(1.0, 10)
    dp.compute(s.coord, s.atype, s.box)
    x = s.coord.copy()
    for call, move in enumerate([0.8, 0.0, 0.3, 0.3]):  # 0.8 > skin / 2; then 0.6 in total from the rebuild
        x[3] += [move, 0.0, 0.0]
        r = dp.compute(x, s.atype, s.box, atomic=True)
        dp.check()
        ref = f.compute(x, s.atype, s.box, atomic=True)
        assert abs(r["energy"] - ref["energy"]) <= 1e-12 * abs(ref["energy"])
        assert rel(r["force"], ref["force"]) <= 1e-12
        assert rel(r["atom_virial"], ref["atom_virial"]) <= 1e-12
        np.testing.assert_array_equal(dp.last_nlist(s.natoms)["nlist"], f.last_nlist(s.natoms)["nlist"])
    assert dp.neighbor_stats() == {"scheduled": 1, "triggered": 2}  # calls 1 and 4
    dp.close()
    f.close()


@pytest.mark.parametrize("ensemble,skin", [(b200dp.NVT, 2.0), (b200dp.NPT, 2.0), (b200dp.NVT, 0.04)])
def test_md_reuse_matches_every_step_builds(model_dir, ensemble, skin):
    s = systems.config0()
    masses = [15.9994 * 4, 1.00794 * 4]  # heavier atoms: smooth dynamics over the test
    out = []
    for every in (10, 0):
        dp = b200dp.DeepPot(str(model_dir / "water.b2dp"), precision=b200dp.FP64)
        md = b200dp.MD(dp, s.coord, s.atype, s.box, masses, dt=0.0005, ensemble=ensemble, t_init=300.0,
                       t_target=300.0, seed=3, p_target=1.0, rebuild_every=every, skin=skin)
        md.run(40)
        th = md.thermo()
        x, v, _ = md.state()
        dp.check()
        if every and skin < 0.1:  # a 0.02 A half-skin is crossed within 10 steps: rebuilt on the device
            assert dp.neighbor_stats()["triggered"] > 0
        out.append((th, x, v))
        md.close()
        dp.close()
    (ta, xa, va), (tb, xb, vb) = out
    assert np.abs(xa - xb).max() < 1e-9
    assert np.abs(va - vb).max() < 1e-9
    assert abs(ta["conserved"] - tb["conserved"]) <= 1e-9 * abs(tb["conserved"])
