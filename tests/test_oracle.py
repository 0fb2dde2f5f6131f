"""CPU oracle checks: golden fixtures, finite differences, symmetries, ghost mode.

The oracle (oracle/sea_oracle.cpp) is the checker for the CUDA path.  Its
parity with the reference is unpinned (the reference holds no implementation of
this model family); these tests pin it to an independent autograd restatement
(tests/golden/torch_sea.py, committed fixtures) and to physics identities.
"""
import hashlib
import os
import tempfile

import numpy as np
import pytest

import modelgen
import oracle
import systems
from conftest import GOLDEN_CASES, golden, golden_model_path, image_codes


def rel(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-300))


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_oracle_matches_golden(model_dir, name):
    g, meta = golden(name)
    path = golden_model_path(model_dir, meta)
    with open(path, "rb") as f:
        assert hashlib.sha256(f.read()).hexdigest() == meta["model_sha256"], "model generator drifted"
    o = oracle.Oracle(path)
    r = o.compute(g["coord"], g["atype"], g["box"])
    assert abs(r["energy"] - float(g["energy"])) <= 1e-12 * abs(float(g["energy"]))
    assert rel(r["force"], g["force"]) < 1e-10
    assert rel(r["virial"], g["virial"]) < 1e-10
    assert rel(r["atom_energy"], g["atom_energy"]) < 1e-11
    assert rel(r["atom_virial"], g["atom_virial"]) < 1e-10
    m = modelgen.load(path)
    nl = oracle.nlist(g["coord"], g["atype"], g["box"], m.rcut, m.sel)
    np.testing.assert_array_equal(nl["nlist"], g["nlist"])
    valid = g["nlist"] >= 0
    np.testing.assert_array_equal(nl["code"][valid], image_codes(g["image"])[valid])


def test_finite_difference_forces(model_dir):
    s = systems.config0()
    o = oracle.Oracle(str(model_dir / "water.b2dp"))
    r = o.compute(s.coord, s.atype, s.box)
    h = 1e-5
    for a, c in [(0, 0), (7, 1), (100, 2), (191, 0)]:
        cp = s.coord.copy()
        cp[a, c] += h
        cm = s.coord.copy()
        cm[a, c] -= h
        fd = -(o.compute(cp, s.atype, s.box)["energy"] - o.compute(cm, s.atype, s.box)["energy"]) / (2 * h)
        assert abs(fd - r["force"][a, c]) < 1e-8 + 1e-5 * abs(fd)


def test_virial_is_strain_derivative(model_dir):
    s = systems.config0()
    o = oracle.Oracle(str(model_dir / "water.b2dp"))
    r = o.compute(s.coord, s.atype, s.box)
    eps = 1e-6
    for a, b in [(0, 0), (0, 1), (2, 1)]:
        def e_of(x):
            M = np.eye(3)
            M[a, b] += x
            return o.compute(s.coord @ M, s.atype, s.box @ M)["energy"]

        fd = -(e_of(eps) - e_of(-eps)) / (2 * eps)
        assert abs(fd - r["virial"][a, b]) < 1e-7 + 1e-5 * abs(fd)
    np.testing.assert_allclose(r["virial"], r["virial"].T, atol=1e-12)
    np.testing.assert_allclose(r["atom_virial"].sum(0).reshape(3, 3), r["virial"], atol=1e-11)


def test_translation_rotation_permutation(model_dir):
    s = systems.config0()
    o = oracle.Oracle(str(model_dir / "water.b2dp"))
    base = o.compute(s.coord, s.atype, s.box)
    # translation (including a wrap across the cell)
    t = o.compute(s.coord + np.array([3.3, -7.1, 20.0]), s.atype, s.box)
    assert abs(t["energy"] - base["energy"]) < 1e-11
    np.testing.assert_allclose(t["force"], base["force"], atol=1e-12)
    # rigid rotation of atoms and cell
    rng = np.random.default_rng(5)
    q, _ = np.linalg.qr(rng.normal(size=(3, 3)))
    if np.linalg.det(q) < 0:
        q[:, 0] = -q[:, 0]
    rr = o.compute(s.coord @ q.T, s.atype, s.box @ q.T)
    assert abs(rr["energy"] - base["energy"]) < 1e-11
    np.testing.assert_allclose(rr["force"], base["force"] @ q.T, atol=1e-12)
    np.testing.assert_allclose(rr["virial"], q @ base["virial"] @ q.T, atol=1e-11)
    # permutation
    perm = rng.permutation(s.natoms)
    p = o.compute(s.coord[perm], s.atype[perm], s.box)
    assert abs(p["energy"] - base["energy"]) < 1e-11
    np.testing.assert_allclose(p["force"], base["force"][perm], atol=1e-12)


def ghost_expand(s, rc):
    """Explicit ghost images of a periodic system (orthorhombic), LAMMPS style."""
    L = np.diag(s.box)
    xw = s.coord - np.floor(s.coord / L) * L
    ghosts, owners = [], []
    reach = [int(np.ceil(rc / l)) for l in L]
    for a in range(-reach[0], reach[0] + 1):
        for b in range(-reach[1], reach[1] + 1):
            for c in range(-reach[2], reach[2] + 1):
                if a == b == c == 0:
                    continue
                sh = np.array([a, b, c]) * L
                y = xw + sh
                inside = np.all((y > -rc) & (y < L + rc), axis=1)
                ghosts.append(y[inside])
                owners.append(np.nonzero(inside)[0])
    g = np.concatenate(ghosts)
    own = np.concatenate(owners)
    return np.concatenate([xw, g]), np.concatenate([s.atype, s.atype[own]]), own


def test_ghost_mode_equals_periodic(model_dir):
    s = systems.config0()
    o = oracle.Oracle(str(model_dir / "water.b2dp"))
    base = o.compute(s.coord, s.atype, s.box)
    coord, atype, own = ghost_expand(s, 6.0)
    n = s.natoms
    gm = o.compute(coord, atype, None, nloc=n)
    assert abs(gm["energy"] - base["energy"]) < 1e-11
    f = gm["force"][:n].copy()
    np.add.at(f, own, gm["force"][n:])
    np.testing.assert_allclose(f, base["force"], atol=1e-12)
    np.testing.assert_allclose(gm["virial"], base["virial"], atol=1e-11)


def test_sel_truncation_keeps_nearest(model_dir):
    s = systems.config0()
    m = modelgen.load(str(model_dir / "water_smallsel.b2dp"))
    full = oracle.nlist(s.coord, s.atype, s.box, 6.0, [46, 92])
    small = oracle.nlist(s.coord, s.atype, s.box, 6.0, m.sel)
    assert small["overflow"] > 0
    np.testing.assert_array_equal(small["nlist"][:, :12], full["nlist"][:, :12])
    np.testing.assert_array_equal(small["nlist"][:, 12:36], full["nlist"][:, 46:70])


def test_empty_and_isolated():
    m = modelgen.random_model("water", seed=0)
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "m.b2dp")
        modelgen.save(m, p)
        o = oracle.Oracle(p)
        # two atoms far apart: no neighbours, energy = sum of fitting(0)
        coord = np.array([[0.0, 0, 0], [50.0, 0, 0]])
        r = o.compute(coord, np.array([0, 1], np.int32), None)
        assert np.all(r["force"] == 0)
        assert np.isfinite(r["energy"])


def test_model_file_roundtrip(tmp_path):
    m = modelgen.random_model("alloy", seed=3)
    p = str(tmp_path / "a.b2dp")
    modelgen.save(m, p)
    m2 = modelgen.load(p)
    assert m2.sel == m.sel and m2.emb == m.emb and m2.fit == m.fit
    for n1, n2 in zip(m.emb_nets + m.fit_nets, m2.emb_nets + m2.fit_nets):
        for (w1, b1), (w2, b2) in zip(n1, n2):
            np.testing.assert_array_equal(w1, w2)
            np.testing.assert_array_equal(b1, b2)


def test_system_generators():
    s0 = systems.config0()
    assert s0.natoms == 192 and abs(s0.box[0, 0] - 12.42) < 1e-12
    oh = np.linalg.norm(s0.coord[1] - s0.coord[0])
    assert abs(oh - 0.96) < 1e-12
    v1 = s0.coord[1] - s0.coord[0]
    v2 = s0.coord[2] - s0.coord[0]
    ang = np.degrees(np.arccos(v1 @ v2 / np.linalg.norm(v1) / np.linalg.norm(v2)))
    assert abs(ang - 104.5) < 1e-9
    assert systems.fcc(2).natoms == 32
    b = systems.bcc_alloy(3)
    assert b.natoms == 54 and set(np.unique(b.atype)) <= {0, 1, 2, 3}
