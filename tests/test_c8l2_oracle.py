"""CPU checks of the C8L2 oracle (the fp64 restatement of the reference's
descriptor, fitting and force path): finite-difference forces, virial against
the strain derivative, invariances, and the model file round trip."""
import os

import numpy as np
import pytest

import modelgen
import systems
import oracle


@pytest.fixture(scope="module")
def c8_path(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("c8") / "c8.b2dp")
    modelgen.save_c8(modelgen.random_c8_model(seed=0), p)
    return p


@pytest.fixture(scope="module")
def c8(c8_path):
    return oracle.C8Oracle(c8_path)


def test_model_roundtrip(c8_path):
    m = modelgen.load_c8(c8_path)
    m2 = modelgen.random_c8_model(seed=0)
    assert np.array_equal(m.table, m2.table) and np.array_equal(m.readout, m2.readout)
    assert m.fit == [96, 96, 96] and m.resnets == [0, 1, 1] and m.activation == 1
    # readout matrices are stored with their transposes (the backward reads those)
    for k in (0, 2, 4, 6):
        assert np.array_equal(m.readout[k + 1], m.readout[k].T)


def test_table_is_c2_continuous():
    m = modelgen.random_c8_model(seed=1)
    w, h = m.channels, m.table_stride
    q = m.table[:, : 4 * w].reshape(-1, w, 4)
    pr = m.table[:, 4 * w:].reshape(-1, w, 2)
    c = np.concatenate([q, pr], -1)
    for d in range(3):  # value, first and second derivative at the shared knots
        k = np.arange(d, 6)
        fac = np.array([np.prod(np.arange(kk - d + 1, kk + 1)) for kk in k], dtype=float)
        end = (c[:-1, :, d:] * fac * h ** (k - d)).sum(-1)
        start = c[1:, :, d] * np.prod(np.arange(1, d + 1))
        assert np.abs(end - start).max() < 1e-9 * max(1.0, np.abs(start).max())


def test_forces_match_finite_differences(c8):
    s = systems.config0()
    r = c8.compute(s.coord, s.atype, s.box)
    assert r["overflow"] == 0
    h = 1e-5
    rng = np.random.default_rng(0)
    for i in rng.choice(s.natoms, 6, replace=False):
        for c in range(3):
            x = s.coord.copy()
            x[i, c] += h
            ep = c8.compute(x, s.atype, s.box)["energy"]
            x[i, c] -= 2 * h
            em = c8.compute(x, s.atype, s.box)["energy"]
            assert abs(-(ep - em) / (2 * h) - r["force"][i, c]) < 1e-6


def test_virial_matches_strain_derivative(c8):
    s = systems.config0()
    r = c8.compute(s.coord, s.atype, s.box)
    box = s.box.reshape(3, 3)
    h = 1e-6
    for a in range(3):
        for b in range(3):
            def energy(eps):
                F = np.eye(3)
                F[a, b] += eps
                return c8.compute(s.coord @ F.T, s.atype, (box @ F.T).reshape(9))["energy"]

            dE = (energy(h) - energy(-h)) / (2 * h)
            assert abs(-dE - r["virial"][a, b]) < 1e-5 * max(1.0, np.abs(r["virial"]).max())


def test_invariances_and_sums(c8):
    s = systems.config0()
    r = c8.compute(s.coord, s.atype, s.box)
    assert abs(r["atom_energy"].sum() - r["energy"]) < 1e-9 * abs(r["energy"])
    assert np.abs(r["force"].sum(0)).max() < 1e-9
    assert np.allclose(r["atom_virial"].sum(0).reshape(3, 3), r["virial"], atol=1e-9)
    # translation
    t = c8.compute(s.coord + np.array([1.3, -0.7, 2.1]), s.atype, s.box)
    assert abs(t["energy"] - r["energy"]) < 1e-9 * abs(r["energy"])
    # rotation of coordinates and cell together
    th = 0.7
    Rz = np.array([[np.cos(th), -np.sin(th), 0], [np.sin(th), np.cos(th), 0], [0, 0, 1.0]])
    Rx = np.array([[1.0, 0, 0], [0, np.cos(0.4), -np.sin(0.4)], [0, np.sin(0.4), np.cos(0.4)]])
    R = Rx @ Rz
    rr = c8.compute(s.coord @ R.T, s.atype, (s.box.reshape(3, 3) @ R.T).reshape(9))
    assert abs(rr["energy"] - r["energy"]) < 1e-9 * abs(r["energy"])
    # The direction is regularized (|u|^2 = r^2 / (r^2 + eps^2)) while the
    # degree-two harmonics substitute |u|^2 = 1, so covariance holds to a
    # relative ~eps^2 / r^2 (1e-7 at eps = 1e-3), as in the reference.
    assert np.abs(rr["force"] - r["force"] @ R.T).max() < 1e-6
    # permutation of atoms
    perm = np.random.default_rng(1).permutation(s.natoms)
    pp = c8.compute(s.coord[perm], s.atype[perm], s.box)
    assert abs(pp["energy"] - r["energy"]) < 1e-9 * abs(r["energy"])
    assert np.abs(pp["force"] - r["force"][perm]).max() < 1e-9


def test_descriptor_block_structure(c8):
    """Degree-zero block is the normalized scalar moments, the divisors are
    sqrt(mass + floor), the last block the type embedding (all after the
    output normalization)."""
    m = modelgen.random_c8_model(seed=0)
    s = systems.config0()
    r = c8.compute(s.coord, s.atype, s.box, extras=True)
    d = r["descriptor"] / m.output_inv_std + m.output_mean
    assert np.allclose(d[:, :8], r["state"][:, :8], atol=1e-12)
    assert np.allclose(d[:, 62:70], m.type_embedding[s.atype], atol=1e-12)
    assert np.allclose(d[:, 60] * r["state"][:, 40], 1.0, atol=1e-12)
    assert np.allclose(d[:, 61] * r["state"][:, 41], 1.0, atol=1e-12)
