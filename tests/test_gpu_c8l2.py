"""GPU parity of the C8L2 profile (the reference's production descriptor)
through the C ABI.

Bars: fp64 mode against the fp64 oracle within 1e-10 relative (energy relative
to |E|, force / virial relative to their largest component); fp32 mode (the
reference's own precision for this profile) against the oracle within 2e-5
relative, and its descriptor against the reference kernels' own fp32 output
(tests/golden/c8l2_*.npz) within 2e-6 of the descriptor scale.
"""
import os

import numpy as np
import pytest

import b200dp
import modelgen
import oracle
import systems
from test_gpu_direct import canonical_graph, run_direct, snapped
from test_oracle import ghost_expand

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FP64_REL = 1e-10
FP32_REL = 2e-5


def rel(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-300))


@pytest.fixture(scope="module")
def c8_path(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("c8gpu") / "c8.b2dp")
    modelgen.save_c8(modelgen.random_c8_model(seed=0), p)
    return p


@pytest.fixture(scope="module")
def ref0(c8_path):
    s = systems.config0()
    return s, oracle.C8Oracle(c8_path).compute(s.coord, s.atype, s.box, extras=True)


@pytest.fixture(scope="module")
def dp64(c8_path):
    dp = b200dp.DeepPot(c8_path, precision=b200dp.FP64)
    yield dp
    dp.close()


@pytest.fixture(scope="module")
def dp32(c8_path):
    dp = b200dp.DeepPot(c8_path, precision=b200dp.MIXED)
    yield dp
    dp.close()


def test_model_info(dp64):
    info = dp64.info
    assert info.descriptor_dim == 70 and info.n_fitting_layers == 3 and info.ntypes == 2
    assert abs(info.rcut - 6.0) < 1e-12


def test_fp64_matches_oracle(dp64, ref0):
    s, ref = ref0
    r = dp64.compute(s.coord, s.atype, s.box, atomic=True)
    assert abs(r["energy"] - ref["energy"]) <= FP64_REL * abs(ref["energy"])
    assert rel(r["force"], ref["force"]) <= FP64_REL
    assert rel(r["virial"], ref["virial"]) <= FP64_REL
    assert rel(r["atom_energy"], ref["atom_energy"]) <= FP64_REL
    assert rel(r["atom_virial"], ref["atom_virial"]) <= FP64_REL
    d, dd = dp64.last_descriptor(s.natoms)
    assert rel(d, ref["descriptor"]) <= FP64_REL
    assert rel(dd, ref["grad_descriptor"]) <= FP64_REL


def test_fp32_matches_oracle(dp32, ref0):
    s, ref = ref0
    r = dp32.compute(s.coord, s.atype, s.box, atomic=True)
    assert abs(r["energy"] - ref["energy"]) <= FP32_REL * abs(ref["energy"])
    assert rel(r["force"], ref["force"]) <= FP32_REL
    assert rel(r["virial"], ref["virial"]) <= FP32_REL
    assert rel(r["atom_virial"], ref["atom_virial"]) <= FP32_REL


@pytest.mark.parametrize("case", ["c8l2_water192", "c8l2_water192_triclinic"])
def test_fp32_matches_reference_kernels(dp32, case):
    """Descriptor and forces against what the reference's own kernels computed."""
    z = np.load(os.path.join(GOLDEN, f"{case}.npz"))
    box = z["box"].reshape(3, 3)
    r = dp32.compute(z["coord"], z["atype"], box)
    d, _ = dp32.last_descriptor(len(z["atype"]))
    assert np.abs(d - z["ref_descriptor"]).max() <= 2e-6 * np.abs(z["ref_descriptor"]).max()
    g = z["ref_edge_grad"].astype(np.float64)
    dst = np.repeat(np.arange(len(z["atype"])), np.diff(z["row_ptr"]))
    f = np.zeros((len(z["atype"]), 3))
    np.add.at(f, dst, g)
    np.subtract.at(f, z["source"].astype(np.int64), g)
    # the engine's backward starts from its own fp32 fitting gradient, the
    # reference's from the oracle's: agreement at fp32 level
    assert rel(r["force"], f) <= FP32_REL


def test_deterministic_bitwise(dp32, ref0):
    s, _ = ref0
    a = dp32.compute(s.coord, s.atype, s.box, atomic=True)
    b = dp32.compute(s.coord, s.atype, s.box, atomic=True)
    for k in ("force", "virial", "atom_energy", "atom_virial"):
        assert np.array_equal(a[k], b[k]), k
    assert a["energy"] == b["energy"]


def test_ghost_mode_equals_periodic(dp64, ref0):
    s, ref = ref0
    coord, atype, own = ghost_expand(s, 6.0)
    n = s.natoms
    r = dp64.compute(coord, atype, None, nghost=len(atype) - n)
    f = r["force"][:n].copy()
    np.add.at(f, own, r["force"][n:])
    assert abs(r["energy"] - ref["energy"]) <= FP64_REL * abs(ref["energy"])
    assert rel(f, ref["force"]) <= 1e-9


@pytest.mark.parametrize("precision,tol", [(b200dp.FP64, 1e-11), (b200dp.MIXED, 2e-5)])
def test_direct_graph_entry(c8_path, precision, tol):
    """The dpa_direct_energy_force-signature entry serves the C8L2 model, the
    reference's own use of that entry."""
    s = systems.config0()
    coord, box = snapped(s)
    graph = canonical_graph(coord, s.atype, box, 6.0, np.random.default_rng(5))
    dp = b200dp.DeepPot(c8_path, precision=precision)
    ref = dp.compute(coord, s.atype, box, atomic=True)
    rc, e, f, v = run_direct(dp, graph, s.natoms)
    dp.check()
    assert rc == 1
    assert rel(f, ref["force"]) < tol
    assert rel(e, ref["atom_energy"]) < tol
    assert rel(v, ref["atom_virial"]) < tol
    b200dp.direct_bind(None)
    dp.close()


def test_fullsize_water_fp32_vs_fp64_and_invariance(c8_path):
    s = systems.config1()  # 12,288 atoms
    d64 = b200dp.DeepPot(c8_path, precision=b200dp.FP64)
    d32 = b200dp.DeepPot(c8_path, precision=b200dp.MIXED)
    a = d64.compute(s.coord, s.atype, s.box)
    b = d32.compute(s.coord, s.atype, s.box)
    assert abs(a["energy"] - b["energy"]) <= FP32_REL * abs(a["energy"])
    assert rel(b["force"], a["force"]) <= FP32_REL
    assert np.abs(a["force"].sum(0)).max() < 1e-8
    t = d64.compute(s.coord + np.array([0.37, -1.1, 2.3]), s.atype, s.box)
    assert abs(t["energy"] - a["energy"]) <= 1e-10 * abs(a["energy"])
    assert rel(t["force"], a["force"]) <= 1e-9
    d64.close()
    d32.close()
