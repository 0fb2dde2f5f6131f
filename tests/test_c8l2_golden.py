"""The C8L2 oracle against outputs of the reference's own descriptor kernels.

The fixtures (tests/golden/c8l2_*.npz, made by make_c8l2_golden.py) hold what
the reference's forward, node-readout VJP and edge recomputation computed on a
B200 for seeded systems and a seeded model; the oracle here recomputes the same
quantities in fp64 on the same fp32 edge vectors.  Tolerances are those of the
reference's fp32 arithmetic."""
import hashlib
import os

import numpy as np
import pytest

import modelgen
import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ["c8l2_water192", "c8l2_water192_triclinic"]


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("c8g") / "c8.b2dp")
    modelgen.save_c8(modelgen.random_c8_model(seed=0), p)
    return p


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_kernels(model, case):
    z = np.load(os.path.join(GOLDEN, f"{case}.npz"))
    assert int(z["model_seed"]) == 0
    assert hashlib.sha256(open(model, "rb").read()).hexdigest() == str(z["model_sha256"])
    o = oracle.C8Oracle(model)
    nl = oracle.nlist(z["coord"], z["atype"], z["box"], o.rcut, o.sel)
    keep = nl["nlist"] >= 0
    # same canonical graph as the reference ran on
    assert np.array_equal(nl["nlist"][keep].astype(np.uint32), z["source"])
    assert np.array_equal(np.concatenate([[0], np.cumsum(keep.sum(1))]), z["row_ptr"])
    assert np.array_equal(nl["rij"][keep].astype(np.float32), z["edge_vec"])
    nl["rij"] = np.where(keep[..., None], nl["rij"].astype(np.float32).astype(np.float64), 0.0)
    r = o.compute(z["coord"], z["atype"], z["box"], extras=True, nl=nl)

    def close(a, b, rtol):
        scale = np.abs(b).max()
        return np.abs(a - b).max() <= rtol * scale

    assert close(r["descriptor"], z["ref_descriptor"], 1e-6)
    assert close(r["state"], z["ref_state"], 1e-6)
    assert close(r["grad_descriptor"], z["grad_descriptor"], 1e-6)
    assert close(r["q"], z["ref_q"], 1e-5)
    assert close(r["edge_grad"][keep], z["ref_edge_grad"], 1e-5)
    # forces assembled from the reference's edge gradients (F[dst] += g, F[src] -= g)
    g = z["ref_edge_grad"].astype(np.float64)
    dst = np.repeat(np.arange(len(z["atype"])), np.diff(z["row_ptr"]))
    f = np.zeros((len(z["atype"]), 3))
    np.add.at(f, dst, g)
    np.subtract.at(f, z["source"].astype(np.int64), g)
    assert close(r["force"], f, 1e-5)
