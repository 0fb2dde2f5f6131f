"""Full-size configurations through size-independent properties.

These checks sit beside the oracle comparisons of test_gpu_fullsize_oracle.py
(configs 2, 3, the 786,432-atom water box and slab against one CPU oracle
evaluation each) and add properties that hold at any size, including the
98,304- and 3,145,728-atom water boxes that have no oracle run:
  * fp64 and mixed precision agree (energy per atom, force RMSE and maximum,
    virial) within the mixed-mode acceptance limits;
  * the total force vanishes (translation invariance) and the virial is
    symmetric (rotation invariance), both to fp64 round-off in fp64 mode;
  * repeated calls are bitwise identical (fixed reduction order);
  * a rigid translation of every atom leaves energy and forces unchanged up to
    round-off of the shifted coordinates.
Config 2 is FCC copper 32^3 cells (131,072 atoms), config 3 the 4-type BCC
alloy 64^3 x 2 (524,288 atoms), config 4 water at 98,304 and 786,432 atoms and
the 786,432-atom slab with 50 % vacuum.  The 3,145,728-atom water box does not
fit the fp64 engine on one GPU; it is held to the mixed-mode properties (total
force, determinism, rigid translation, no sel overflow).
"""
import numpy as np
import pytest

import b200dp
import systems
from conftest import TOLERANCES

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

CASES = [("c2", systems.config2, "cu"), ("c3", systems.config3, "alloy"), ("c4_98k", lambda: systems.config4("98k"), "water"),
         ("c4_786k", lambda: systems.config4("786k"), "water"),
         ("c4_786k_slab", lambda: systems.config4("786k-slab"), "water")]


@pytest.mark.parametrize("name,make,kind", CASES)
def test_full_size_properties(model_dir, name, make, kind):
    s = make()
    path = str(model_dir / f"{kind}.b2dp")
    d64 = b200dp.DeepPot(path, precision=b200dp.FP64)
    dmx = b200dp.DeepPot(path, precision=b200dp.MIXED)
    r64 = d64.compute(s.coord, s.atype, s.box)
    rmx = dmx.compute(s.coord, s.atype, s.box)
    n = s.natoms
    fscale = np.abs(r64["force"]).max()
    # translation / rotation invariance in fp64
    assert np.abs(r64["force"].sum(0)).max() < 1e-9 * fscale * np.sqrt(n)
    w = r64["virial"]
    assert np.abs(w - w.T).max() < 1e-9 * np.abs(w).max()
    # mixed vs fp64
    err = rmx["force"] - r64["force"]
    assert abs(rmx["energy"] - r64["energy"]) / n < TOLERANCES["energy_per_atom"]
    assert np.sqrt((err ** 2).mean()) < TOLERANCES["force_rmse"]
    assert np.abs(err).max() < TOLERANCES["force_max"]
    assert np.abs(err).max() < 2e-4 * fscale
    assert np.abs(rmx["virial"] - w).max() < 2e-4 * np.abs(w).max()
    # determinism
    again = dmx.compute(s.coord, s.atype, s.box)
    assert again["energy"] == rmx["energy"]
    assert np.array_equal(again["force"], rmx["force"])
    # rigid translation
    shifted = d64.compute(s.coord + np.array([0.37, -1.11, 2.03]), s.atype, s.box)
    assert abs(shifted["energy"] - r64["energy"]) < 1e-9 * abs(r64["energy"])
    assert np.abs(shifted["force"] - r64["force"]).max() < 1e-7 * fscale
    for dp in (d64, dmx):
        assert dp.sel_overflow_count() == 0
        dp.close()


def test_3m_water_mixed_properties(model_dir):
    s = systems.config4("3.1M")
    dp = b200dp.DeepPot(str(model_dir / "water.b2dp"), precision=b200dp.MIXED)
    r = dp.compute(s.coord, s.atype, s.box)
    n = s.natoms
    fscale = np.abs(r["force"]).max()
    assert np.isfinite(r["force"]).all() and np.isfinite(r["energy"])
    # every edge's gradient enters its two atoms with opposite signs (fixed-point sums)
    assert np.abs(r["force"].sum(0)).max() < 1e-9 * fscale * np.sqrt(n)
    again = dp.compute(s.coord, s.atype, s.box)
    assert again["energy"] == r["energy"]
    assert np.array_equal(again["force"], r["force"])
    shifted = dp.compute(s.coord + np.array([0.37, -1.11, 2.03]), s.atype, s.box)
    assert abs(shifted["energy"] - r["energy"]) / n < TOLERANCES["energy_per_atom"]
    err = shifted["force"] - r["force"]
    assert np.sqrt((err ** 2).mean()) < TOLERANCES["force_rmse"]
    assert dp.sel_overflow_count() == 0
    dp.close()
