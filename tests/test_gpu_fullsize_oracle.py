"""Full-size configurations 2-4 against the CPU oracle.

The bars are the same as for the small systems (test_gpu_parity.py), applied
at the configurations' own sizes:
  * the neighbour list is bit-exact: for every centre and slot the neighbour
    index, the periodic image code and the fp64 edge vector r_ij equal the
    oracle's (oracle_nlist, the same (r^2, j, image) ordering rule);
  * fp64 mode: energy, every force component and the virial within 1e-10
    relative of one fp64 oracle evaluation (energy relative to |E|, force and
    virial relative to their largest component);
  * mixed mode: within the acceptance limits of the reference's
    data/numeric-tolerances.json:3-9 (energy/atom 2e-5 eV, force RMSE
    4e-5 eV/A, force max 5e-4 eV/A, stress 4e-4 GPa) of that same oracle
    result, plus 2e-4 relative.
Config 2 is FCC copper 32^3 cells (131,072 atoms), config 3 the 4-type BCC
alloy (524,288 atoms), config 4 the 786,432-atom water box and the
786,432-atom slab with 50 % vacuum.  One oracle evaluation takes 15-90 s on
16 host cores; the oracle runs with every host thread.
"""
import numpy as np
import pytest

import b200dp
import oracle
import systems
from test_gpu_parity import check_fp64, check_mixed

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

CASES = [("c2", systems.config2, "cu"), ("c3", systems.config3, "alloy"),
         ("c4_786k", lambda: systems.config4("786k"), "water"),
         ("c4_786k_slab", lambda: systems.config4("786k-slab"), "water")]


@pytest.mark.parametrize("name,make,kind", CASES)
def test_full_size_matches_oracle(model_dir, name, make, kind):
    import modelgen

    s = make()
    path = str(model_dir / f"{kind}.b2dp")
    m = modelgen.load(path)
    n = s.natoms
    volume = abs(np.linalg.det(s.box))

    d64 = b200dp.DeepPot(path, precision=b200dp.FP64)
    r64 = d64.compute(s.coord, s.atype, s.box)
    got = d64.last_nlist(n)
    assert d64.sel_overflow_count() == 0
    d64.close()

    # (a) neighbour list, image codes and edge vectors bit for bit
    ref_nl = oracle.nlist(s.coord, s.atype, s.box, m.rcut, m.sel)
    assert ref_nl["overflow"] == 0
    np.testing.assert_array_equal(got["nlist"], ref_nl["nlist"])
    np.testing.assert_array_equal(got["code"], ref_nl["code"])
    np.testing.assert_array_equal(got["rij"], ref_nl["rij"])
    del got, ref_nl

    # (b) fp64 mode against one fp64 oracle evaluation
    ref = oracle.Oracle(path).compute(s.coord, s.atype, s.box, atomic=False)
    check_fp64(r64, ref, n)

    # (c) mixed mode against the same oracle result
    dmx = b200dp.DeepPot(path, precision=b200dp.MIXED)
    rmx = dmx.compute(s.coord, s.atype, s.box)
    assert dmx.sel_overflow_count() == 0
    dmx.close()
    check_mixed(rmx, ref, n, volume)
