"""GPU parity: the CUDA path through the C ABI against the CPU oracle and the
golden fixtures.

Bars: neighbour list bit-exact (j and image); fp64 mode within 1e-10 relative
(energy relative to |E|, force and virial relative to their largest
component); mixed mode within the acceptance limits of the reference's
data/numeric-tolerances.json (energy/atom 2e-5 eV, force RMSE 4e-5 eV/A, force
max 5e-4 eV/A, stress 4e-4 GPa) and additionally within 2e-4 relative, since the
random-init forces here are small.
"""
import numpy as np
import pytest

import b200dp
import oracle
import systems
from conftest import EV_A3_TO_GPA, GOLDEN_CASES, TOLERANCES, golden, golden_model_path, image_codes

pytestmark = pytest.mark.gpu

FP64_REL = 1e-10
MIXED_REL = 2e-4


def rel(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-300))


def check_fp64(r, ref, nloc):
    assert abs(r["energy"] - ref["energy"]) <= FP64_REL * abs(ref["energy"])
    assert rel(r["force"], ref["force"]) <= FP64_REL
    assert rel(r["virial"], ref["virial"]) <= FP64_REL


def check_mixed(r, ref, natoms, volume):
    de = abs(r["energy"] - ref["energy"]) / natoms
    df = np.asarray(r["force"]) - np.asarray(ref["force"])
    dv = np.abs(np.asarray(r["virial"]) - np.asarray(ref["virial"])).max() / volume * EV_A3_TO_GPA
    assert de <= TOLERANCES["energy_per_atom"], de
    assert np.sqrt(np.mean(df ** 2)) <= TOLERANCES["force_rmse"]
    assert np.abs(df).max() <= TOLERANCES["force_max"]
    assert dv <= TOLERANCES["stress_GPa"]
    assert abs(r["energy"] - ref["energy"]) <= MIXED_REL * abs(ref["energy"])
    assert rel(r["force"], ref["force"]) <= MIXED_REL
    assert rel(r["virial"], ref["virial"]) <= MIXED_REL


@pytest.fixture(scope="module")
def engines(model_dir):
    cache = {}

    def get(path, precision):
        key = (path, precision)
        if key not in cache:
            cache[key] = b200dp.DeepPot(path, precision=precision)
        return cache[key]

    yield get
    for e in cache.values():
        e.close()


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_fp64_matches_golden(engines, model_dir, name):
    g, meta = golden(name)
    dp = engines(golden_model_path(model_dir, meta), b200dp.FP64)
    r = dp.compute(g["coord"], g["atype"], g["box"], atomic=True)
    ref = dict(energy=float(g["energy"]), force=g["force"], virial=g["virial"])
    check_fp64(r, ref, len(g["atype"]))
    assert rel(r["atom_energy"], g["atom_energy"]) <= FP64_REL
    assert rel(r["atom_virial"], g["atom_virial"]) <= FP64_REL
    nl = dp.last_nlist(len(g["atype"]))
    np.testing.assert_array_equal(nl["nlist"], g["nlist"])
    valid = g["nlist"] >= 0
    np.testing.assert_array_equal(nl["code"][valid], image_codes(g["image"])[valid])


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_mixed_matches_golden(engines, model_dir, name):
    g, meta = golden(name)
    dp = engines(golden_model_path(model_dir, meta), b200dp.MIXED)
    r = dp.compute(g["coord"], g["atype"], g["box"])
    ref = dict(energy=float(g["energy"]), force=g["force"], virial=g["virial"])
    check_mixed(r, ref, len(g["atype"]), abs(np.linalg.det(g["box"])))


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_nlist_bit_exact_vs_oracle(engines, model_dir, name):
    g, meta = golden(name)
    path = golden_model_path(model_dir, meta)
    dp = engines(path, b200dp.FP64)
    dp.compute(g["coord"], g["atype"], g["box"])
    got = dp.last_nlist(len(g["atype"]))
    import modelgen

    m = modelgen.load(path)
    ref = oracle.nlist(g["coord"], g["atype"], g["box"], m.rcut, m.sel)
    np.testing.assert_array_equal(got["nlist"], ref["nlist"])
    np.testing.assert_array_equal(got["code"], ref["code"])
    # rij is recomputed from identical fp64 operations: bit-exact too
    np.testing.assert_array_equal(got["rij"], ref["rij"])


def test_descriptor_stage_matches_oracle(engines, model_dir):
    s = systems.config0()
    path = str(model_dir / "water.b2dp")
    dp = engines(path, b200dp.FP64)
    dp.compute(s.coord, s.atype, s.box)
    d, dd = dp.last_descriptor(s.natoms)
    ref = oracle.Oracle(path).compute(s.coord, s.atype, s.box, descriptor_dim=d.shape[1])
    assert rel(d, ref["descriptor"]) < 1e-12
    assert rel(dd, ref["grad_descriptor"]) < 1e-11


@pytest.mark.parametrize("precision", [b200dp.FP64, b200dp.MIXED])
def test_config1_full_size_vs_oracle(engines, model_dir, precision):
    s = systems.config1()
    path = str(model_dir / "water.b2dp")
    dp = engines(path, precision)
    r = dp.compute(s.coord, s.atype, s.box)
    ref = oracle.Oracle(path).compute(s.coord, s.atype, s.box)
    if precision == b200dp.FP64:
        check_fp64(r, ref, s.natoms)
    else:
        check_mixed(r, ref, s.natoms, abs(np.linalg.det(s.box)))


@pytest.mark.parametrize("precision", [b200dp.FP64, b200dp.MIXED])
def test_deterministic_bitwise(engines, model_dir, precision):
    s = systems.config1()
    dp = engines(str(model_dir / "water.b2dp"), precision)
    a = dp.compute(s.coord, s.atype, s.box, atomic=True)
    b = dp.compute(s.coord, s.atype, s.box, atomic=True)
    assert a["energy"] == b["energy"]
    for k in ("force", "virial", "atom_energy", "atom_virial"):
        np.testing.assert_array_equal(a[k], b[k])


def test_ghost_mode_matches_periodic(engines, model_dir):
    from test_oracle import ghost_expand

    s = systems.config0()
    dp = engines(str(model_dir / "water.b2dp"), b200dp.FP64)
    base = dp.compute(s.coord, s.atype, s.box)
    coord, atype, own = ghost_expand(s, 6.0)
    n = s.natoms
    gm = dp.compute(coord, atype, None, nghost=len(atype) - n)
    assert abs(gm["energy"] - base["energy"]) <= 1e-11 * abs(base["energy"])
    f = gm["force"][:n].copy()
    np.add.at(f, own, gm["force"][n:])
    assert rel(f, base["force"]) < 1e-10
    assert rel(gm["virial"], base["virial"]) < 1e-10
    ref = oracle.Oracle(str(model_dir / "water.b2dp")).compute(coord, atype, None, nloc=n)
    assert rel(gm["force"], ref["force"]) < 1e-10


def test_caller_neighbour_list(engines, model_dir):
    """LAMMPS-style full list with skin candidates gives the same result."""
    from test_oracle import ghost_expand

    s = systems.config0()
    coord, atype, own = ghost_expand(s, 8.0)
    n = s.natoms
    dp = engines(str(model_dir / "water.b2dp"), b200dp.FP64)
    auto = dp.compute(coord, atype, None, nghost=len(atype) - n)
    d2 = ((coord[:n, None, :] - coord[None, :, :]) ** 2).sum(-1)
    lists = [np.nonzero((d2[i] < 8.0 ** 2) & (np.arange(len(coord)) != i))[0][::-1] for i in range(n)]
    given = dp.compute(coord, atype, None, nghost=len(atype) - n, nlist=lists)
    assert abs(given["energy"] - auto["energy"]) <= 1e-12 * abs(auto["energy"])
    assert rel(given["force"], auto["force"]) < 1e-12


def test_sel_overflow_truncates_like_oracle(model_dir):
    s = systems.config0()
    path = str(model_dir / "water_smallsel.b2dp")
    dp = b200dp.DeepPot(path, precision=b200dp.FP64)
    r = dp.compute(s.coord, s.atype, s.box)
    ref = oracle.Oracle(path).compute(s.coord, s.atype, s.box)
    assert dp.sel_overflow_count() == ref["overflow"] > 0
    check_fp64(r, ref, s.natoms)
    dp.close()
    strict = b200dp.DeepPot(path, precision=b200dp.FP64, sel_overflow_is_error=True)
    with pytest.raises(b200dp.B200DPError) as e:
        strict.compute(s.coord, s.atype, s.box)
    assert e.value.status == 4
    strict.close()


def test_bad_type_reported(engines, model_dir):
    s = systems.config0()
    dp = engines(str(model_dir / "water.b2dp"), b200dp.FP64)
    at = s.atype.copy()
    at[5] = 7
    with pytest.raises(b200dp.B200DPError) as e:
        dp.compute(s.coord, at, s.box)
    assert e.value.status == 6
    # the engine stays usable
    r = dp.compute(s.coord, s.atype, s.box)
    assert np.isfinite(r["energy"])


def test_empty_system(engines, model_dir):
    dp = engines(str(model_dir / "water.b2dp"), b200dp.FP64)
    r = dp.compute(np.zeros((0, 3)), np.zeros(0, np.int32), np.eye(3) * 10)
    assert r["energy"] == 0.0 and r["force"].shape == (0, 3)


def test_isolated_atoms(engines, model_dir):
    dp = engines(str(model_dir / "water.b2dp"), b200dp.FP64)
    coord = np.array([[0.0, 0, 0], [50.0, 0, 0]])
    at = np.array([0, 1], np.int32)
    r = dp.compute(coord, at, None)
    ref = oracle.Oracle(str(model_dir / "water.b2dp")).compute(coord, at, None)
    assert np.all(r["force"] == 0)
    assert abs(r["energy"] - ref["energy"]) <= 1e-12 * abs(ref["energy"])


def test_device_entry_on_torch_stream(engines, model_dir):
    torch = pytest.importorskip("torch")
    s = systems.config1()
    dp = engines(str(model_dir / "water.b2dp"), b200dp.MIXED)
    host = dp.compute(s.coord, s.atype, s.box)
    dev = torch.device("cuda:0")
    x = torch.tensor(s.coord, device=dev)
    t = torch.tensor(s.atype, device=dev)
    e = torch.zeros(1, dtype=torch.float64, device=dev)
    f = torch.zeros(s.natoms, 3, dtype=torch.float64, device=dev)
    v = torch.zeros(9, dtype=torch.float64, device=dev)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        dp.compute_device(st.cuda_stream, s.natoms, 0, x.data_ptr(), t.data_ptr(), s.box, None, e.data_ptr(),
                          f.data_ptr(), v.data_ptr())
    st.synchronize()
    dp.check()
    assert float(e.item()) == host["energy"]
    np.testing.assert_array_equal(f.cpu().numpy(), host["force"])


@pytest.mark.parametrize("name", ["water192", "cu108", "alloy128", "water192_two_side"])
def test_tensor_core_descriptor_matches_simt(model_dir, name):
    """The tcgen05 embedding path and the SIMT fp32 path give the same descriptor."""
    g, meta = golden(name)
    path = golden_model_path(model_dir, meta)
    tc = b200dp.DeepPot(path, precision=b200dp.MIXED, keep_descriptor=True)
    simt = b200dp.DeepPot(path, precision=b200dp.MIXED, simt_only=True)
    n = len(g["atype"])
    rt = tc.compute(g["coord"], g["atype"], g["box"])
    rs = simt.compute(g["coord"], g["atype"], g["box"])
    d_tc, dd_tc = tc.last_descriptor(n)
    d_s, dd_s = simt.last_descriptor(n)
    assert rel(d_tc, d_s) < 2e-5
    assert rel(dd_tc, dd_s) < 2e-4
    assert abs(rt["energy"] - rs["energy"]) <= 2e-5 * abs(rs["energy"])
    assert rel(rt["force"], rs["force"]) < 2e-4
    tc.close()
    simt.close()


def test_descriptor_not_kept_is_an_error(model_dir):
    """The tensor-core mixed path never materialises D and dE/dD unless asked to."""
    s = systems.config0()
    dp = b200dp.DeepPot(str(model_dir / "water.b2dp"), precision=b200dp.MIXED)
    dp.compute(s.coord, s.atype, s.box)
    with pytest.raises(b200dp.B200DPError):
        dp.last_descriptor(s.natoms)
    dp.close()
