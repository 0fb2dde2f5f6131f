"""The neighbour-list entry point that allocates no device memory.

b200dp_build_nlist_noalloc is for callers that cannot call cudaMalloc while
they run: an MD engine whose memory pool already owns the GPU, or a step loop
that cannot afford the device synchronisation cudaMalloc/cudaFree may cause.
Its scratch lives in a static device array inside the library.  These tests
call it through the C ABI twice in a row and check that it returns exactly the
list of the regular entry point (b200dp_compute_host, read back with
b200dp_last_nlist): neighbour indices, image codes and r_ij bit for bit, the
same bar as every other neighbour-list test.  The file is named so that pytest
collects it last.
"""
import ctypes

import numpy as np
import pytest

import b200dp
import modelgen
import systems
from conftest import golden, golden_model_path

pytestmark = pytest.mark.gpu


def call_noalloc(coord, atype, box, m, nghost=0, region=None, out=None):
    """One call through the C ABI; returns (status, dropped candidates, outputs).

    `out` reuses output buffers of an earlier call (so that a call allocates
    nothing on the torch side either)."""
    torch = pytest.importorskip("torch")
    dev = torch.device("cuda:0")
    L = b200dp.load_library()
    n = len(atype)
    nloc = n - nghost
    selt = int(sum(m.sel))
    if out is None:
        x = torch.tensor(np.ascontiguousarray(coord, dtype=np.float64), device=dev)
        t = torch.tensor(np.ascontiguousarray(atype, dtype=np.int32), device=dev)
        nl = torch.full((nloc, selt), -7, dtype=torch.int32, device=dev)
        img = torch.zeros((nloc, selt), dtype=torch.int32, device=dev)
        rij = torch.zeros((nloc, selt, 3), dtype=torch.float64, device=dev)
        out = (x, t, nl, img, rij)
    x, t, nl, img, rij = out
    sel = (ctypes.c_int * len(m.sel))(*m.sel)
    dp_ = ctypes.POINTER(ctypes.c_double)
    b = None if box is None else np.ascontiguousarray(np.asarray(box, dtype=np.float64).reshape(9))
    r = None if region is None else np.ascontiguousarray(np.asarray(region, dtype=np.float64).reshape(6))
    stream = torch.cuda.current_stream(dev).cuda_stream
    dropped = ctypes.c_longlong(-1)
    rc = L.b200dp_build_nlist_noalloc(stream, nloc, nghost, x.data_ptr(), t.data_ptr(),
                                      None if b is None else b.ctypes.data_as(dp_),
                                      None if r is None else r.ctypes.data_as(dp_), m.rcut, len(m.sel), sel,
                                      nl.data_ptr(), img.data_ptr(), rij.data_ptr(), ctypes.byref(dropped))
    return rc, dropped.value, out


def build_noalloc(coord, atype, box, m, nghost=0, region=None):
    rc, dropped, (_, _, nl, img, rij) = call_noalloc(coord, atype, box, m, nghost, region)
    return rc, nl.cpu().numpy(), img.cpu().numpy(), rij.cpu().numpy()


@pytest.mark.parametrize("name", ["water192", "water192_triclinic", "cu108", "alloy128"])
def test_noalloc_list_equals_regular_entry(model_dir, name):
    g, meta = golden(name)
    path = golden_model_path(model_dir, meta)
    m = modelgen.load(path)
    dp = b200dp.DeepPot(path, precision=b200dp.FP64)
    dp.compute(g["coord"], g["atype"], g["box"])
    ref = dp.last_nlist(len(g["atype"]))
    dp.close()
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        rc, nl, img, rij = build_noalloc(g["coord"], g["atype"], g["box"], m)
        assert rc == 0
        np.testing.assert_array_equal(nl, ref["nlist"])
        np.testing.assert_array_equal(img, ref["code"])
        np.testing.assert_array_equal(rij, ref["rij"])


def test_noalloc_full_size_and_ghost_mode(model_dir):
    path = str(model_dir / "water.b2dp")
    m = modelgen.load(path)
    dp = b200dp.DeepPot(path, precision=b200dp.FP64)
    s = systems.config1()
    dp.compute(s.coord, s.atype, s.box)
    ref = dp.last_nlist(s.natoms)
    for _ in range(2):
        rc, nl, img, rij = build_noalloc(s.coord, s.atype, s.box, m)
        assert rc == 0
        np.testing.assert_array_equal(nl, ref["nlist"])
        np.testing.assert_array_equal(img, ref["code"])
        np.testing.assert_array_equal(rij, ref["rij"])
    # ghost mode: explicit ghost images, grid region from the coordinates
    from test_oracle import ghost_expand

    s0 = systems.config0()
    coord, atype, _ = ghost_expand(s0, 6.0)
    nghost = len(atype) - s0.natoms
    dp.compute(coord, atype, None, nghost=nghost)
    ref = dp.last_nlist(s0.natoms)
    region = np.concatenate([coord.min(0), coord.max(0)])
    for _ in range(2):
        rc, nl, img, rij = build_noalloc(coord, atype, None, m, nghost=nghost, region=region)
        assert rc == 0
        np.testing.assert_array_equal(nl, ref["nlist"])
        np.testing.assert_array_equal(img, ref["code"])
        np.testing.assert_array_equal(rij, ref["rij"])
    dp.close()


def test_noalloc_rejects_sizes_beyond_its_scratch(model_dir):
    m = modelgen.load(str(model_dir / "water.b2dp"))
    torch = pytest.importorskip("torch")
    L = b200dp.load_library()
    x = torch.zeros(3, dtype=torch.float64, device="cuda:0")
    t = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    sel = (ctypes.c_int * 2)(*m.sel)
    box = np.ascontiguousarray(np.eye(3).reshape(9) * 100.0)
    rc = L.b200dp_build_nlist_noalloc(None, 70000, 0, x.data_ptr(), t.data_ptr(),
                                      box.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), None, m.rcut, 2, sel,
                                      x.data_ptr(), x.data_ptr(), x.data_ptr(), None)
    assert rc == 5  # B200DP_ERR_CAPACITY, before any memory is touched


def test_noalloc_reports_truncated_rows_and_bad_types(model_dir):
    """Rows truncated at sel are counted like the engine counts them, and an
    out-of-range type is reported by status; the next valid call is exact again."""
    path = str(model_dir / "water_smallsel.b2dp")
    m = modelgen.load(path)
    s = systems.config0()
    dp = b200dp.DeepPot(path, precision=b200dp.FP64)
    dp.compute(s.coord, s.atype, s.box)
    ref = dp.last_nlist(s.natoms)
    ref_dropped = dp.sel_overflow_count()
    dp.close()
    assert ref_dropped > 0
    rc, dropped, out = call_noalloc(s.coord, s.atype, s.box, m)
    assert rc == 0 and dropped == ref_dropped
    bad = s.atype.copy()
    bad[5] = 7
    rc, _, _ = call_noalloc(s.coord, bad, s.box, m)
    assert rc == 6  # B200DP_ERR_BAD_TYPE
    rc, dropped, (_, _, nl, img, rij) = call_noalloc(s.coord, s.atype, s.box, m)
    assert rc == 0 and dropped == ref_dropped
    np.testing.assert_array_equal(nl.cpu().numpy(), ref["nlist"])
    np.testing.assert_array_equal(img.cpu().numpy(), ref["code"])
    np.testing.assert_array_equal(rij.cpu().numpy(), ref["rij"])


def test_noalloc_second_call_reserves_no_device_memory(model_dir):
    """After the first call (which loads the module holding the static array),
    a call leaves the device's free memory unchanged."""
    torch = pytest.importorskip("torch")
    m = modelgen.load(str(model_dir / "water.b2dp"))
    s = systems.config1()
    rc, _, out = call_noalloc(s.coord, s.atype, s.box, m)
    assert rc == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        rc, _, _ = call_noalloc(s.coord, s.atype, s.box, m, out=out)
        assert rc == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
