"""b200dp_direct_energy_force: the reference's direct-engine entry on a canonical graph.

The caller hands a destination-major CSR graph (int64 types and row pointers,
uint32 sources, fp32 edge vectors x_j - x_i with periodic images as separate
edges) and device outputs; the entry returns 1 when it handled the call and 0
when the caller must fall back.  With coordinates and box on a 2^-10 grid every
edge vector is exact in fp32, so the graph path must agree with the periodic
coordinate path to fp64 round-off; with arbitrary coordinates the fp32 edge
vectors bound the agreement (1e-5 relative).
"""
import numpy as np
import pytest

import b200dp
import systems

pytestmark = pytest.mark.gpu


def snapped(s, q=1024.0):
    L = np.round(np.diag(s.box) * q) / q
    box = np.diag(L)
    coord = np.round((s.coord - np.floor(s.coord / L) * L) * q) / q
    return coord, box


def canonical_graph(coord, atype, box, rc, rng):
    """All (i, j, image) pairs within rc, rows shuffled; int64 / uint32 / fp32 arrays."""
    L = np.diag(box)
    n = len(atype)
    reach = [int(np.ceil(rc / l)) for l in L]
    rows = [[] for _ in range(n)]
    for a in range(-reach[0], reach[0] + 1):
        for b in range(-reach[1], reach[1] + 1):
            for c in range(-reach[2], reach[2] + 1):
                d = coord[None, :, :] + np.array([a, b, c]) * L - coord[:, None, :]  # [i, j, 3]
                r2 = (d ** 2).sum(-1)
                ii, jj = np.nonzero((r2 < rc * rc) & (r2 > 0))
                for i, j in zip(ii, jj):
                    rows[i].append((j, d[i, j]))
    row_ptr = np.zeros(n + 1, np.int64)
    src, vec = [], []
    for i in range(n):
        order = rng.permutation(len(rows[i]))
        for k in order:
            src.append(rows[i][k][0])
            vec.append(rows[i][k][1])
        row_ptr[i + 1] = row_ptr[i] + len(rows[i])
    return (np.asarray(atype, np.int64), row_ptr, np.asarray(src, np.uint32),
            np.asarray(vec, np.float32).reshape(-1, 3))


def run_direct(dp, graph, n, nloc=None):
    import torch

    dev = torch.device("cuda:0")
    at, rp, src, vec = (torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in graph)
    e = torch.full((n,), np.nan, dtype=torch.float64, device=dev)
    f = torch.full((n, 3), np.nan, dtype=torch.float64, device=dev)
    v = torch.full((n, 9), np.nan, dtype=torch.float64, device=dev)
    stream = torch.cuda.current_stream(dev)
    b200dp.direct_bind(dp, stream.cuda_stream)
    rc = b200dp.direct_energy_force(at.data_ptr(), rp.data_ptr(), src.data_ptr(), vec.data_ptr(), n,
                                    n if nloc is None else nloc, len(graph[2]), e.data_ptr(), f.data_ptr(),
                                    v.data_ptr())
    torch.cuda.synchronize()
    return rc, e.cpu().numpy(), f.cpu().numpy(), v.cpu().numpy()


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-300))


def assert_matches_oracle(model_path, coord, atype, box, e, f, v, tol):
    """The direct entry's per-atom outputs against the CPU oracle's periodic evaluation
    of the same coordinates (fp64 1e-10, mixed 2e-4 of the largest component)."""
    import oracle

    ref = oracle.Oracle(model_path).compute(coord, atype, box, atomic=True)
    assert rel(f, ref["force"]) < tol
    assert rel(e, ref["atom_energy"]) < tol
    assert rel(v, ref["atom_virial"]) < tol
    assert abs(e.sum() - ref["energy"]) <= tol * abs(ref["energy"])


@pytest.mark.parametrize("precision,tol", [(b200dp.FP64, 1e-11), (b200dp.MIXED, 2e-4)])
def test_direct_graph_equals_periodic_coordinates(model_dir, precision, tol):
    s = systems.config0()
    coord, box = snapped(s)
    graph = canonical_graph(coord, s.atype, box, 6.0, np.random.default_rng(1))
    dp = b200dp.DeepPot(str(model_dir / "water.b2dp"), precision=precision)
    ref = dp.compute(coord, s.atype, box, atomic=True)
    for _ in range(2):
        rc, e, f, v = run_direct(dp, graph, s.natoms)
        dp.check()
        assert rc == 1
        assert rel(f, ref["force"]) < tol
        assert rel(e, ref["atom_energy"]) < tol
        assert rel(v, ref["atom_virial"]) < tol
        assert abs(e.sum() - ref["energy"]) <= tol * abs(ref["energy"])
        assert rel(v.sum(0).reshape(3, 3), ref["virial"]) < tol
    assert_matches_oracle(str(model_dir / "water.b2dp"), coord, s.atype, box, e, f, v,
                          1e-10 if precision == b200dp.FP64 else tol)
    b200dp.direct_bind(None)
    dp.close()


def test_direct_graph_fp32_edges(model_dir):
    """Arbitrary coordinates: the fp32 edge vectors limit the agreement."""
    s = systems.config0()
    graph = canonical_graph(s.coord - np.floor(s.coord / np.diag(s.box)) * np.diag(s.box), s.atype, s.box, 6.0,
                            np.random.default_rng(2))
    dp = b200dp.DeepPot(str(model_dir / "water.b2dp"), precision=b200dp.FP64)
    ref = dp.compute(s.coord, s.atype, s.box, atomic=True)
    rc, e, f, v = run_direct(dp, graph, s.natoms)
    assert rc == 1
    assert rel(f, ref["force"]) < 1e-5
    assert rel(e, ref["atom_energy"]) < 1e-5
    b200dp.direct_bind(None)
    dp.close()


def test_direct_declines_what_it_cannot_handle(model_dir):
    s = systems.config0()
    coord, box = snapped(s)
    graph = canonical_graph(coord, s.atype, box, 6.0, np.random.default_rng(3))
    dp = b200dp.DeepPot(str(model_dir / "water.b2dp"), precision=b200dp.MIXED)
    b200dp.direct_bind(None)
    assert b200dp.direct_energy_force(1, 1, 1, 1, s.natoms, s.natoms, 1, 1, 1, 1) == 0  # no engine bound
    rc, *_ = run_direct(dp, graph, s.natoms, nloc=s.natoms - 1)  # ghost nodes: caller's fallback
    assert rc == 0
    b200dp.direct_bind(dp, 0)
    assert b200dp.direct_energy_force(1, 1, 1, 1, 0, 0, 0, 1, 1, 1) == 0  # empty graph
    b200dp.direct_bind(None)
    dp.close()


def raw_graph(coord, atype, box, rc_graph, rng):
    """A canonical graph with skin candidates (every (i, j, image) within rc_graph) plus what a
    LAMMPS builder binds for the raw-neighbour view: positions of the local atoms followed by one
    ghost position per image edge, and per edge the candidate atom index into them."""
    L = np.diag(box)
    n = len(atype)
    reach = [int(np.ceil(rc_graph / l)) for l in L]
    rows = [[] for _ in range(n)]
    ghosts = []
    for a in range(-reach[0], reach[0] + 1):
        for b in range(-reach[1], reach[1] + 1):
            for c in range(-reach[2], reach[2] + 1):
                shift = np.array([a, b, c]) * L
                d = coord[None, :, :] + shift - coord[:, None, :]
                r2 = (d ** 2).sum(-1)
                ii, jj = np.nonzero((r2 < rc_graph * rc_graph) & (r2 > 0))
                for i, j in zip(ii, jj):
                    if a == 0 and b == 0 and c == 0:
                        cand = j
                    else:
                        cand = n + len(ghosts)
                        ghosts.append(coord[j] + shift)
                    rows[i].append((j, d[i, j], cand))
    row_ptr = np.zeros(n + 1, np.int64)
    src, vec, cand = [], [], []
    for i in range(n):
        for k in rng.permutation(len(rows[i])):
            src.append(rows[i][k][0])
            vec.append(rows[i][k][1])
            cand.append(rows[i][k][2])
        row_ptr[i + 1] = row_ptr[i] + len(rows[i])
    x_ext = np.concatenate([coord, np.asarray(ghosts).reshape(-1, 3)])
    graph = (np.asarray(atype, np.int64), row_ptr, np.asarray(src, np.uint32),
             np.asarray(vec, np.float32).reshape(-1, 3))
    return graph, x_ext, np.asarray(cand, np.int32)


@pytest.mark.parametrize("precision,tol", [(b200dp.FP64, 1e-10), (b200dp.MIXED, 2e-4)])
def test_raw_neighbour_view(model_dir, precision, tol):
    """With a bound raw-neighbour view the entry recomputes edge vectors in fp64 from the
    positions and cuts at the model's rcut, so a graph with 1 A of skin candidates and
    arbitrary (unsnapped) coordinates gives the periodic evaluation to fp64 round-off."""
    import torch

    s = systems.config0()
    coord = s.coord - np.floor(s.coord / np.diag(s.box)) * np.diag(s.box)
    graph, x_ext, cand = raw_graph(coord, s.atype, s.box, 7.0, np.random.default_rng(4))
    n = s.natoms
    dp = b200dp.DeepPot(str(model_dir / "water.b2dp"), precision=precision)
    ref = dp.compute(coord, s.atype, s.box, atomic=True)
    dev = torch.device("cuda:0")
    at, rp, src, vec = (torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in graph)
    xt = torch.from_numpy(x_ext).to(dev)
    m2a = torch.arange(n, dtype=torch.int32, device=dev)
    ct = torch.from_numpy(cand).to(dev)
    vec.fill_(float("nan"))  # the entry must not read the fp32 vectors while the view is bound
    e = torch.full((n,), np.nan, dtype=torch.float64, device=dev)
    f = torch.full((n, 3), np.nan, dtype=torch.float64, device=dev)
    v = torch.full((n, 9), np.nan, dtype=torch.float64, device=dev)
    stream = torch.cuda.current_stream(dev)
    b200dp.direct_bind(dp, stream.cuda_stream)
    assert b200dp.direct_destination_only_ready(n, n) == 1
    assert b200dp.direct_destination_only_ready(n, n - 1) == 0
    b200dp.bind_direct_neighbor_view(xt.data_ptr(), m2a.data_ptr(), ct.data_ptr(), src.data_ptr(), 3, 1, n, 49.0, 1.0)
    view = b200dp.get_direct_neighbor_view()
    assert view.node_count == n and view.source == src.data_ptr()
    call = lambda: b200dp.direct_energy_force(at.data_ptr(), rp.data_ptr(), src.data_ptr(), vec.data_ptr(), n, n,
                                              len(graph[2]), e.data_ptr(), f.data_ptr(), v.data_ptr())
    assert call() == 1
    torch.cuda.synchronize()
    dp.check()
    assert rel(f.cpu().numpy(), ref["force"]) < tol
    assert rel(e.cpu().numpy(), ref["atom_energy"]) < tol
    assert rel(v.cpu().numpy(), ref["atom_virial"]) < tol
    assert_matches_oracle(str(model_dir / "water.b2dp"), coord, s.atype, s.box, e.cpu().numpy(), f.cpu().numpy(),
                          v.cpu().numpy(), tol)
    # the 9-float global virial of the call, at a stable device address
    ptr = b200dp.direct_fp32_global_virial_pointer()
    assert ptr

    class DeviceArray:  # zero-copy view of the engine's buffer
        __cuda_array_interface__ = {"shape": (9,), "typestr": "<f4", "data": (ptr, False), "version": 2}

    g32 = torch.as_tensor(DeviceArray(), device=dev).cpu().numpy()
    assert np.abs(g32 - ref["virial"].reshape(9)).max() <= 1e-5 * np.abs(ref["virial"]).max()
    assert b200dp.direct_fp32_global_virial_pointer() == ptr
    # no virial requested: the per-atom virial is left untouched, forces unchanged
    b200dp.direct_set_need_virial(0)
    v.fill_(float("nan"))
    f2 = f.clone()
    assert call() == 1
    torch.cuda.synchronize()
    assert torch.isnan(v).all()
    assert rel(f.cpu().numpy(), f2.cpu().numpy()) == 0.0
    b200dp.direct_set_need_virial(1)
    # a view bound for another graph is stale: the fp32 vectors are used again
    b200dp.bind_direct_neighbor_view(xt.data_ptr(), m2a.data_ptr(), ct.data_ptr(), src.data_ptr() + 4, 3, 1, n, 49.0,
                                     1.0)
    vec.copy_(torch.from_numpy(graph[3]).to(dev))
    assert call() == 1
    torch.cuda.synchronize()
    assert rel(f.cpu().numpy(), ref["force"]) < 1e-4
    b200dp.bind_direct_neighbor_view(0)
    b200dp.direct_bind(None)
    assert b200dp.direct_destination_only_ready(n, n) == 0
    dp.close()
