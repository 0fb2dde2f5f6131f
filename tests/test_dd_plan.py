"""The host plan of the C++ decomposed driver (b200dp_dd_*), checked on CPU.

b200dp_dd_plan_emulate runs the driver's own migration and ghost-plan code
with threads standing in for the ranks (the same code that exchanges its
messages over NCCL on GPUs).  Against a brute-force enumeration in numpy:
  * every atom is owned by exactly one rank, the one whose sub-box holds its
    wrapped position, and each rank keeps its atoms in global-id order;
  * each rank's ghosts are exactly the periodic images (atom, shift with
    components in {-L, 0, L}) that fall inside the sub-box widened by the
    halo, minus the rank's own atoms, each once;
  * every ghost's position is its owner's position plus its shift (bit for
    bit) and its origin (owner rank, owner's row) names that atom;
  * after a displacement that takes atoms across sub-box faces, edges,
    corners and the periodic boundary, the migration hands every atom to its
    new owner.
"""
import itertools

import numpy as np
import pytest

import b200dp
import systems


def wrap(x, L):
    w = x - np.floor(x / L) * L
    return np.where(w >= L, w - L, w)


def bounds(rank, grid, L):
    px, py, pz = grid
    cell = np.array([rank // (py * pz), (rank // pz) % py, rank % pz])
    w = L / np.array(grid)
    return cell * w, (cell + 1) * w


def check_plan(ranks, grid, L, halo, pos):
    n = pos.shape[0]
    owner = np.full(n, -1)
    for r, d in enumerate(ranks):
        lo, hi = bounds(r, grid, L)
        ids = d["owned"]
        assert np.all(np.diff(ids) > 0)
        inside = np.all((pos[ids] >= lo) & (pos[ids] < hi), axis=1)
        assert inside.all()
        assert np.all(owner[ids] == -1)
        owner[ids] = r
    assert np.all(owner >= 0)
    shifts = np.array(list(itertools.product((-1.0, 0.0, 1.0), repeat=3))) * L
    for r, d in enumerate(ranks):
        lo, hi = bounds(r, grid, L)
        expect = []
        for s in shifts:
            q = pos + s
            ok = np.all((q >= lo - halo) & (q < hi + halo), axis=1)
            if not np.any(s):
                ok &= owner != r
            for i in np.nonzero(ok)[0]:
                expect.append((int(i), float(s[0]), float(s[1]), float(s[2])))
        got = [(int(i), float(a), float(b), float(c)) for i, (a, b, c) in zip(d["ghost_ids"], d["ghost_shift"])]
        assert len(got) == len(set(got))
        assert sorted(got) == sorted(expect)
        # positions and origins
        gid = d["ghost_ids"]
        np.testing.assert_array_equal(d["ghost_x"], pos[gid] + d["ghost_shift"])
        for (orank, orow), i in zip(d["ghost_origin"], gid):
            assert ranks[orank]["owned"][orow] == i


@pytest.mark.parametrize("grid", [(1, 1, 1), (2, 1, 1), (3, 1, 1), (2, 2, 1), (2, 2, 2)])
def test_plan_matches_brute_force(grid):
    s = systems.water(8)  # 1,536 atoms, 24.84 A cube
    L = np.diag(s.box)
    halo = 6.0
    nr = int(np.prod(grid))
    ranks = b200dp.dd_plan_emulate(nr, grid, s.box, halo, s.coord)
    check_plan(ranks, grid, L, halo, wrap(s.coord, L))


@pytest.mark.parametrize("grid", [(2, 1, 1), (2, 2, 2), (3, 1, 1)])
def test_migration_after_a_move(grid):
    s = systems.water(8)
    L = np.diag(s.box)
    halo = 6.0
    rng = np.random.default_rng(5)
    disp = rng.uniform(-2.5, 2.5, size=s.coord.shape)
    # atoms next to the periodic faces step across them
    w = wrap(s.coord, L)
    disp[w[:, 0] < 1.0, 0] = -1.7
    disp[w[:, 1] > L[1] - 1.0, 1] = 1.9
    nr = int(np.prod(grid))
    ranks = b200dp.dd_plan_emulate(nr, grid, s.box, halo, s.coord, disp=disp)
    pos = wrap(w + disp, L)
    check_plan(ranks, grid, L, halo, pos)
    moved = sum(len(d["owned"]) for d in ranks)
    assert moved == s.natoms


def test_plan_rejects_a_halo_wider_than_a_sub_box():
    s = systems.water(4)  # 12.42 A: two ranks give 6.21 A sub-boxes
    with pytest.raises(b200dp.B200DPError):
        b200dp.dd_plan_emulate(2, (2, 1, 1), s.box, 7.0, s.coord)
