"""Spatial domain decomposition for multi-GPU evaluation.

One process per GPU.  The periodic orthorhombic box is split into a
px x py x pz grid of sub-boxes; each rank owns the atoms inside its sub-box and
receives a ghost shell of width `halo` (>= rcut) from its face neighbours by a
staged exchange along x, then y, then z (ghosts received in an earlier
dimension are forwarded in later ones, which covers edges and corners).  Atoms
sent across the periodic boundary are shifted by one box length, so the
engine's ghost mode (nghost > 0, no periodic images of its own) sees every
neighbour within rcut.  After the force call the ghost forces travel back
through the same passes in reverse order and are added onto the atoms they
came from (LAMMPS' reverse communication, which the reference performs with
MPI in components/lammps-deepmd-plugin/src/pair_deepmd_kokkos.cpp:931).
Energy and virial are summed over ranks with one all-reduce.

The exchanges use torch.distributed point-to-point calls (NCCL on GPUs, gloo
on CPUs), so the same code runs the CPU tests and the GPU benchmark.  Within
one pass the atoms sent in one direction are distinct, so the reverse fold is
a plain indexed add with no colliding indices (deterministic).

With GPUs that are NVLink peers both exchanges can be left out (PeerFold):
the plan also records every ghost's origin (owner rank, owner's row) and its
periodic shift.  Each step every rank publishes its owned positions into a
buffer the others map (CUDA IPC), a one-element all-reduce orders the
publishes before any read, and one kernel fills the ghost rows from the
owners' buffers over NVLink.  After the force call the engine adds each ghost
row's reverse contribution directly into the owner's fixed-point force
accumulator in the owner's memory; the all-reduce of energy and virial orders
every rank's additions before any rank converts its accumulator into forces.
When every rank has a GPU of its own, the barrier and the all-reduce are the
engine's device-side rendezvous through the same peer buffers
(b200dp_peer_reduce: plain peer stores, an arrival counter per rank, bounded
waits); ranks that share a GPU use the process group instead.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import torch
import torch.distributed as dist


def rank_grid(nranks: int) -> tuple[int, int, int]:
    """Slab for 2 ranks, 2x2x1 for 4, 2x2x2 for 8 (x fastest to split)."""
    table = {1: (1, 1, 1), 2: (2, 1, 1), 4: (2, 2, 1), 8: (2, 2, 2)}
    if nranks in table:
        return table[nranks]
    return (nranks, 1, 1)


@dataclasses.dataclass
class Pass:
    dim: int
    direction: int          # +1: send to the +dim neighbour, -1: to the -dim neighbour
    peer_send: int
    peer_recv: int
    shift: float            # added to coordinate `dim` of the atoms sent
    send_idx: torch.Tensor  # rows of the local array that are sent
    recv_off: int           # first row of the received block
    n_recv: int


class Decomposition:
    def __init__(self, box: np.ndarray, grid: tuple[int, int, int], rank: int, halo: float):
        box = np.asarray(box, dtype=np.float64).reshape(3, 3)
        if np.abs(box - np.diag(np.diag(box))).max() > 0:
            raise ValueError("domain decomposition supports orthorhombic boxes")
        self.L = np.diag(box).copy()
        self.grid = tuple(int(g) for g in grid)
        self.rank = rank
        px, py, pz = self.grid
        self.cell = np.array([rank // (py * pz), (rank // pz) % py, rank % pz])
        width = self.L / np.array(self.grid)
        self.lo = self.cell * width
        self.hi = (self.cell + 1) * width
        if np.any(halo > width):
            raise ValueError(f"halo {halo} wider than a sub-box {width}")
        self.halo = float(halo)

    def rank_of(self, cell) -> int:
        px, py, pz = self.grid
        c = [int(cell[d]) % self.grid[d] for d in range(3)]
        return (c[0] * py + c[1]) * pz + c[2]

    def neighbour(self, dim: int, direction: int) -> int:
        c = self.cell.copy()
        c[dim] += direction
        return self.rank_of(c)

    def send_shift(self, dim: int, direction: int) -> float:
        """Shift for atoms sent in `direction` along `dim` (across the box edge)."""
        if direction > 0 and self.cell[dim] == self.grid[dim] - 1:
            return -self.L[dim]
        if direction < 0 and self.cell[dim] == 0:
            return self.L[dim]
        return 0.0

    def owns(self, coord: np.ndarray) -> np.ndarray:
        """Mask of atoms (wrapped into the box) that fall in this rank's sub-box."""
        w = wrap(np.asarray(coord, dtype=np.float64), self.L)
        return np.all((w >= self.lo) & (w < self.hi), axis=1)

    def region(self) -> np.ndarray:
        return np.concatenate([self.lo - self.halo, self.hi + self.halo])


def _exchange(send: torch.Tensor, peer_send: int, recv: torch.Tensor, peer_recv: int, rank: int) -> None:
    if peer_send == rank and peer_recv == rank:
        recv.copy_(send)
        return
    ops = []
    if recv.numel():
        ops.append(dist.P2POp(dist.irecv, recv, peer_recv))
    if send.numel():
        ops.append(dist.P2POp(dist.isend, send.contiguous(), peer_send))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


def _exchange_many(items, rank: int) -> None:
    """Several (send, peer_send, recv, peer_recv) exchanges in one batch.

    Every rank posts the same sequence, so point-to-point messages between a
    pair of ranks match in posting order; self-exchanges are local copies.
    """
    ops = []
    for send, peer_send, recv, peer_recv in items:
        if peer_send == rank and peer_recv == rank:
            recv.copy_(send)
            continue
        if recv.numel():
            ops.append(dist.P2POp(dist.irecv, recv, peer_recv))
        if send.numel():
            ops.append(dist.P2POp(dist.isend, send.contiguous(), peer_send))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


def _exchange_counts(n_send: int, peer_send: int, peer_recv: int, rank: int, device) -> int:
    s = torch.tensor([n_send], dtype=torch.int64, device=device)
    r = torch.zeros(1, dtype=torch.int64, device=device)
    if peer_send == rank and peer_recv == rank:
        return n_send
    for req in dist.batch_isend_irecv([dist.P2POp(dist.irecv, r, peer_recv), dist.P2POp(dist.isend, s, peer_send)]):
        req.wait()
    return int(r.item())


class HaloExchange:
    """Exchange plan for fixed owned atoms; built once, replayed every step."""

    def __init__(self, dd: Decomposition, x_owned: torch.Tensor, types_owned: torch.Tensor,
                 ids_owned: torch.Tensor | None = None):
        self.dd = dd
        self.rank = dd.rank
        dev = x_owned.device
        self.device = dev
        x = x_owned.clone()
        t = types_owned.clone()
        ids = ids_owned.clone() if ids_owned is not None else None
        # origin of every row: (owner rank, owner's row); forwarded like the ids
        org = torch.stack([torch.full((x.shape[0],), self.rank, dtype=torch.int32, device=dev),
                           torch.arange(x.shape[0], dtype=torch.int32, device=dev)], dim=1)
        sh = torch.zeros_like(x)  # periodic shift of every row from its owner's position
        self.nloc = x.shape[0]
        self.passes: list[Pass] = []
        for dim in range(3):
            base_n = x.shape[0]  # both directions select from the atoms present before this dimension
            blocks = []
            for direction in (-1, +1):
                xs = x[:base_n, dim]
                if direction > 0:
                    sel = xs >= dd.hi[dim] - dd.halo
                else:
                    sel = xs < dd.lo[dim] + dd.halo
                idx = torch.nonzero(sel).flatten()
                peer_send = dd.neighbour(dim, direction)
                peer_recv = dd.neighbour(dim, -direction)
                shift = dd.send_shift(dim, direction)
                n_recv = _exchange_counts(int(idx.numel()), peer_send, peer_recv, self.rank, dev)
                sp = x[idx].clone()
                sp[:, dim] += shift
                rp = torch.empty((n_recv, 3), dtype=x.dtype, device=dev)
                _exchange(sp, peer_send, rp, peer_recv, self.rank)
                rt = torch.empty(n_recv, dtype=t.dtype, device=dev)
                _exchange(t[idx].clone(), peer_send, rt, peer_recv, self.rank)
                if ids is not None:
                    ri = torch.empty(n_recv, dtype=ids.dtype, device=dev)
                    _exchange(ids[idx].clone(), peer_send, ri, peer_recv, self.rank)
                else:
                    ri = None
                ro = torch.empty((n_recv, 2), dtype=org.dtype, device=dev)
                _exchange(org[idx].contiguous(), peer_send, ro, peer_recv, self.rank)
                ssh = sh[idx].clone()
                ssh[:, dim] += shift
                rsh = torch.empty((n_recv, 3), dtype=sh.dtype, device=dev)
                _exchange(ssh, peer_send, rsh, peer_recv, self.rank)
                off = x.shape[0] + sum(b[0].shape[0] for b in blocks)
                self.passes.append(Pass(dim, direction, peer_send, peer_recv, shift, idx, off, n_recv))
                blocks.append((rp, rt, ri, ro, rsh))
            x = torch.cat([x] + [b[0] for b in blocks])
            t = torch.cat([t] + [b[1] for b in blocks])
            org = torch.cat([org] + [b[3] for b in blocks])
            sh = torch.cat([sh] + [b[4] for b in blocks])
            if ids is not None:
                ids = torch.cat([ids] + [b[2] for b in blocks])
        self.nall = x.shape[0]
        self.x = x
        self.types = t
        self.ids = ids
        self.origin = org[self.nloc:].contiguous()  # [nghost, 2] int32: owner rank, owner's row
        # [nghost, 3]: each component is one pass's shift (or 0), so owner + shift is the
        # same single addition the staged exchange makes
        self.shift = sh[self.nloc:].contiguous()

    @property
    def nghost(self) -> int:
        return self.nall - self.nloc

    def forward(self, x_all: torch.Tensor) -> None:
        """Refreshes the ghost rows of x_all ([nall, 3]) from the owners' rows.

        Dimensions go in order (a later one forwards ghosts of an earlier one);
        the two directions of a dimension are independent and share one batch.
        """
        for d in range(3):
            items = []
            for p in self.passes[2 * d:2 * d + 2]:
                sp = x_all.index_select(0, p.send_idx)
                if p.shift:
                    sp[:, p.dim] += p.shift
                items.append((sp, p.peer_send, x_all[p.recv_off:p.recv_off + p.n_recv], p.peer_recv))
            _exchange_many(items, self.rank)

    def reverse(self, f_all: torch.Tensor) -> None:
        """Folds ghost forces back onto the atoms they were copied from
        (dimensions in reverse order, both directions of one in one batch)."""
        for d in (2, 1, 0):
            items, backs = [], []
            for p in reversed(self.passes[2 * d:2 * d + 2]):
                back = torch.empty((p.send_idx.numel(), f_all.shape[1]), dtype=f_all.dtype, device=self.device)
                items.append((f_all[p.recv_off:p.recv_off + p.n_recv].contiguous(), p.peer_recv, back, p.peer_send))
                backs.append((p, back))
            _exchange_many(items, self.rank)
            for p, back in backs:
                f_all.index_add_(0, p.send_idx, back)


def wrap(coord: np.ndarray, L: np.ndarray) -> np.ndarray:
    """Positions wrapped into [0, L) per axis (a rounding result of exactly L goes to 0)."""
    w = coord - np.floor(coord / L) * L
    return np.where(w >= L, w - L, w)


def distribute(coord: np.ndarray, atype: np.ndarray, dd: Decomposition):
    """Owned atoms of this rank from a global system: wrapped positions, types, global ids."""
    w = wrap(np.asarray(coord, dtype=np.float64), dd.L)
    mask = dd.owns(w)
    ids = np.nonzero(mask)[0]
    return w[mask], np.asarray(atype)[mask], ids


class PeerFold:
    """Halo exchange and reverse pass through peer memory for a b200dp engine
    (b200dp_fold_* / b200dp_halo_*).

    Each rank exports one buffer (CUDA IPC handle) holding its owned atoms'
    published positions and fixed-point force accumulator, and opens every
    other rank's.  `publish` + `gather` replace the forward exchange: the
    ghost rows are read from the owners' positions (plus the periodic shift)
    by one kernel, after a barrier that orders every rank's publish before
    any read.  The force call adds the reverse contribution of every ghost
    row straight into the owner's accumulator (integer atomics over NVLink,
    order-independent sums) instead of returning ghost forces; `finish`
    converts this rank's accumulator into the owned rows' forces and must run
    after every rank's force call has completed, which the all-reduce of
    energy and virial on the same stream guarantees.  Ranks that share one
    GPU work too (the handles then map the same device's memory).
    """

    gathers = True

    def __init__(self, dp, device, stream=None, capacity_margin: float = 2.0, device_sync: bool | None = None):
        self.dp = dp
        self.device = torch.device(device)
        self.stream = stream
        self.margin = capacity_margin
        self.origin = self.shift = None
        # None: the device-side rendezvous (b200dp_peer_reduce) when every rank has a GPU of its own,
        # else the process group's all-reduce
        self.device_sync = device_sync

    def _stream(self) -> int:
        if self.stream is not None:
            return self.stream.cuda_stream
        return torch.cuda.current_stream(self.device).cuda_stream

    def setup(self, rank: int, nranks: int, nloc: int, origin: torch.Tensor, shift: torch.Tensor) -> None:
        """Collective over all ranks: export (one capacity for all), exchange handles, open them,
        upload the ghost origins and shifts."""
        nlocs = [nloc]
        if dist.is_initialized():
            nlocs = [None] * nranks
            dist.all_gather_object(nlocs, nloc)
        h = self.dp.fold_export(int(self.margin * max(nlocs)) + 1024)
        handles = [h]
        if dist.is_initialized():
            handles = [None] * nranks
            dist.all_gather_object(handles, h)
        self.dp.fold_connect(rank, handles)
        if self.device_sync is None:
            import socket

            me = (socket.gethostname(), str(torch.cuda.get_device_properties(self.device).uuid))
            ids = [me]
            if dist.is_initialized():
                ids = [None] * nranks
                dist.all_gather_object(ids, me)
            self.device_sync = len(set(ids)) == len(ids)
        self.origin = origin.to(device=self.device, dtype=torch.int32).contiguous()
        self.shift = shift.to(device=self.device, dtype=torch.float64).contiguous()
        self.dp.fold_origins(self.origin.shape[0], self.origin.data_ptr(), self.shift.data_ptr())

    def publish(self, x_all, nloc) -> None:
        self.dp.halo_publish(self._stream(), nloc, x_all.data_ptr())

    def gather(self, x_all, nloc, nghost) -> None:
        self.dp.halo_gather(self._stream(), nloc, nghost, x_all.data_ptr())

    def compute(self, x_all, t_all, nloc, nghost, region, e, f, v):
        self.dp.compute_device_fold(self._stream(), nloc, nghost, x_all.data_ptr(), t_all.data_ptr(), region,
                                    e.data_ptr(), f.data_ptr(), v.data_ptr())

    def finish(self, f, nloc) -> None:
        self.dp.fold_finish(self._stream(), nloc, f.data_ptr())

    def barrier(self) -> None:
        """Every rank's publish is complete before any rank's gather reads it."""
        if self.device_sync:
            self.dp.peer_reduce(self._stream(), 0)
        elif dist.is_initialized():
            dist.all_reduce(torch.zeros(1, device=self.device))

    def reduce(self, ev) -> None:
        """Sum of energy and virial over the ranks (in place); also orders every rank's force
        additions before any rank's finish."""
        if self.device_sync:
            self.dp.peer_reduce(self._stream(), ev.numel(), ev.data_ptr(), ev.data_ptr())
        elif dist.is_initialized():
            dist.all_reduce(ev, op=dist.ReduceOp.SUM)


class DistributedDeepPot:
    """Energy, forces and virial of a periodic system split over the ranks.

    `compute(x_all, t_all, nloc, nghost, region, e, f, v)` is the per-rank
    force call in ghost mode: it reads nloc owned + nghost ghost rows and
    writes the energy of the owned atoms into e[0], forces on all rows into
    f [nall, 3] (ghost rows are partial forces for the owners) and the virial
    of the owned atoms' edges into v [9].  With the b200dp engine this is
    b200dp_compute_device on the rank's stream; the tests pass the CPU oracle.
    Per step: forward halo of coordinates, the force call, reverse fold of the
    ghost forces, one all-reduce of energy and virial (10 fp64).  With
    `fold` (a PeerFold, or anything with its methods) the ghost rows come
    from fold.publish / barrier / fold.gather (or the staged forward exchange
    when fold.gathers is false), the force call is fold.compute, the reverse
    exchange is left out and fold.finish follows the all-reduce.
    """

    def __init__(self, compute, box, grid, rank, halo, x_owned, t_owned, ids_owned=None, device="cpu", fold=None):
        self.dd = Decomposition(box, grid, rank, halo)
        self.compute = compute
        self.fold = fold
        dev = torch.device(device)
        self.device = dev
        x = torch.as_tensor(np.asarray(x_owned, dtype=np.float64), device=dev)
        t = torch.as_tensor(np.asarray(t_owned, dtype=np.int32), device=dev)
        ids = None if ids_owned is None else torch.as_tensor(np.asarray(ids_owned, dtype=np.int64), device=dev)
        if dist.is_initialized():  # first collective on every rank before any point-to-point call
            dist.barrier()
        self.plan = HaloExchange(self.dd, x, t, ids)
        self.x = self.plan.x.contiguous()
        self.types = self.plan.types.to(torch.int32).contiguous()
        self.ids = self.plan.ids
        self.nloc = self.plan.nloc
        self.nghost = self.plan.nghost
        self.force = torch.zeros((self.plan.nall, 3), dtype=torch.float64, device=dev)
        self.ev = torch.zeros(10, dtype=torch.float64, device=dev)  # energy, virial[9]
        self.region = self.dd.region()
        if fold is not None:
            nranks = dist.get_world_size() if dist.is_initialized() else 1
            fold.setup(rank, nranks, self.nloc, self.plan.origin, self.plan.shift)
        self._bar = torch.zeros(1, dtype=torch.float32, device=dev)

    def set_positions(self, x_owned: torch.Tensor) -> None:
        """New owned positions (same atoms, same owner; migration needs a new plan)."""
        self.x[: self.nloc].copy_(x_owned)

    def step(self):
        """Returns (energy [1], force of owned atoms [nloc, 3], virial [9]) summed over ranks."""
        if self._graph is not None:
            self._graph.replay()
            return self.ev[0:1], self.force[: self.nloc], self.ev[1:10]
        if self.fold is not None and self.fold.gathers:
            self.fold.publish(self.x, self.nloc)
            self._barrier()  # every rank's positions are published before any is read
            self.fold.gather(self.x, self.nloc, self.nghost)
        else:
            self.plan.forward(self.x)
        if self.fold is not None:
            self.fold.compute(self.x, self.types, self.nloc, self.nghost, self.region, self.ev[0:1], self.force,
                              self.ev[1:10])
            self._reduce_ev()  # every rank's additions are done once this completes
            self.fold.finish(self.force, self.nloc)
            return self.ev[0:1], self.force[: self.nloc], self.ev[1:10]
        self.compute(self.x, self.types, self.nloc, self.nghost, self.region, self.ev[0:1], self.force,
                     self.ev[1:10])
        self.plan.reverse(self.force)
        if dist.is_initialized():
            dist.all_reduce(self.ev, op=dist.ReduceOp.SUM)
        return self.ev[0:1], self.force[: self.nloc], self.ev[1:10]

    def _barrier(self) -> None:
        if hasattr(self.fold, "barrier"):
            self.fold.barrier()
        elif dist.is_initialized():
            dist.all_reduce(self._bar)

    def _reduce_ev(self) -> None:
        if hasattr(self.fold, "reduce"):
            self.fold.reduce(self.ev)
        elif dist.is_initialized():
            dist.all_reduce(self.ev, op=dist.ReduceOp.SUM)

    _graph = None

    def capture(self) -> None:
        """Records one whole step (halo exchange, force call, reverse fold,
        all-reduce) as a CUDA graph; later step() calls replay it.  The many
        small exchange launches then cost no host time.  Every rank captures
        together; `compute` must launch on torch's current stream; positions
        change through `set_positions` (same buffer).  Call release() before
        the process group is destroyed."""
        if self.device.type != "cuda":
            return
        cur = torch.cuda.current_stream(self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            self.step()  # warm-up on the capturing stream
        cur.wait_stream(side)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step()
        self._graph = g

    def release(self) -> None:
        self._graph = None
