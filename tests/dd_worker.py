"""One rank of the domain-decomposition tests, run as a subprocess.

--engine oracle: the per-rank force call is the CPU oracle in ghost mode, the
  exchange runs over gloo on CPU tensors.
--engine b200dp --backend gloo: the force call is b200dp_compute_device on
  cuda:0 (every rank on the same GPU, each with its own engine; nothing on
  the GPU waits for another rank), the exchange over gloo on CPU tensors.
--engine b200dp --backend nccl: one GPU per rank, exchange over NCCL.
--fold: the reverse exchange is replaced by the engine's peer fold (ghost
  contributions added into the owners' accumulators through CUDA IPC); with
  gloo the ranks share cuda:0 and the host synchronises before the all-reduce.
The rank also records its ghost origins (owner rank, owner's row) and the
global ids of its ghost rows.
The rank writes its owned atoms' global ids and forces plus the all-reduced
energy and virial to an .npz for the parent test.
"""
import argparse
import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "dpa4c-scale-aware-md_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import domain  # noqa: E402
import systems  # noqa: E402


def oracle_compute(model):
    import oracle

    oracle.set_threads(1)
    o = oracle.Oracle(model)

    def compute(x_all, t_all, nloc, nghost, region, e, f, v):
        r = o.compute(x_all.numpy(), t_all.numpy(), None, nloc=nloc, atomic=False)
        e.copy_(torch.tensor([r["energy"]], dtype=torch.float64))
        f.copy_(torch.from_numpy(r["force"]))
        v.copy_(torch.from_numpy(r["virial"].reshape(9)))

    return compute


def b200dp_compute(model, precision, device, staged):
    import b200dp

    dev = torch.device(device)
    dp = b200dp.DeepPot(model, precision=b200dp.FP64 if precision == "fp64" else b200dp.MIXED,
                        device=dev.index or 0)
    stream = torch.cuda.current_stream(dev)

    def compute(x_all, t_all, nloc, nghost, region, e, f, v):
        if staged:  # CPU exchange buffers: copy to the GPU and back around the force call
            xd, td = x_all.to(dev), t_all.to(dev)
            ed = torch.zeros(1, dtype=torch.float64, device=dev)
            fd = torch.zeros_like(xd)
            vd = torch.zeros(9, dtype=torch.float64, device=dev)
        else:
            xd, td, ed, fd, vd = x_all, t_all, e, f, v
        dp.compute_device(stream.cuda_stream, nloc, nghost, xd.data_ptr(), td.data_ptr(), None, region,
                          ed.data_ptr(), fd.data_ptr(), vd.data_ptr())
        if staged:
            e.copy_(ed.cpu())
            f.copy_(fd.cpu())
            v.copy_(vd.cpu())
        dp.check()

    compute.engine = dp
    return compute


class SharedMemoryFold:
    """CPU stand-in for domain.PeerFold (oracle ranks over gloo): the peers'
    buffers are POSIX shared-memory segments, one per rank, holding the owned
    positions and one force slot per (owner, source rank) so that no two ranks
    add into the same memory.  The step follows PeerFold's sequence and its
    ordering rules (publish, barrier, gather; force call whose ghost rows go to
    the owners' slots; all-reduce; finish), so the host orchestration of the
    peer mode is exercised without GPUs."""

    gathers = True

    def __init__(self, compute, tag):
        self.compute_rows = compute
        self.tag = tag
        self.segs = []

    def setup(self, rank, nranks, nloc, origin, shift):
        from multiprocessing import shared_memory

        self.rank, self.nranks = rank, nranks
        nlocs = [None] * nranks
        dist.all_gather_object(nlocs, nloc)
        self.cap = max(nlocs)
        nbytes = 8 * self.cap * 3 * (1 + nranks)  # positions, then a force slot per source rank
        mine = shared_memory.SharedMemory(name=f"{self.tag}_{rank}", create=True, size=nbytes)
        self.segs = [mine]
        dist.barrier()
        self.views = []
        for r in range(nranks):
            seg = mine if r == rank else shared_memory.SharedMemory(name=f"{self.tag}_{r}")
            if r != rank:
                self.segs.append(seg)
            self.views.append(np.ndarray((1 + nranks, self.cap, 3), dtype=np.float64, buffer=seg.buf))
        self.views[rank][:] = 0.0
        dist.barrier()
        self.origin = origin.numpy().astype(np.int64)
        self.shift = shift.numpy()

    def publish(self, x_all, nloc):
        self.views[self.rank][0, :nloc] = x_all[:nloc].numpy()

    def gather(self, x_all, nloc, nghost):
        o = self.origin
        xs = np.empty((nghost, 3))
        for r in range(self.nranks):
            m = o[:, 0] == r
            xs[m] = self.views[r][0, o[m, 1]]
        x_all[nloc:] = torch.from_numpy(xs + self.shift)

    def compute(self, x_all, t_all, nloc, nghost, region, e, f, v):
        fa = torch.zeros_like(x_all)
        self.compute_rows(x_all, t_all, nloc, nghost, region, e, fa, v)
        f[:nloc] = fa[:nloc]
        gf = fa[nloc:].numpy()
        o = self.origin
        for r in range(self.nranks):  # ghost rows into the owners' slot for this source rank
            m = o[:, 0] == r
            slot = self.views[r][1 + self.rank]
            np.add.at(slot, o[m, 1], gf[m])

    def finish(self, f, nloc):
        acc = self.views[self.rank]
        total = np.zeros((nloc, 3))
        for src in range(self.nranks):  # fixed order
            total += acc[1 + src, :nloc]
            acc[1 + src, :nloc] = 0.0
        f[:nloc] += torch.from_numpy(total)

    def close(self):
        for seg in self.segs:
            seg.close()
        if self.segs:
            self.segs[0].unlink()
        self.segs = []


class StagedFold:
    """PeerFold for ranks that exchange CPU tensors over gloo and share one GPU
    (the host synchronises after every device step, so no rank's kernel waits
    for another's)."""

    gathers = True

    def __init__(self, dp, device):
        self.pf = domain.PeerFold(dp, device)
        self.dev = torch.device(device)
        self.dp = dp

    def setup(self, rank, nranks, nloc, origin, shift):
        self.pf.setup(rank, nranks, nloc, origin, shift)

    def publish(self, x_all, nloc):
        self.xp = x_all.to(self.dev)
        self.pf.publish(self.xp, nloc)
        torch.cuda.synchronize(self.dev)

    def gather(self, x_all, nloc, nghost):
        xd = x_all.to(self.dev)
        self.pf.gather(xd, nloc, nghost)
        x_all[nloc:].copy_(xd[nloc:].cpu())

    def compute(self, x_all, t_all, nloc, nghost, region, e, f, v):
        self.xd, self.td = x_all.to(self.dev), t_all.to(self.dev)
        self.fd = torch.zeros_like(self.xd)
        ed = torch.zeros(1, dtype=torch.float64, device=self.dev)
        vd = torch.zeros(9, dtype=torch.float64, device=self.dev)
        self.pf.compute(self.xd, self.td, nloc, nghost, region, ed, self.fd, vd)
        e.copy_(ed.cpu())  # host sync: this rank's additions into the peers are complete
        v.copy_(vd.cpu())
        self.dp.check()

    def finish(self, f, nloc):
        self.pf.finish(self.fd, nloc)
        f[:nloc].copy_(self.fd[:nloc].cpu())
        self.dp.check()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--mol", type=int, nargs=3, required=True)
    ap.add_argument("--grid", type=int, nargs=3, required=True)
    ap.add_argument("--halo", type=float, required=True)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--engine", default="oracle", choices=["oracle", "b200dp"])
    ap.add_argument("--backend", default="gloo", choices=["gloo", "nccl"])
    ap.add_argument("--precision", default="fp64", choices=["fp64", "mixed"])
    ap.add_argument("--fold", action="store_true")
    ap.add_argument("--capture", action="store_true", help="replay the step as a CUDA graph (nccl)")
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    device = "cpu"
    kw = {}
    if a.backend == "nccl":
        device = f"cuda:{rank}"
        torch.cuda.set_device(rank)
        kw["device_id"] = torch.device(device)
    dist.init_process_group(a.backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60), **kw)
    s = systems.water(*a.mol, seed=3)
    dd = domain.Decomposition(s.box, a.grid, rank, a.halo)
    x, t, ids = domain.distribute(s.coord, s.atype, dd)
    fold = None
    if a.engine == "oracle":
        compute = oracle_compute(a.model)
        if a.fold:
            fold = SharedMemoryFold(compute, f"b2dp_fold_{os.environ['MASTER_PORT']}")
    else:
        compute = b200dp_compute(a.model, a.precision, device if a.backend == "nccl" else "cuda:0",
                                 staged=a.backend == "gloo")
        if a.fold:
            fold = domain.PeerFold(compute.engine, device) if a.backend == "nccl" else \
                StagedFold(compute.engine, "cuda:0")
    ddp = domain.DistributedDeepPot(compute, s.box, a.grid, rank, a.halo, x, t, ids, device=device, fold=fold)
    if a.capture:
        ddp.capture()
    for _ in range(a.steps):  # the plan is replayed: each step must give the same answer
        e, f, v = ddp.step()
    if a.engine == "b200dp":
        torch.cuda.synchronize()
        compute.engine.check()
    np.savez(a.out, ids=ids, force=f.cpu().numpy(), energy=e.cpu().numpy(), virial=v.cpu().numpy(),
             nghost=ddp.nghost, origin=ddp.plan.origin.cpu().numpy(),
             ghost_ids=ddp.plan.ids[ddp.nloc:].cpu().numpy(), shift=ddp.plan.shift.cpu().numpy(),
             x_owned=ddp.x[: ddp.nloc].cpu().numpy(), x_ghost=ddp.x[ddp.nloc:].cpu().numpy())
    ddp.release()  # the graph holds NCCL calls: release it before the group goes
    dist.barrier()
    if isinstance(fold, SharedMemoryFold):
        fold.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
