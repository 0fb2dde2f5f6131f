"""One rank of the domain-decomposition tests, run as a subprocess.

--engine oracle: the per-rank force call is the CPU oracle in ghost mode, the
  exchange runs over gloo on CPU tensors.
--engine b200dp --backend gloo: the force call is b200dp_compute_device on
  cuda:0 (every rank on the same GPU, each with its own engine; nothing on
  the GPU waits for another rank), the exchange over gloo on CPU tensors.
--engine b200dp --backend nccl: one GPU per rank, exchange over NCCL.
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
    if a.engine == "oracle":
        compute = oracle_compute(a.model)
    else:
        compute = b200dp_compute(a.model, a.precision, device if a.backend == "nccl" else "cuda:0",
                                 staged=a.backend == "gloo")
    ddp = domain.DistributedDeepPot(compute, s.box, a.grid, rank, a.halo, x, t, ids, device=device)
    for _ in range(a.steps):  # the plan is replayed: each step must give the same answer
        e, f, v = ddp.step()
    np.savez(a.out, ids=ids, force=f.cpu().numpy(), energy=e.cpu().numpy(), virial=v.cpu().numpy(),
             nghost=ddp.nghost)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
