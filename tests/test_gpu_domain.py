"""Domain decomposition with the b200dp engine on the GPU.

The force call of every rank is b200dp_compute_device in ghost mode.  The
result must match one periodic evaluation of the whole box by the same engine:
fp64 within 1e-10 relative (only the summation order differs), mixed precision
within the mixed-mode acceptance limits against the fp64 result.  Ranks that
share one GPU exchange over gloo on CPU tensors (each has its own engine and
nothing on the GPU waits for another rank); with two GPUs the exchange runs
over NCCL, one rank per GPU.  The peer fold (reverse exchange replaced by
additions into the owners' accumulators through CUDA IPC) is held to the same
bar, on one GPU (self-exchange; gloo ranks sharing it) and on two.
"""
import numpy as np
import pytest

import b200dp
import domain
import systems
from conftest import TOLERANCES
from test_domain import check, check_origins, run_ranks

pytestmark = pytest.mark.gpu


def periodic(model, mol, precision):
    s = systems.water(*mol, seed=3)
    dp = b200dp.DeepPot(model, precision=precision)
    out = dp.compute(s.coord, s.atype, s.box)
    dp.close()
    return s, out


@pytest.mark.parametrize("precision", [b200dp.FP64, b200dp.MIXED])
def test_self_exchange_on_one_gpu(model_dir, precision):
    """grid 1x1x1 on cuda:0: ghost shell from self-exchange, device tensors end to end."""
    import torch

    model = str(model_dir / "water.b2dp")
    mol = (8, 8, 8)
    s, ref = periodic(model, mol, b200dp.FP64)
    dev = torch.device("cuda:0")
    dp = b200dp.DeepPot(model, precision=precision)
    stream = torch.cuda.current_stream(dev)

    def compute(x_all, t_all, nloc, nghost, region, e, f, v):
        dp.compute_device(stream.cuda_stream, nloc, nghost, x_all.data_ptr(), t_all.data_ptr(), None, region,
                          e.data_ptr(), f.data_ptr(), v.data_ptr())

    dd = domain.Decomposition(s.box, (1, 1, 1), 0, 8.0)
    x, t, ids = domain.distribute(s.coord, s.atype, dd)
    ddp = domain.DistributedDeepPot(compute, s.box, (1, 1, 1), 0, 8.0, x, t, ids, device=dev)
    for _ in range(2):
        e, f, v = ddp.step()
    dp.check()
    part = dict(ids=ids, force=f.cpu().numpy(), energy=e.cpu().numpy(), virial=v.cpu().numpy())
    if precision == b200dp.FP64:
        check(s, ref, [part])
    else:
        fo = np.empty_like(ref["force"])
        fo[ids] = part["force"]
        err = fo - ref["force"]
        assert np.sqrt((err ** 2).mean()) < TOLERANCES["force_rmse"]
        assert np.abs(err).max() < TOLERANCES["force_max"]
        assert abs(float(part["energy"][0]) - ref["energy"]) / s.natoms < TOLERANCES["energy_per_atom"]
    dp.close()


@pytest.mark.parametrize("grid,mol", [((2, 1, 1), (8, 4, 4)), ((2, 2, 1), (8, 8, 4))])
def test_gloo_ranks_sharing_one_gpu(tmp_path, model_dir, grid, mol):
    model = str(model_dir / "water.b2dp")
    s, ref = periodic(model, mol, b200dp.FP64)
    parts = run_ranks(tmp_path, model, mol, grid, 6.0, extra=("--engine", "b200dp", "--backend", "gloo"))
    check(s, ref, parts)


def test_nccl_two_gpus(tmp_path, model_dir):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    model = str(model_dir / "water.b2dp")
    mol = (12, 6, 6)
    s, ref = periodic(model, mol, b200dp.FP64)
    parts = run_ranks(tmp_path, model, mol, (2, 1, 1), 8.0, extra=("--engine", "b200dp", "--backend", "nccl"))
    check(s, ref, parts)


def test_fold_self_exchange_on_one_gpu(model_dir):
    """grid 1x1x1 with the peer fold: every ghost's origin is an owned row of this rank."""
    import torch

    model = str(model_dir / "water.b2dp")
    mol = (8, 8, 8)
    s, ref = periodic(model, mol, b200dp.FP64)
    dev = torch.device("cuda:0")
    dp = b200dp.DeepPot(model, precision=b200dp.FP64)
    dd = domain.Decomposition(s.box, (1, 1, 1), 0, 8.0)
    x, t, ids = domain.distribute(s.coord, s.atype, dd)
    ddp = domain.DistributedDeepPot(None, s.box, (1, 1, 1), 0, 8.0, x, t, ids, device=dev,
                                    fold=domain.PeerFold(dp, dev))
    for _ in range(3):  # the accumulator is cleared by every finish
        e, f, v = ddp.step()
    torch.cuda.synchronize()
    dp.check()
    check(s, ref, [dict(ids=ids, force=f.cpu().numpy(), energy=e.cpu().numpy(), virial=v.cpu().numpy())])
    ddp.capture()
    x2 = ddp.x[: ddp.nloc] + 0.01 * torch.sin(ddp.x[: ddp.nloc])
    ddp.set_positions(x2)
    e2, f2, _ = ddp.step()
    g = ddp.step()[1].clone()
    torch.cuda.synchronize()
    ddp.release()
    ref2 = b200dp.DeepPot(model, precision=b200dp.FP64)
    xs = np.empty_like(s.coord)
    xs[ids] = x2.cpu().numpy()
    r2 = ref2.compute(xs, s.atype, s.box)
    assert abs(float(e2[0]) - r2["energy"]) <= 1e-10 * abs(r2["energy"])
    assert np.abs(g.cpu().numpy() - r2["force"][ids]).max() <= 1e-10 * np.abs(r2["force"]).max()
    ref2.close()
    dp.close()


@pytest.mark.parametrize("grid,mol", [((2, 1, 1), (8, 4, 4)), ((2, 2, 1), (8, 8, 4)), ((2, 2, 2), (8, 8, 8))])
def test_fold_gloo_ranks_sharing_one_gpu(tmp_path, model_dir, grid, mol):
    model = str(model_dir / "water.b2dp")
    s, ref = periodic(model, mol, b200dp.FP64)
    parts = run_ranks(tmp_path, model, mol, grid, 6.0,
                      extra=("--engine", "b200dp", "--backend", "gloo", "--fold"))
    check(s, ref, parts)
    check_origins(parts)


@pytest.mark.parametrize("capture", [False, True])
def test_fold_nccl_two_gpus(tmp_path, model_dir, capture):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    model = str(model_dir / "water.b2dp")
    mol = (12, 6, 6)
    s, ref = periodic(model, mol, b200dp.FP64)
    extra = ("--engine", "b200dp", "--backend", "nccl", "--fold", "--steps", "3") + (("--capture",) if capture else ())
    parts = run_ranks(tmp_path, model, mol, (2, 1, 1), 8.0, extra=extra)
    check(s, ref, parts)
