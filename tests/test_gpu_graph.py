"""b200dp_compute_device inside a CUDA graph.

The reference's caller may capture the whole force call into a CUDA graph
(components/deepmd-op/overlays/api_cc/src/DeepPotPTExpt.cc:2941-2951), so the
device entry must make no host synchronisation and keep stable pointers once
its buffers have grown to the system size.  After one eager warm-up call the
call is captured, replayed, and replayed again after the coordinates in the
captured input buffer moved; every replay must equal an eager call on the same
input bit for bit (the pipeline is deterministic).
"""
import numpy as np
import pytest

import b200dp
import systems

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("precision", [b200dp.FP64, b200dp.MIXED])
def test_capture_and_replay(model_dir, precision):
    import torch

    dev = torch.device("cuda:0")
    s = systems.config1() if precision == b200dp.MIXED else systems.config0()
    n = s.natoms
    dp = b200dp.DeepPot(str(model_dir / "water.b2dp"), precision=precision)
    x = torch.tensor(s.coord, device=dev)
    t = torch.tensor(s.atype, device=dev)
    e = torch.zeros(1, dtype=torch.float64, device=dev)
    f = torch.zeros(n, 3, dtype=torch.float64, device=dev)
    v = torch.zeros(9, dtype=torch.float64, device=dev)

    def call():
        dp.compute_device(torch.cuda.current_stream(dev).cuda_stream, n, 0, x.data_ptr(), t.data_ptr(), s.box, None,
                          e.data_ptr(), f.data_ptr(), v.data_ptr())

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        call()  # grows every buffer to this system
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    eager = (e.clone(), f.clone(), v.clone())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        call()
    e.zero_()
    f.zero_()
    g.replay()
    torch.cuda.synchronize()
    dp.check()
    assert torch.equal(e, eager[0]) and torch.equal(f, eager[1]) and torch.equal(v, eager[2])
    # move the atoms inside the captured input buffer, replay, compare with eager
    rng = np.random.default_rng(5)
    x.add_(torch.tensor(rng.normal(0, 0.02, size=(n, 3)), device=dev))
    g.replay()
    torch.cuda.synchronize()
    replayed = (e.clone(), f.clone(), v.clone())
    call()
    torch.cuda.synchronize()
    dp.check()
    assert torch.equal(replayed[0], e) and torch.equal(replayed[1], f) and torch.equal(replayed[2], v)
    assert not torch.equal(replayed[1], eager[1])
    del g
    dp.close()
