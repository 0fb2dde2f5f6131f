"""The device-side rendezvous of the ranks (b200dp_peer_reduce) on one GPU.

With one rank the rendezvous is a plain copy of the rank's values.  With two
ranks whose second one never arrives (this process maps its own exported
buffer for both, so nobody raises rank 1's arrival counter) the wait runs
out after its poll bound: the kernel records the timeout, leaves the output
alone and returns; b200dp_check reports B200DP_ERR_PEER_TIMEOUT once, and the
engine keeps working.  No GPU fault or hang is involved: the wait is bounded
by design and the test only lets that bound expire.
"""
import numpy as np
import pytest

import b200dp
import systems

pytestmark = pytest.mark.gpu


def test_rendezvous_one_rank_and_timeout(model_dir):
    torch = pytest.importorskip("torch")
    dev = torch.device("cuda:0")
    dp = b200dp.DeepPot(str(model_dir / "water.b2dp"), precision=b200dp.FP64)
    h = dp.fold_export(256)
    dp.fold_connect(0, [h])
    stream = torch.cuda.current_stream(dev).cuda_stream
    x = torch.arange(1, 11, dtype=torch.float64, device=dev) * 0.5
    out = torch.full((10,), -1.0, dtype=torch.float64, device=dev)
    for _ in range(3):  # consecutive rendezvous alternate mailboxes
        dp.peer_reduce(stream, 10, x.data_ptr(), out.data_ptr())
        torch.cuda.synchronize()
        assert torch.equal(out, x)
    dp.peer_reduce(stream, 0)  # plain barrier
    dp.check()

    dp.fold_connect(0, [h, h])  # rank 1 never arrives
    out.fill_(-1.0)
    dp.peer_reduce(stream, 10, x.data_ptr(), out.data_ptr(), max_polls=1 << 14)
    torch.cuda.synchronize()
    with pytest.raises(b200dp.B200DPError) as e:
        dp.check()
    assert e.value.status == 8  # B200DP_ERR_PEER_TIMEOUT
    assert torch.all(out == -1.0)
    dp.check()  # reported once

    s = systems.config0()
    r = dp.compute(s.coord, s.atype, s.box)
    ref = b200dp.DeepPot(str(model_dir / "water.b2dp"), precision=b200dp.FP64)
    r2 = ref.compute(s.coord, s.atype, s.box)
    assert r["energy"] == r2["energy"] and np.array_equal(r["force"], r2["force"])
    ref.close()
    dp.close()
