"""Replay of repeated periodic host calls (b200dp_compute_host).

A periodic call on page-locked host buffers whose atom count, buffers, box and
device buffers repeat is recorded at its second occurrence and replayed as one
CUDA graph (copies in, evaluation, copies out).  Checked against the direct
path, i.e. the same calls made from pageable numpy arrays on a second engine
(never recorded): bitwise-equal energy, forces, virial and per-atom outputs
while the coordinates change between calls, after a box change (recorded
again), after an atom-count change, in both precisions; the kernel-launch
counter advances by the same count for a replayed call as for a direct one.
"""
import ctypes

import numpy as np
import pytest

import b200dp
import systems

pytestmark = pytest.mark.gpu

DP = ctypes.POINTER(ctypes.c_double)
IP = ctypes.POINTER(ctypes.c_int)


class PinnedCall:
    def __init__(self, dp, n, atomic, torch):
        self.dp, self.n, self.atomic = dp, n, atomic
        self.coord = torch.zeros(n, 3, dtype=torch.float64).pin_memory()
        self.atype = torch.zeros(n, dtype=torch.int32).pin_memory()
        self.force = torch.zeros(n, 3, dtype=torch.float64).pin_memory()
        self.ae = torch.zeros(n, dtype=torch.float64).pin_memory() if atomic else None
        self.av = torch.zeros(n, 9, dtype=torch.float64).pin_memory() if atomic else None
        self.e = np.zeros(1)
        self.v = np.zeros(9)

    def __call__(self, coord, atype, box, torch):
        self.coord.copy_(torch.from_numpy(np.ascontiguousarray(coord, dtype=np.float64)))
        self.atype.copy_(torch.from_numpy(np.ascontiguousarray(atype, dtype=np.int32)))
        b = np.ascontiguousarray(box, dtype=np.float64).reshape(9)

        def p(t, ty):
            return None if t is None else ctypes.cast(t.data_ptr(), ty)

        rc = self.dp.L.b200dp_compute_host(self.dp.h, self.n, 0, p(self.coord, DP), p(self.atype, IP),
                                           b.ctypes.data_as(DP), self.e.ctypes.data_as(DP), p(self.force, DP),
                                           self.v.ctypes.data_as(DP), p(self.ae, DP), p(self.av, DP))
        self.dp._raise(rc)
        out = dict(energy=float(self.e[0]), force=self.force.numpy().copy(), virial=self.v.reshape(3, 3).copy())
        if self.atomic:
            out["atom_energy"] = self.ae.numpy().copy()
            out["atom_virial"] = self.av.numpy().copy()
        return out


def same(a, b):
    assert a["energy"] == b["energy"]
    np.testing.assert_array_equal(a["force"], b["force"])
    np.testing.assert_array_equal(a["virial"], b["virial"])
    for k in ("atom_energy", "atom_virial"):
        if k in a:
            np.testing.assert_array_equal(a[k], b[k].reshape(a[k].shape))


@pytest.mark.parametrize("precision", [b200dp.MIXED, b200dp.FP64])
def test_replayed_host_calls_match_direct_calls(model_dir, precision):
    torch = pytest.importorskip("torch")
    model = str(model_dir / "water.b2dp")
    rec = b200dp.DeepPot(model, precision=precision)
    ref = b200dp.DeepPot(model, precision=precision)
    rng = np.random.default_rng(11)
    try:
        for mol, atomic in ((8, False), (6, True)):
            s = systems.water(mol)
            call = PinnedCall(rec, s.natoms, atomic, torch)
            box = s.box.copy()
            per_call = []
            for k in range(6):
                if k == 4:  # a new box (NPT-like): recorded again
                    box = s.box * 1.01
                x = s.coord + rng.uniform(-0.05, 0.05, size=s.coord.shape)
                l0 = b200dp.kernel_launches()
                got = call(x, s.atype, box, torch)
                per_call.append(b200dp.kernel_launches() - l0)
                same(got, ref.compute(x, s.atype, box, atomic=atomic))
            # every call (direct, recording + replay, replays) counts the same launches
            assert len(set(per_call)) == 1 and per_call[0] > 0, per_call
    finally:
        rec.close()
        ref.close()
