"""DeePMD C++ API shim (include/b200dp_deepmd.hpp) driven by a LAMMPS-style stub caller.

The stub (tests/cpp/pair_stub.cpp) includes the shim as deepmd::hpp, hands it a
full neighbour list with ghost atoms and special-bond mask bits exactly as a
DeePMD pair style does, folds ghost forces onto their owners and writes the
result; the GPU test compares it with the periodic evaluation of the same box.
The CPU test only compiles and links the stub.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import b200dp
import systems
from test_oracle import ghost_expand

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "dpa4c-scale-aware-md_b200")


def build_stub(tmp_path):
    exe = str(tmp_path / "pair_stub")
    cmd = ["g++", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include",
           os.path.join(HERE, "cpp", "pair_stub.cpp"), "-o", exe, "-L", PKG, "-lb200dp", "-Wl,-rpath," + PKG,
           "-L", "/usr/local/cuda/lib64", "-lcudart", "-Wl,-rpath,/usr/local/cuda/lib64"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_stub_compiles_against_shim(tmp_path):
    if not os.path.exists(os.path.join(PKG, "libb200dp.so")):
        pytest.skip("library not built")
    assert os.path.exists(build_stub(tmp_path))


@pytest.mark.gpu
def test_stub_caller_matches_periodic(tmp_path, model_dir):
    s = systems.config0()
    coord, atype, owner = ghost_expand(s, 8.0)  # rcut 6 + 2 A skin
    n = s.natoms
    nghost = len(atype) - n
    rng = np.random.default_rng(0)
    d2 = ((coord[:n, None, :] - coord[None, :, :]) ** 2).sum(-1)
    flat, cnt = [], []
    for i in range(n):
        js = np.nonzero((d2[i] < 64.0) & (np.arange(len(atype)) != i))[0]
        js = rng.permutation(js)
        bits = rng.integers(0, 4, size=len(js)) << 30  # special-bond flags above NEIGHMASK
        flat.extend((js | bits).astype(np.int64).astype(np.uint32).view(np.int32))
        cnt.append(len(js))
    inp = tmp_path / "in.bin"
    with open(inp, "wb") as fh:
        np.array([n, nghost, len(flat)], np.int32).tofile(fh)
        coord.astype(np.float64).tofile(fh)
        atype.astype(np.int32).tofile(fh)
        owner.astype(np.int32).tofile(fh)
        np.array(cnt, np.int32).tofile(fh)
        np.array(flat, np.int32).tofile(fh)
    model = str(model_dir / "water.b2dp")
    exe = build_stub(tmp_path)
    out = tmp_path / "out.bin"
    r = subprocess.run([exe, model, str(inp), str(out), "fp64"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    res = np.fromfile(out, np.float64)
    e, f, v = res[0], res[1:1 + 3 * n].reshape(n, 3), res[1 + 3 * n:10 + 3 * n].reshape(3, 3)
    e_at, ae, v_at = res[10 + 3 * n], res[11 + 3 * n:11 + 4 * n], res[11 + 4 * n:20 + 4 * n].reshape(3, 3)
    dp = b200dp.DeepPot(model, precision=b200dp.FP64)
    ref = dp.compute(s.coord, s.atype, s.box, atomic=True)
    scale = np.abs(ref["force"]).max()
    assert abs(e - ref["energy"]) < 1e-10 * abs(ref["energy"])
    assert np.abs(f - ref["force"]).max() < 1e-10 * scale
    assert np.abs(v - ref["virial"]).max() < 1e-10 * np.abs(ref["virial"]).max()
    assert abs(e_at - e) < 1e-10 * abs(e)
    assert np.abs(ae - ref["atom_energy"]).max() < 1e-10 * np.abs(ref["atom_energy"]).max()
    assert np.abs(v_at - v).max() < 1e-10 * np.abs(v).max()
    dp.close()
