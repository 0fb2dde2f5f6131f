"""Generates the C8L2 golden fixtures from the reference's own kernels.

    python tests/golden/make_c8l2_golden.py [--out DIR]     (needs a CUDA GPU)

The reference's descriptor forward, node-readout VJP and edge recomputation
(components/deepmd-op/overlays/op/pt/dpa4c/graph_compress_kernel.cuh of the
dpa4c-runtime project) are compiled, unchanged, into
oracle/_ref/libref_c8l2.so by ``make -C oracle ref`` (harness:
oracle/ref_c8l2.cu) and run here on seeded systems with a seeded random-init
C8L2 model.  The fitting net is not part of those kernels, so its gradient
dE/dD is taken from the fp64 oracle and handed to the reference backward
as fp32; the fixture stores it with the reference outputs:

    descriptor [n, 70], state [n, 42], moment cotangents q [n, 42] and
    dE/d(edge vector) [E, 3], all fp32, on the canonical destination-major
    graph (row_ptr, source, fp32 edge vectors) built from the formatted
    neighbour list's kept slots in slot order.

Each fixture records the model recipe (seed) and a SHA-256 of the model file.
"""
from __future__ import annotations

import argparse
import ctypes
import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, os.path.join(ROOT, "dpa4c-scale-aware-md_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, HERE)

import modelgen  # noqa: E402
import oracle  # noqa: E402
import systems  # noqa: E402
from make_golden import sheared_water  # noqa: E402

MODEL_SEED = 0


def graph_of(nl):
    """Canonical destination-major graph of a formatted list's kept slots."""
    nlj = nl["nlist"]
    keep = nlj >= 0
    counts = keep.sum(1)
    row_ptr = np.zeros(len(nlj) + 1, np.int64)
    row_ptr[1:] = np.cumsum(counts)
    source = nlj[keep].astype(np.uint32)
    edge_vec = nl["rij"][keep].astype(np.float32)
    return row_ptr, source, edge_vec, keep


def run_reference(lib, m, atype, row_ptr, source, edge_vec, dD):
    n, E = len(atype), len(source)
    f32 = lambda a: np.ascontiguousarray(a, np.float32)
    out = dict(descriptor=np.zeros((n, 70), np.float32), state=np.zeros((n, 42), np.float32),
               q=np.zeros((n, 42), np.float32), edge_grad=np.zeros((E, 3), np.float32))
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    args = [f32(m.table), f32(m.pair_film), f32(m.type_embedding), f32(m.readout), f32(m.output_mean),
            f32(m.output_inv_std), f32(dD)]
    rc = lib.ref_c8l2_run(ctypes.c_long(n), ctypes.c_long(E), P(np.ascontiguousarray(row_ptr)),
                          P(np.ascontiguousarray(source)), P(np.ascontiguousarray(edge_vec)),
                          P(np.ascontiguousarray(atype, np.int64)), ctypes.c_int(m.ntypes),
                          ctypes.c_int(m.interval_count), ctypes.c_float(m.table_stride),
                          ctypes.c_float(m.table_max), ctypes.c_float(m.rcut), ctypes.c_float(m.eps),
                          ctypes.c_float(m.degree_floor), *[P(a) for a in args], P(out["descriptor"]),
                          P(out["state"]), P(out["q"]), P(out["edge_grad"]))
    if rc != 0:
        raise RuntimeError(f"reference harness returned {rc}")
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_c8l2.so"))
    lib.ref_c8l2_run.restype = ctypes.c_int
    tmp = tempfile.mkdtemp()
    m = modelgen.random_c8_model(seed=MODEL_SEED)
    path = os.path.join(tmp, "c8.b2dp")
    modelgen.save_c8(m, path)
    sha = hashlib.sha256(open(path, "rb").read()).hexdigest()
    orc = oracle.C8Oracle(path)
    for name, s in (("c8l2_water192", systems.config0()), ("c8l2_water192_triclinic", sheared_water())):
        box = s.box.reshape(9)
        nl = oracle.nlist(s.coord, s.atype, box, m.rcut, m.sel)
        row_ptr, source, edge_vec, keep = graph_of(nl)
        # the oracle sees the same fp32-rounded edge vectors
        nl32 = dict(nl)
        nl32["rij"] = np.where(keep[..., None], nl["rij"].astype(np.float32).astype(np.float64), 0.0)
        r = orc.compute(s.coord, s.atype, box, extras=True, nl=nl32)
        ref = run_reference(lib, m, s.atype, row_ptr, source, edge_vec, r["grad_descriptor"])
        np.savez_compressed(os.path.join(args.out, f"{name}.npz"), coord=s.coord, atype=s.atype, box=box,
                            model_seed=MODEL_SEED, model_sha256=sha, row_ptr=row_ptr, source=source,
                            edge_vec=edge_vec, grad_descriptor=r["grad_descriptor"].astype(np.float32),
                            **{f"ref_{k}": v for k, v in ref.items()})
        d = np.abs(ref["descriptor"] - r["descriptor"]).max()
        g = np.abs(ref["edge_grad"] - r["edge_grad"][keep]).max()
        print(f"{name}: nodes {len(s.atype)} edges {len(source)} |d desc| {d:.3e} |d edge grad| {g:.3e}")


if __name__ == "__main__":
    main()
