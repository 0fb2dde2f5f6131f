"""ctypes binding of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module; the product path never imports it.  Parity status of the SEA model:
unpinned (no reference implementation of the model exists to pin against; see
sea_oracle.cpp).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_dp = ctypes.POINTER(ctypes.c_double)
_ip = ctypes.POINTER(ctypes.c_int)
_lp = ctypes.POINTER(ctypes.c_long)


def build(force: bool = False) -> str:
    path = os.path.join(_HERE, "liboracle.so")
    srcs = [os.path.join(_HERE, s) for s in ("sea_oracle.cpp", "c8l2_oracle.cpp", "Makefile")]
    if force or not os.path.exists(path) or any(os.path.getmtime(path) < os.path.getmtime(s) for s in srcs):
        subprocess.run(["make", "-C", _HERE, "-B" if force else "all"], check=True,
                       stdout=subprocess.DEVNULL)
    return path


def lib():
    global _LIB
    if _LIB is None:
        L = ctypes.CDLL(build())
        L.oracle_load.restype = ctypes.c_void_p
        L.oracle_load.argtypes = [ctypes.c_char_p]
        L.oracle_free.argtypes = [ctypes.c_void_p]
        L.oracle_last_error.restype = ctypes.c_char_p
        L.oracle_set_threads.argtypes = [ctypes.c_int]
        L.oracle_set_threads.restype = ctypes.c_int
        L.oracle_nlist.restype = ctypes.c_long
        L.oracle_nlist.argtypes = [ctypes.c_int, ctypes.c_int, _dp, _ip, _dp, ctypes.c_double, ctypes.c_int,
                                   _ip, _ip, _ip, _dp, _ip]
        L.oracle_compute.restype = ctypes.c_int
        L.oracle_compute.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _dp, _ip, _dp, _dp, _dp, _dp,
                                     _dp, _dp, _dp, _dp, _lp]
        L.c8_load.restype = ctypes.c_void_p
        L.c8_load.argtypes = [ctypes.c_char_p]
        L.c8_free.argtypes = [ctypes.c_void_p]
        L.c8_last_error.restype = ctypes.c_char_p
        L.c8_compute.restype = ctypes.c_int
        L.c8_compute.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _ip, _dp, _ip] + [_dp] * 10
        _LIB = L
    return _LIB


def _p(a, t):
    return None if a is None else a.ctypes.data_as(t)


def set_threads(n: int) -> int:
    return lib().oracle_set_threads(int(n))


def nlist(coord, atype, box, rcut, sel, nloc=None):
    coord = np.ascontiguousarray(coord, dtype=np.float64).reshape(-1, 3)
    atype = np.ascontiguousarray(atype, dtype=np.int32)
    nall = coord.shape[0]
    nloc = nall if nloc is None else nloc
    sel = np.ascontiguousarray(sel, dtype=np.int32)
    selt = int(sel.sum())
    nl = np.empty((nloc, selt), np.int32)
    code = np.empty((nloc, selt), np.int32)
    rij = np.empty((nloc, selt, 3), np.float64)
    cnt = np.empty((nloc, len(sel)), np.int32)
    b = None if box is None else np.ascontiguousarray(box, dtype=np.float64).reshape(9)
    ov = lib().oracle_nlist(nloc, nall, _p(coord, _dp), _p(atype, _ip), _p(b, _dp), float(rcut), len(sel),
                            _p(sel, _ip), _p(nl, _ip), _p(code, _ip), _p(rij, _dp), _p(cnt, _ip))
    return dict(nlist=nl, code=code, rij=rij, counts=cnt, overflow=int(ov))


class Oracle:
    def __init__(self, model_path: str):
        self.h = lib().oracle_load(model_path.encode())
        if not self.h:
            raise RuntimeError(lib().oracle_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_free(self.h)
            self.h = None

    def compute(self, coord, atype, box, nloc=None, descriptor_dim=None, atomic=True):
        coord = np.ascontiguousarray(coord, dtype=np.float64).reshape(-1, 3)
        atype = np.ascontiguousarray(atype, dtype=np.int32)
        nall = coord.shape[0]
        nloc = nall if nloc is None else nloc
        b = None if box is None else np.ascontiguousarray(box, dtype=np.float64).reshape(9)
        e = np.zeros(1)
        f = np.zeros((nall, 3))
        v = np.zeros(9)
        ae = np.zeros(nloc) if atomic else None
        av = np.zeros((nall, 9)) if atomic else None
        d = dd = None
        if descriptor_dim:
            d = np.zeros((nloc, descriptor_dim))
            dd = np.zeros((nloc, descriptor_dim))
        ov = ctypes.c_long(0)
        rc = lib().oracle_compute(self.h, nloc, nall, _p(coord, _dp), _p(atype, _ip), _p(b, _dp), _p(e, _dp),
                                  _p(f, _dp), _p(v, _dp), _p(ae, _dp), _p(av, _dp), _p(d, _dp), _p(dd, _dp),
                                  ctypes.byref(ov))
        if rc != 0:
            raise RuntimeError("oracle_compute failed")
        out = dict(energy=float(e[0]), force=f, virial=v.reshape(3, 3), overflow=int(ov.value))
        if atomic:
            out["atom_energy"] = ae
            out["atom_virial"] = av
        if descriptor_dim:
            out["descriptor"] = d
            out["grad_descriptor"] = dd
        return out


def c8_header(model_path: str):
    """(ntypes, sel, rcut) of a B2DPC8L2 model file."""
    import struct

    with open(model_path, "rb") as f:
        data = f.read()
    if data[:8] != b"B2DPC8L2":
        raise ValueError(f"{model_path}: not a C8L2 model")
    version, ntypes, ch, lmax, nint, width, nfit = struct.unpack_from("<7i", data, 8)
    off = 8 + 28 + 8 * nfit
    (act,) = struct.unpack_from("<i", data, off)
    off += 4
    sel = list(struct.unpack_from(f"<{ntypes}i", data, off))
    off += 4 * ntypes
    stride, tmax, rcut = struct.unpack_from("<3d", data, off)
    return ntypes, sel, rcut


class C8Oracle:
    """fp64 restatement of the reference's C8L2 descriptor, fitting and force
    path (c8l2_oracle.cpp) on this framework's formatted neighbour list."""

    def __init__(self, model_path: str):
        self.ntypes, self.sel, self.rcut = c8_header(model_path)
        self.h = lib().c8_load(model_path.encode())
        if not self.h:
            raise RuntimeError(lib().c8_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            lib().c8_free(self.h)
            self.h = None

    def compute(self, coord, atype, box, nloc=None, extras=False, nl=None):
        coord = np.ascontiguousarray(coord, dtype=np.float64).reshape(-1, 3)
        atype = np.ascontiguousarray(atype, dtype=np.int32)
        nall = coord.shape[0]
        nloc = nall if nloc is None else nloc
        if nl is None:
            nl = nlist(coord, atype, box, self.rcut, self.sel, nloc)
        nlj = np.ascontiguousarray(nl["nlist"], dtype=np.int32)
        rij = np.ascontiguousarray(nl["rij"], dtype=np.float64)
        selt = nlj.shape[1]
        e = np.zeros(1)
        f = np.zeros((nall, 3))
        v = np.zeros(9)
        ae = np.zeros(nloc)
        av = np.zeros((nall, 9))
        x = {}
        if extras:
            x = dict(descriptor=np.zeros((nloc, 70)), state=np.zeros((nloc, 42)),
                     grad_descriptor=np.zeros((nloc, 70)), q=np.zeros((nloc, 42)),
                     edge_grad=np.zeros((nloc, selt, 3)))
        rc = lib().c8_compute(self.h, nloc, nall, selt, _p(nlj, _ip), _p(rij, _dp), _p(atype, _ip), _p(e, _dp),
                              _p(f, _dp), _p(v, _dp), _p(ae, _dp), _p(av, _dp), _p(x.get("descriptor"), _dp),
                              _p(x.get("state"), _dp), _p(x.get("grad_descriptor"), _dp), _p(x.get("q"), _dp),
                              _p(x.get("edge_grad"), _dp))
        if rc != 0:
            raise RuntimeError(lib().c8_last_error().decode())
        out = dict(energy=float(e[0]), force=f, virial=v.reshape(3, 3), atom_energy=ae, atom_virial=av,
                   overflow=int(nl["overflow"]), nlist=nl)
        out.update(x)
        return out
