"""Python binding of the b200dp C ABI (include/b200dp.h) over ctypes.

Mirrors DeePMD's ``DeepPot`` surface for this path: ``DeepPot(model).compute
(coord, atype, box)`` returns energy, forces and virial (plus atomic terms),
and ``compute(..., nghost=...)`` follows the LAMMPS ghost-atom convention of
``DeepPot::compute(..., nghost, lmp_list, ago)``
(components/deepmd-op/overlays/api_cc/include/DeepPot.h:605-690 in the
reference).  Errors are raised as ``B200DPError`` carrying the C status.

The shared library is the only compute path: there is no CPU fallback, and a
missing or unloadable ``libb200dp.so`` raises at import of the engine.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb200dp.so")

FP64 = 0
MIXED = 1

STATUS = {0: "OK", 1: "INVALID", 2: "IO", 3: "CUDA", 4: "SEL_OVERFLOW", 5: "CAPACITY", 6: "BAD_TYPE",
          7: "UNSUPPORTED"}

EXPORTS = [
    "b200dp_options_default", "b200dp_create", "b200dp_destroy", "b200dp_last_error", "b200dp_model_info_get",
    "b200dp_engine_device", "b200dp_compute_host", "b200dp_compute_host_nlist", "b200dp_compute_device", "b200dp_check",
    "b200dp_sel_overflow_count", "b200dp_last_nlist", "b200dp_last_descriptor", "b200dp_set_stage_timing",
    "b200dp_set_neighbor_reuse", "b200dp_neighbor_stats", "b200dp_fold_export", "b200dp_fold_connect", "b200dp_fold_origins",
    "b200dp_compute_device_fold", "b200dp_fold_finish", "b200dp_halo_publish", "b200dp_halo_gather",
    "b200dp_peer_reduce", "b200dp_fold_scale_shifts", "b200dp_compute_device_dbox",
    "b200dp_stage_times", "b200dp_kernel_launches", "b200dp_selftest_mma", "b200dp_build_nlist_noalloc",
    "b200dp_direct_bind", "b200dp_direct_energy_force", "b200dp_direct_destination_only_ready",
    "b200dp_bind_direct_neighbor_view", "b200dp_get_direct_neighbor_view", "b200dp_direct_set_need_virial",
    "b200dp_direct_fp32_global_virial_pointer", "b200dp_md_params_default", "b200dp_md_create",
    "b200dp_md_run", "b200dp_md_thermo", "b200dp_md_state", "b200dp_md_destroy", "b200dp_md_snapshot_bytes",
    "b200dp_md_snapshot", "b200dp_md_restore", "b200dp_md_write_restart", "b200dp_md_read_restart",
    "b200dp_dd_params_default", "b200dp_dd_unique_id", "b200dp_dd_create", "b200dp_dd_destroy",
    "b200dp_dd_last_error", "b200dp_dd_stream", "b200dp_dd_counts", "b200dp_dd_force", "b200dp_dd_result",
    "b200dp_dd_owned", "b200dp_dd_set_positions", "b200dp_dd_get_forces", "b200dp_dd_md_start", "b200dp_dd_md_run",
    "b200dp_dd_md_thermo", "b200dp_dd_plan_emulate",
]

NVE, NVT, NPT = 0, 1, 2


class MDParams(ctypes.Structure):
    _fields_ = [("dt", ctypes.c_double), ("ensemble", ctypes.c_int), ("chain", ctypes.c_int),
                ("t_target", ctypes.c_double), ("t_damp", ctypes.c_double), ("t_init", ctypes.c_double),
                ("seed", ctypes.c_ulonglong), ("mass", ctypes.c_double * 8), ("p_target", ctypes.c_double),
                ("p_damp", ctypes.c_double), ("pchain", ctypes.c_int), ("rebuild_every", ctypes.c_int),
                ("skin", ctypes.c_double), ("reserved", ctypes.c_int * 8)]


class DDParams(ctypes.Structure):
    _fields_ = [("grid", ctypes.c_int * 3), ("halo", ctypes.c_double), ("max_polls", ctypes.c_longlong),
                ("capacity", ctypes.c_int), ("reserved", ctypes.c_int * 9)]


class NeighborView(ctypes.Structure):
    """b200dp_neighbor_view (the layout of the reference's DpaDirectNeighborView)."""
    _fields_ = [("x", ctypes.c_void_p), ("model_to_atom", ctypes.c_void_p), ("candidate_atom", ctypes.c_void_p),
                ("source", ctypes.c_void_p), ("stride_atom", ctypes.c_int64), ("stride_xyz", ctypes.c_int64),
                ("node_count", ctypes.c_int64), ("cutoff_squared", ctypes.c_double),
                ("inverse_distance_unit", ctypes.c_double)]


class B200DPError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"b200dp status {STATUS.get(status, status)}: {msg}")
        self.status = status


class Options(ctypes.Structure):
    _fields_ = [("precision", ctypes.c_int), ("device", ctypes.c_int), ("sel_overflow_is_error", ctypes.c_int),
                ("simt_only", ctypes.c_int), ("keep_descriptor", ctypes.c_int), ("reserved", ctypes.c_int * 11)]


class ModelInfo(ctypes.Structure):
    _fields_ = [("ntypes", ctypes.c_int), ("sel_total", ctypes.c_int), ("descriptor_dim", ctypes.c_int),
                ("embedding_out", ctypes.c_int), ("axis", ctypes.c_int), ("n_embedding_layers", ctypes.c_int),
                ("n_fitting_layers", ctypes.c_int), ("type_one_side", ctypes.c_int), ("rcut", ctypes.c_double),
                ("rcut_smth", ctypes.c_double)]


class NList(ctypes.Structure):
    _fields_ = [("inum", ctypes.c_int), ("ilist", ctypes.POINTER(ctypes.c_int)),
                ("numneigh", ctypes.POINTER(ctypes.c_int)),
                ("firstneigh", ctypes.POINTER(ctypes.POINTER(ctypes.c_int)))]


_dp = ctypes.POINTER(ctypes.c_double)
_ip = ctypes.POINTER(ctypes.c_int)
_vp = ctypes.c_void_p
_L = None


def load_library(path: str = LIB_PATH):
    """Loads libb200dp.so (raises OSError if it is missing)."""
    global _L
    if _L is not None:
        return _L
    if not os.path.exists(path):
        raise OSError(f"{path} not built; run dpa4c-scale-aware-md_b200/build.py")
    L = ctypes.CDLL(path)
    L.b200dp_options_default.argtypes = [ctypes.POINTER(Options)]
    L.b200dp_create.argtypes = [ctypes.c_char_p, ctypes.POINTER(Options), ctypes.POINTER(_vp)]
    L.b200dp_create.restype = ctypes.c_int
    L.b200dp_destroy.argtypes = [_vp]
    L.b200dp_last_error.argtypes = [_vp]
    L.b200dp_last_error.restype = ctypes.c_char_p
    L.b200dp_model_info_get.argtypes = [_vp, ctypes.POINTER(ModelInfo)]
    L.b200dp_compute_host.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _dp, _ip, _dp, _dp, _dp, _dp, _dp, _dp]
    L.b200dp_compute_host_nlist.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _dp, _ip, ctypes.POINTER(NList), _dp,
                                            _dp, _dp, _dp, _dp]
    L.b200dp_compute_device.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _dp, _dp, _vp, _vp, _vp,
                                        _vp, _vp]
    L.b200dp_check.argtypes = [_vp]
    L.b200dp_sel_overflow_count.argtypes = [_vp]
    L.b200dp_sel_overflow_count.restype = ctypes.c_longlong
    L.b200dp_last_nlist.argtypes = [_vp, _ip, _ip, _dp]
    L.b200dp_last_descriptor.argtypes = [_vp, _dp, _dp]
    L.b200dp_set_stage_timing.argtypes = [_vp, ctypes.c_int]
    L.b200dp_set_neighbor_reuse.argtypes = [_vp, ctypes.c_double, ctypes.c_int]
    L.b200dp_neighbor_stats.argtypes = [_vp, ctypes.POINTER(ctypes.c_longlong)]
    L.b200dp_fold_export.argtypes = [_vp, ctypes.c_int, _vp]
    L.b200dp_fold_connect.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp]
    L.b200dp_fold_origins.argtypes = [_vp, ctypes.c_int, _vp, _vp]
    L.b200dp_halo_publish.argtypes = [_vp, _vp, ctypes.c_int, _vp]
    L.b200dp_halo_gather.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]
    L.b200dp_compute_device_fold.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _dp, _vp, _vp, _vp]
    L.b200dp_fold_finish.argtypes = [_vp, _vp, ctypes.c_int, _vp]
    L.b200dp_peer_reduce.argtypes = [_vp, _vp, ctypes.c_int, _vp, _vp, ctypes.c_longlong]
    L.b200dp_stage_times.argtypes = [_vp, ctypes.POINTER(ctypes.c_float)]
    L.b200dp_selftest_mma.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float),
                                      ctypes.POINTER(ctypes.c_float)]
    L.b200dp_build_nlist_noalloc.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _dp, _dp, ctypes.c_double,
                                             ctypes.c_int, _ip, _vp, _vp, _vp, ctypes.POINTER(ctypes.c_longlong)]
    L.b200dp_kernel_launches.argtypes = []
    L.b200dp_kernel_launches.restype = ctypes.c_longlong
    L.b200dp_direct_bind.argtypes = [_vp, _vp]
    L.b200dp_md_create.argtypes = [_vp, ctypes.c_int, _dp, _dp, _ip, _dp, ctypes.c_void_p, ctypes.POINTER(_vp)]
    L.b200dp_md_run.argtypes = [_vp, ctypes.c_int]
    L.b200dp_md_thermo.argtypes = [_vp, _dp]
    L.b200dp_md_state.argtypes = [_vp, _dp, _dp, _dp]
    L.b200dp_md_destroy.argtypes = [_vp]
    _lp = ctypes.POINTER(ctypes.c_longlong)
    L.b200dp_dd_params_default.argtypes = [ctypes.POINTER(DDParams)]
    L.b200dp_dd_params_default.restype = None
    L.b200dp_dd_unique_id.argtypes = [_vp]
    L.b200dp_dd_create.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _dp, ctypes.POINTER(DDParams), ctypes.c_int,
                                   _dp, _ip, ctypes.POINTER(_vp)]
    L.b200dp_dd_destroy.argtypes = [_vp]
    L.b200dp_dd_destroy.restype = None
    L.b200dp_dd_last_error.argtypes = [_vp]
    L.b200dp_dd_last_error.restype = ctypes.c_char_p
    L.b200dp_dd_stream.argtypes = [_vp]
    L.b200dp_dd_stream.restype = _vp
    L.b200dp_dd_counts.argtypes = [_vp, _ip, _ip]
    L.b200dp_dd_force.argtypes = [_vp, _vp]
    L.b200dp_dd_result.argtypes = [_vp, _vp, _dp, _dp]
    L.b200dp_dd_owned.argtypes = [_vp, _lp, _dp, _dp, _dp]
    L.b200dp_dd_set_positions.argtypes = [_vp, _vp, _vp]
    L.b200dp_dd_get_forces.argtypes = [_vp, _vp, _vp, _vp]
    L.b200dp_dd_md_start.argtypes = [_vp, ctypes.POINTER(MDParams), _dp]
    L.b200dp_dd_md_run.argtypes = [_vp, ctypes.c_int]
    L.b200dp_dd_md_thermo.argtypes = [_vp, _dp]
    L.b200dp_dd_plan_emulate.argtypes = [ctypes.c_int, _ip, _dp, ctypes.c_double, ctypes.c_int, _dp, _dp, _lp, _ip,
                                         _lp, _dp, _dp, _ip, _ip, ctypes.c_int]
    L.b200dp_md_snapshot_bytes.argtypes = [_vp, ctypes.POINTER(ctypes.c_size_t)]
    L.b200dp_md_snapshot.argtypes = [_vp, _vp]
    L.b200dp_md_restore.argtypes = [_vp, _vp]
    L.b200dp_md_write_restart.argtypes = [_vp, ctypes.c_char_p]
    L.b200dp_md_read_restart.argtypes = [_vp, ctypes.c_char_p]
    L.b200dp_direct_destination_only_ready.restype = ctypes.c_int
    L.b200dp_direct_destination_only_ready.argtypes = [ctypes.c_int64, ctypes.c_int64]
    L.b200dp_bind_direct_neighbor_view.argtypes = [ctypes.POINTER(NeighborView)]
    L.b200dp_bind_direct_neighbor_view.restype = None
    L.b200dp_get_direct_neighbor_view.argtypes = []
    L.b200dp_get_direct_neighbor_view.restype = NeighborView
    L.b200dp_direct_set_need_virial.argtypes = [ctypes.c_int, _vp]
    L.b200dp_direct_set_need_virial.restype = None
    L.b200dp_direct_fp32_global_virial_pointer.argtypes = []
    L.b200dp_direct_fp32_global_virial_pointer.restype = ctypes.c_void_p
    L.b200dp_direct_energy_force.restype = ctypes.c_int
    L.b200dp_direct_energy_force.argtypes = [_vp, _vp, _vp, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                             _vp, _vp, _vp]
    for name in EXPORTS:
        getattr(L, name)  # every declared symbol must resolve
    _L = L
    return L


def _p(a, t):
    return None if a is None else a.ctypes.data_as(t)


class DeepPot:
    """One engine = one model on one device with one precision."""

    def __init__(self, model_path: str, precision: int = MIXED, device: int = 0, sel_overflow_is_error: bool = False,
                 simt_only: bool = False, keep_descriptor: bool = False):
        L = load_library()
        o = Options()
        L.b200dp_options_default(ctypes.byref(o))
        o.precision = precision
        o.device = device
        o.sel_overflow_is_error = int(sel_overflow_is_error)
        o.simt_only = int(simt_only)
        o.keep_descriptor = int(keep_descriptor)
        h = _vp()
        rc = L.b200dp_create(model_path.encode(), ctypes.byref(o), ctypes.byref(h))
        if rc != 0:
            raise B200DPError(rc, f"cannot create engine for {model_path}")
        self.h = h
        self.L = L
        info = ModelInfo()
        L.b200dp_model_info_get(h, ctypes.byref(info))
        self.info = info

    def close(self):
        if getattr(self, "h", None):
            self.L.b200dp_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _raise(self, rc):
        if rc != 0:
            raise B200DPError(rc, self.L.b200dp_last_error(self.h).decode())

    def compute(self, coord, atype, box=None, nghost: int = 0, atomic: bool = False, nlist=None):
        """Energy, force [nall,3], virial [3,3] (+ atom_energy, atom_virial)."""
        coord = np.ascontiguousarray(coord, dtype=np.float64).reshape(-1, 3)
        atype = np.ascontiguousarray(atype, dtype=np.int32)
        nall = coord.shape[0]
        nloc = nall - nghost
        b = None if box is None else np.ascontiguousarray(box, dtype=np.float64).reshape(9)
        e = np.zeros(1)
        f = np.zeros((nall, 3))
        v = np.zeros(9)
        ae = np.zeros(nloc) if atomic else None
        av = np.zeros((nall, 9)) if atomic else None
        if nlist is None:
            rc = self.L.b200dp_compute_host(self.h, nloc, nghost, _p(coord, _dp), _p(atype, _ip), _p(b, _dp),
                                            _p(e, _dp), _p(f, _dp), _p(v, _dp), _p(ae, _dp), _p(av, _dp))
        else:
            nl, keep = _make_nlist(nlist)
            rc = self.L.b200dp_compute_host_nlist(self.h, nloc, nghost, _p(coord, _dp), _p(atype, _ip),
                                                  ctypes.byref(nl), _p(e, _dp), _p(f, _dp), _p(v, _dp),
                                                  _p(ae, _dp), _p(av, _dp))
        self._raise(rc)
        out = dict(energy=float(e[0]), force=f, virial=v.reshape(3, 3))
        if atomic:
            out["atom_energy"] = ae
            out["atom_virial"] = av
        return out

    def compute_device(self, stream: int, nloc: int, nghost: int, coord_ptr: int, atype_ptr: int, box, region,
                       energy_ptr: int, force_ptr: int, virial_ptr: int, atom_energy_ptr: int = 0,
                       atom_virial_ptr: int = 0):
        b = None if box is None else np.ascontiguousarray(box, dtype=np.float64).reshape(9)
        r = None if region is None else np.ascontiguousarray(region, dtype=np.float64).reshape(6)
        rc = self.L.b200dp_compute_device(self.h, stream or None, nloc, nghost, coord_ptr, atype_ptr, _p(b, _dp),
                                          _p(r, _dp), energy_ptr, force_ptr, virial_ptr, atom_energy_ptr or None,
                                          atom_virial_ptr or None)
        self._raise(rc)

    def check(self):
        self._raise(self.L.b200dp_check(self.h))

    def sel_overflow_count(self) -> int:
        return int(self.L.b200dp_sel_overflow_count(self.h))

    def last_nlist(self, nloc: int):
        selt = self.info.sel_total
        nl = np.empty((nloc, selt), np.int32)
        code = np.empty((nloc, selt), np.int32)
        rij = np.empty((nloc, selt, 3))
        self._raise(self.L.b200dp_last_nlist(self.h, _p(nl, _ip), _p(code, _ip), _p(rij, _dp)))
        return dict(nlist=nl, code=code, rij=rij)

    def last_descriptor(self, nloc: int):
        d = np.empty((nloc, self.info.descriptor_dim))
        dd = np.empty_like(d)
        self._raise(self.L.b200dp_last_descriptor(self.h, _p(d, _dp), _p(dd, _dp)))
        return d, dd

    def set_neighbor_reuse(self, skin: float, every: int):
        """Periodic calls reuse rcut + skin candidates, built at least every `every` calls and
        whenever an atom moved more than skin / 2 (0: off)."""
        self._raise(self.L.b200dp_set_neighbor_reuse(self.h, float(skin), int(every)))

    # peer fold (domain decomposition over NVLink peers; see domain.PeerFold)
    def fold_export(self, capacity: int) -> bytes:
        """Allocates the owned-atom accumulator; returns its 64-byte CUDA IPC handle."""
        h = ctypes.create_string_buffer(64)
        self._raise(self.L.b200dp_fold_export(self.h, int(capacity), h))
        return h.raw

    def fold_connect(self, rank: int, handles) -> None:
        buf = b"".join(bytes(h) for h in handles)
        if len(buf) != 64 * len(handles):
            raise ValueError("every handle is 64 bytes")
        cbuf = ctypes.create_string_buffer(buf, len(buf))
        self._raise(self.L.b200dp_fold_connect(self.h, len(handles), int(rank), cbuf))

    def fold_origins(self, nghost: int, origin_ptr: int, shift_ptr: int = 0) -> None:
        self._raise(self.L.b200dp_fold_origins(self.h, int(nghost), origin_ptr or None, shift_ptr or None))

    def halo_publish(self, stream: int, nloc: int, coord_ptr: int) -> None:
        self._raise(self.L.b200dp_halo_publish(self.h, stream or None, int(nloc), coord_ptr))

    def halo_gather(self, stream: int, nloc: int, nghost: int, coord_ptr: int) -> None:
        self._raise(self.L.b200dp_halo_gather(self.h, stream or None, int(nloc), int(nghost), coord_ptr))

    def compute_device_fold(self, stream: int, nloc: int, nghost: int, coord_ptr: int, atype_ptr: int, region,
                            energy_ptr: int, force_ptr: int, virial_ptr: int):
        r = np.ascontiguousarray(region, dtype=np.float64).reshape(6)
        self._raise(self.L.b200dp_compute_device_fold(self.h, stream or None, nloc, nghost, coord_ptr, atype_ptr,
                                                      _p(r, _dp), energy_ptr, force_ptr, virial_ptr))

    def fold_finish(self, stream: int, nloc: int, force_ptr: int) -> None:
        self._raise(self.L.b200dp_fold_finish(self.h, stream or None, int(nloc), force_ptr))

    def peer_reduce(self, stream: int, nv: int, in_ptr: int = 0, out_ptr: int = 0, max_polls: int = 0) -> None:
        """Device-side rendezvous of the ranks (sum of nv doubles in rank order, or a barrier for nv = 0)."""
        self._raise(self.L.b200dp_peer_reduce(self.h, stream or None, int(nv), in_ptr or None, out_ptr or None,
                                              int(max_polls)))

    def neighbor_stats(self) -> dict:
        """Candidate builds so far: scheduled and triggered by the displacement check."""
        b = (ctypes.c_longlong * 2)()
        self._raise(self.L.b200dp_neighbor_stats(self.h, b))
        return {"scheduled": int(b[0]), "triggered": int(b[1])}

    def set_stage_timing(self, on: bool):
        self._raise(self.L.b200dp_set_stage_timing(self.h, int(on)))

    def stage_times(self):
        ms = (ctypes.c_float * 5)()
        self._raise(self.L.b200dp_stage_times(self.h, ms))
        return list(ms)


def selftest_mma(A, B, passes=3, a_mn_major=False, b_mn_major=False):
    """C = A @ B.T on the tensor cores (bf16 split, 1 or 3 products); A [128,K], B [N,K]."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    K = A.shape[1]
    N = B.shape[0]
    C = np.zeros((128, N), np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    rc = load_library().b200dp_selftest_mma(K, N, int(a_mn_major), int(b_mn_major), passes, A.ctypes.data_as(fp),
                                            B.ctypes.data_as(fp), C.ctypes.data_as(fp))
    if rc != 0:
        raise B200DPError(rc, "tcgen05 self-test failed")
    return C


class MD:
    """Device-resident MD driver (velocity Verlet, optional Nose-Hoover chain) around a DeepPot engine."""

    THERMO = ("step", "pe", "ke", "temp", "conserved", "press", "volume", "e_thermostat")

    def __init__(self, dp: DeepPot, coord, atype, box, masses, dt=0.0005, ensemble=NVE, vel=None, t_init=0.0,
                 t_target=300.0, t_damp=0.05, chain=3, seed=0, p_target=1.0, p_damp=0.5, pchain=3, skin=2.0,
                 rebuild_every=10):
        L = load_library()
        p = MDParams()
        L.b200dp_md_params_default(ctypes.byref(p))
        p.dt, p.ensemble, p.chain = dt, ensemble, chain
        p.t_target, p.t_damp, p.t_init, p.seed = t_target, t_damp, t_init, seed
        p.p_target, p.p_damp, p.pchain = p_target, p_damp, pchain
        p.skin, p.rebuild_every = skin, rebuild_every
        for t, m in enumerate(masses):
            p.mass[t] = m
        coord = np.ascontiguousarray(coord, dtype=np.float64).reshape(-1, 3)
        atype = np.ascontiguousarray(atype, dtype=np.int32)
        box = np.ascontiguousarray(box, dtype=np.float64).reshape(9)
        v = None if vel is None else np.ascontiguousarray(vel, dtype=np.float64).reshape(-1, 3)
        self.n = coord.shape[0]
        self.L = L
        self.dp = dp
        h = _vp()
        rc = L.b200dp_md_create(dp.h, self.n, _p(coord, _dp), _p(v, _dp), _p(atype, _ip), _p(box, _dp),
                                ctypes.byref(p), ctypes.byref(h))
        if rc != 0:
            raise B200DPError(rc, dp.L.b200dp_last_error(dp.h).decode())
        self.h = h

    def run(self, nsteps: int):
        rc = self.L.b200dp_md_run(self.h, int(nsteps))
        if rc != 0:
            raise B200DPError(rc, self.dp.L.b200dp_last_error(self.dp.h).decode())

    def thermo(self) -> dict:
        t = np.zeros(8)
        rc = self.L.b200dp_md_thermo(self.h, _p(t, _dp))
        if rc != 0:
            raise B200DPError(rc, self.dp.L.b200dp_last_error(self.dp.h).decode())
        return dict(zip(self.THERMO, t))

    def state(self):
        x, v, f = (np.zeros((self.n, 3)) for _ in range(3))
        rc = self.L.b200dp_md_state(self.h, _p(x, _dp), _p(v, _dp), _p(f, _dp))
        if rc != 0:
            raise B200DPError(rc, self.dp.L.b200dp_last_error(self.dp.h).decode())
        return x, v, f

    def _check(self, rc):
        if rc != 0:
            raise B200DPError(rc, self.dp.L.b200dp_last_error(self.dp.h).decode())

    def snapshot_bytes(self) -> int:
        n = ctypes.c_size_t()
        self._check(self.L.b200dp_md_snapshot_bytes(self.h, ctypes.byref(n)))
        return int(n.value)

    def snapshot(self, buf_ptr: int) -> None:
        """Enqueues a copy of the whole integrator state into device memory at buf_ptr."""
        self._check(self.L.b200dp_md_snapshot(self.h, buf_ptr))

    def restore(self, buf_ptr: int) -> None:
        self._check(self.L.b200dp_md_restore(self.h, buf_ptr))

    def write_restart(self, path: str) -> None:
        self._check(self.L.b200dp_md_write_restart(self.h, os.fsencode(path)))

    def read_restart(self, path: str) -> None:
        self._check(self.L.b200dp_md_read_restart(self.h, os.fsencode(path)))

    def close(self):
        if getattr(self, "h", None):
            self.L.b200dp_md_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def direct_bind(engine, stream: int = 0):
    """Binds `engine` (a DeepPot, or None) and a CUDA stream to direct_energy_force."""
    load_library().b200dp_direct_bind(engine.h if engine is not None else None, stream or None)


def direct_energy_force(atype_ptr, row_ptr_ptr, source_ptr, edge_vec_ptr, node_count, nloc, edge_storage,
                        energy_ptr, force_ptr, virial_ptr) -> int:
    """dpa_direct_energy_force on device pointers: 1 = handled, 0 = caller must fall back."""
    return int(load_library().b200dp_direct_energy_force(atype_ptr or None, row_ptr_ptr or None, source_ptr or None,
                                                         edge_vec_ptr or None, node_count, nloc, edge_storage,
                                                         energy_ptr or None, force_ptr or None, virial_ptr or None))


def direct_destination_only_ready(node_count: int, nloc: int) -> int:
    return int(load_library().b200dp_direct_destination_only_ready(node_count, nloc))


def bind_direct_neighbor_view(x_ptr=0, model_to_atom_ptr=0, candidate_atom_ptr=0, source_ptr=0, stride_atom=3,
                              stride_xyz=1, node_count=0, cutoff_squared=0.0, inverse_distance_unit=1.0) -> None:
    """Binds the raw-neighbour view (x_ptr = 0 unbinds)."""
    L = load_library()
    if not x_ptr:
        L.b200dp_bind_direct_neighbor_view(None)
        return
    v = NeighborView(x_ptr, model_to_atom_ptr, candidate_atom_ptr, source_ptr, stride_atom, stride_xyz, node_count,
                     cutoff_squared, inverse_distance_unit)
    L.b200dp_bind_direct_neighbor_view(ctypes.byref(v))


def get_direct_neighbor_view() -> NeighborView:
    return load_library().b200dp_get_direct_neighbor_view()


def direct_set_need_virial(need_virial: int, stream: int = 0) -> None:
    load_library().b200dp_direct_set_need_virial(int(need_virial), stream or None)


def direct_fp32_global_virial_pointer() -> int:
    return int(load_library().b200dp_direct_fp32_global_virial_pointer() or 0)


def dd_unique_id() -> bytes:
    """128 bytes identifying one group of ranks (made by rank 0, handed to all)."""
    L = load_library()
    buf = ctypes.create_string_buffer(128)
    rc = L.b200dp_dd_unique_id(buf)
    if rc != 0:
        raise B200DPError(rc, "ncclGetUniqueId failed")
    return buf.raw


class DD:
    """Domain-decomposed force evaluation and MD (b200dp_dd_*), one process per GPU.

    Every rank passes the whole system; the rank keeps the atoms of its sub-box."""

    THERMO = MD.THERMO

    def __init__(self, dp: DeepPot, uid: bytes, nranks: int, rank: int, coord, atype, box, grid, halo=8.0,
                 max_polls=0, capacity=0):
        L = load_library()
        p = DDParams()
        L.b200dp_dd_params_default(ctypes.byref(p))
        for k in range(3):
            p.grid[k] = int(grid[k])
        p.halo, p.max_polls, p.capacity = float(halo), int(max_polls), int(capacity)
        coord = np.ascontiguousarray(coord, dtype=np.float64).reshape(-1, 3)
        atype = np.ascontiguousarray(atype, dtype=np.int32)
        box = np.ascontiguousarray(box, dtype=np.float64).reshape(9)
        self.natoms = coord.shape[0]
        self.L, self.dp = L, dp
        h = _vp()
        idb = ctypes.create_string_buffer(bytes(uid), 128)
        rc = L.b200dp_dd_create(dp.h, idb, int(nranks), int(rank), _p(box, _dp), ctypes.byref(p), self.natoms,
                                _p(coord, _dp), _p(atype, _ip), ctypes.byref(h))
        if rc != 0:
            raise B200DPError(rc, "b200dp_dd_create failed: " + dp.L.b200dp_last_error(dp.h).decode())
        self.h = h

    def _check(self, rc):
        if rc != 0:
            raise B200DPError(rc, self.L.b200dp_dd_last_error(self.h).decode())

    @property
    def stream(self) -> int:
        return self.L.b200dp_dd_stream(self.h) or 0

    def counts(self):
        n, g = ctypes.c_int(), ctypes.c_int()
        self._check(self.L.b200dp_dd_counts(self.h, ctypes.byref(n), ctypes.byref(g)))
        return n.value, g.value

    def force(self, stream: int = 0) -> None:
        self._check(self.L.b200dp_dd_force(self.h, stream or None))

    def result(self, stream: int = 0):
        e = np.zeros(1)
        v = np.zeros(9)
        self._check(self.L.b200dp_dd_result(self.h, stream or None, _p(e, _dp), _p(v, _dp)))
        return float(e[0]), v.reshape(3, 3)

    def owned(self):
        n, _ = self.counts()
        ids = np.zeros(n, np.int64)
        x, v, f = (np.zeros((n, 3)) for _ in range(3))
        self._check(self.L.b200dp_dd_owned(self.h, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_longlong)),
                                           _p(x, _dp), _p(v, _dp), _p(f, _dp)))
        return ids, x, v, f

    def set_positions(self, stream: int, host_ptr: int) -> None:
        self._check(self.L.b200dp_dd_set_positions(self.h, stream or None, host_ptr))

    def get_forces(self, stream: int, force_ptr: int, ev_ptr: int) -> None:
        self._check(self.L.b200dp_dd_get_forces(self.h, stream or None, force_ptr or None, ev_ptr or None))

    def md_start(self, masses, dt=0.0005, ensemble=NVE, vel=None, t_init=0.0, t_target=300.0, t_damp=0.05, chain=3,
                 seed=0, rebuild_every=10, p_target=1.0, p_damp=0.5, pchain=3):
        p = MDParams()
        self.L.b200dp_md_params_default(ctypes.byref(p))
        p.dt, p.ensemble, p.chain = dt, ensemble, chain
        p.t_target, p.t_damp, p.t_init, p.seed = t_target, t_damp, t_init, seed
        p.p_target, p.p_damp, p.pchain = p_target, p_damp, pchain
        p.rebuild_every = rebuild_every
        for t, m in enumerate(masses):
            p.mass[t] = m
        v = None if vel is None else np.ascontiguousarray(vel, dtype=np.float64).reshape(-1, 3)
        self._check(self.L.b200dp_dd_md_start(self.h, ctypes.byref(p), _p(v, _dp)))

    def md_run(self, nsteps: int) -> None:
        self._check(self.L.b200dp_dd_md_run(self.h, int(nsteps)))

    def thermo(self) -> dict:
        t = np.zeros(8)
        self._check(self.L.b200dp_dd_md_thermo(self.h, _p(t, _dp)))
        return dict(zip(self.THERMO, t))

    def close(self):
        if getattr(self, "h", None):
            self.L.b200dp_dd_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def dd_plan_emulate(nranks, grid, box, halo, coord, disp=None, ghost_cap=None):
    """The decomposed driver's host plan for nranks ranks emulated by threads (no GPU):
    per rank the owned ids and the ghosts (id, position, shift, origin)."""
    L = load_library()
    coord = np.ascontiguousarray(coord, dtype=np.float64).reshape(-1, 3)
    n = coord.shape[0]
    box = np.ascontiguousarray(box, dtype=np.float64).reshape(9)
    g = (ctypes.c_int * 3)(*[int(x) for x in grid])
    d = None if disp is None else np.ascontiguousarray(disp, dtype=np.float64).reshape(-1, 3)
    cap = int(ghost_cap if ghost_cap is not None else 8 * n + 1024)
    oid = np.zeros(n, np.int64)
    ocnt = np.zeros(nranks, np.int32)
    gid = np.zeros(cap, np.int64)
    gx = np.zeros((cap, 3))
    gs = np.zeros((cap, 3))
    go = np.zeros((cap, 2), np.int32)
    gcnt = np.zeros(nranks, np.int32)
    lp = ctypes.POINTER(ctypes.c_longlong)
    rc = L.b200dp_dd_plan_emulate(int(nranks), g, _p(box, _dp), float(halo), n, _p(coord, _dp), _p(d, _dp),
                                  oid.ctypes.data_as(lp), _p(ocnt, _ip), gid.ctypes.data_as(lp), _p(gx, _dp),
                                  _p(gs, _dp), _p(go, _ip), _p(gcnt, _ip), cap)
    if rc != 0:
        raise B200DPError(rc, "plan emulation failed")
    ranks, o, q = [], 0, 0
    for r in range(nranks):
        no, ng = int(ocnt[r]), int(gcnt[r])
        ranks.append(dict(owned=oid[o:o + no].copy(), ghost_ids=gid[q:q + ng].copy(), ghost_x=gx[q:q + ng].copy(),
                          ghost_shift=gs[q:q + ng].copy(), ghost_origin=go[q:q + ng].copy()))
        o += no
        q += ng
    return ranks


def kernel_launches() -> int:
    return int(load_library().b200dp_kernel_launches())


def _make_nlist(nlist):
    """nlist: list of neighbour index arrays, one per local atom (ilist = 0..n-1)."""
    n = len(nlist)
    arrs = [np.ascontiguousarray(a, dtype=np.int32) for a in nlist]
    ilist = np.arange(n, dtype=np.int32)
    numneigh = np.array([len(a) for a in arrs], dtype=np.int32)
    firstneigh = (ctypes.POINTER(ctypes.c_int) * max(n, 1))()
    for k, a in enumerate(arrs):
        firstneigh[k] = a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
    nl = NList(n, ilist.ctypes.data_as(_ip), numneigh.ctypes.data_as(_ip), firstneigh)
    return nl, (arrs, ilist, numneigh, firstneigh)
