"""Random-init DPA4C-style (se_e2_a type) model files.

File layout (little endian), read by ``b200dp_create`` and by the CPU oracle:

    char[8]  magic "B2DPSEA1"
    int32    version (1), ntypes, n_emb, emb[n_emb], axis, n_fit, fit[n_fit],
             type_one_side, activation (0 = tanh), sel[ntypes]
    float64  rcut, rcut_smth, bias_atom_e[ntypes]
    float64  embedding nets, then fitting nets (see below)

Embedding nets: ``ntypes`` nets when ``type_one_side`` (indexed by neighbour
type), else ``ntypes**2`` (indexed ``t_centre * ntypes + t_neighbour``).  Each
net maps 1 -> emb[0] -> ... -> emb[-1]; for every layer W [d_in, d_out]
row-major then b [d_out].  Fitting nets: one per centre type, mapping
emb[-1]*axis -> fit[0] -> ... -> fit[-1] -> 1, same per-layer order.

Weights and biases are N(0, 1/fan_in), fp64, drawn from
``np.random.default_rng(seed)`` in file order.
"""
from __future__ import annotations

import dataclasses
import struct

import numpy as np

MAGIC = b"B2DPSEA1"


@dataclasses.dataclass
class SeaModel:
    ntypes: int
    sel: list[int]
    emb: list[int]
    axis: int
    fit: list[int]
    rcut: float = 6.0
    rcut_smth: float = 0.5
    type_one_side: bool = True
    activation: int = 0
    bias_atom_e: list[float] | None = None
    emb_nets: list[list[tuple[np.ndarray, np.ndarray]]] = dataclasses.field(default_factory=list)
    fit_nets: list[list[tuple[np.ndarray, np.ndarray]]] = dataclasses.field(default_factory=list)

    @property
    def n_emb_nets(self) -> int:
        return self.ntypes if self.type_one_side else self.ntypes * self.ntypes

    @property
    def sel_total(self) -> int:
        return int(sum(self.sel))

    @property
    def descriptor_dim(self) -> int:
        return self.emb[-1] * self.axis

    def emb_dims(self) -> list[int]:
        return [1] + list(self.emb)

    def fit_dims(self) -> list[int]:
        return [self.descriptor_dim] + list(self.fit) + [1]


PRESETS = {
    # water: sel [46,92], embedding [25,50,100], axis 16, fitting [240]*3
    "water": dict(ntypes=2, sel=[46, 92], emb=[25, 50, 100], axis=16, fit=[240, 240, 240]),
    # copper: sel [140], embedding [32,64,128], fitting [256]*3
    "cu": dict(ntypes=1, sel=[140], emb=[32, 64, 128], axis=16, fit=[256, 256, 256]),
    # 4-type BCC alloy: sel [40]*4
    "alloy": dict(ntypes=4, sel=[40, 40, 40, 40], emb=[32, 64, 128], axis=16, fit=[256, 256, 256]),
}


def random_model(kind: str = "water", seed: int = 0, **over) -> SeaModel:
    """Random-init model of a preset shape; every W, b ~ N(0, 1/fan_in)."""
    kw = dict(PRESETS[kind])
    kw.update(over)
    m = SeaModel(**kw)
    if m.bias_atom_e is None:
        m.bias_atom_e = [0.0] * m.ntypes
    rng = np.random.default_rng(seed)
    dims = m.emb_dims()
    for _ in range(m.n_emb_nets):
        net = []
        for l in range(len(dims) - 1):
            std = np.sqrt(1.0 / dims[l])
            w = rng.normal(0.0, std, size=(dims[l], dims[l + 1]))
            b = rng.normal(0.0, std, size=(dims[l + 1],))
            net.append((w, b))
        m.emb_nets.append(net)
    fdims = m.fit_dims()
    for _ in range(m.ntypes):
        net = []
        for l in range(len(fdims) - 1):
            std = np.sqrt(1.0 / fdims[l])
            w = rng.normal(0.0, std, size=(fdims[l], fdims[l + 1]))
            b = rng.normal(0.0, std, size=(fdims[l + 1],))
            net.append((w, b))
        m.fit_nets.append(net)
    return m


def save(m: SeaModel, path: str) -> None:
    with open(path, "wb") as f:
        f.write(MAGIC)
        ints = [1, m.ntypes, len(m.emb), *m.emb, m.axis, len(m.fit), *m.fit,
                int(m.type_one_side), int(m.activation), *m.sel]
        f.write(struct.pack(f"<{len(ints)}i", *ints))
        dbl = [m.rcut, m.rcut_smth, *m.bias_atom_e]
        f.write(struct.pack(f"<{len(dbl)}d", *dbl))
        for net in m.emb_nets + m.fit_nets:
            for w, b in net:
                f.write(np.ascontiguousarray(w, dtype="<f8").tobytes())
                f.write(np.ascontiguousarray(b, dtype="<f8").tobytes())


def load(path: str) -> SeaModel:
    with open(path, "rb") as f:
        data = f.read()
    if data[:8] != MAGIC:
        raise ValueError(f"{path}: not a B2DPSEA1 model file")
    off = 8

    def ints(n):
        nonlocal off
        v = struct.unpack_from(f"<{n}i", data, off)
        off += 4 * n
        return list(v)

    version, ntypes, n_emb = ints(3)
    if version != 1:
        raise ValueError(f"{path}: unsupported version {version}")
    emb = ints(n_emb)
    axis, n_fit = ints(2)
    fit = ints(n_fit)
    tos, act = ints(2)
    sel = ints(ntypes)
    rcut, rs = struct.unpack_from("<2d", data, off)
    off += 16
    bias = list(struct.unpack_from(f"<{ntypes}d", data, off))
    off += 8 * ntypes
    m = SeaModel(ntypes=ntypes, sel=sel, emb=emb, axis=axis, fit=fit, rcut=rcut, rcut_smth=rs,
                 type_one_side=bool(tos), activation=act, bias_atom_e=bias)

    def arr(shape):
        nonlocal off
        n = int(np.prod(shape))
        a = np.frombuffer(data, dtype="<f8", count=n, offset=off).reshape(shape).copy()
        off += 8 * n
        return a

    dims = m.emb_dims()
    for _ in range(m.n_emb_nets):
        m.emb_nets.append([(arr((dims[l], dims[l + 1])), arr((dims[l + 1],))) for l in range(len(dims) - 1)])
    fd = m.fit_dims()
    for _ in range(ntypes):
        m.fit_nets.append([(arr((fd[l], fd[l + 1])), arr((fd[l + 1],))) for l in range(len(fd) - 1)])
    if off != len(data):
        raise ValueError(f"{path}: {len(data) - off} trailing bytes")
    return m
