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


# ---------------------------------------------------------------- C8L2 profile
# The reference's production descriptor ("DPA4C-Nano"): 8 scalar channels,
# angular degrees up to 2, no radial modes and no spin.  Per destination node
# it reduces degree-wise moments of a tabulated radial branch over the node's
# edges, normalizes them, aligns and projects them through fixed readout
# matrices and emits 70 rotation invariants (8 scalars, two 10-entry Grams,
# 20 + 4 bispectrum entries, 8 quartic entries, 2 moment divisors and an
# 8-wide type embedding), followed by a shared 70 -> 96 -> 96 -> 96 SiLU
# fitting net with a 96 -> 1 head.  Widths follow
# include/dpa_chain/graph_compress_launch.h:270-396 of the reference
# (Profile<8, 2, false>), the tensor set its direct-engine cache
# (components/deepmd-op/overlays/op/pt/dpa4c/graph_compress.cu:1451-1466).
#
# File layout (little endian):
#
#     char[8]  magic "B2DPC8L2"
#     int32    version (1), ntypes, channels (8), lmax (2), interval_count,
#              table_width (8), n_fit, fit[n_fit], resnets[n_fit],
#              activation (1 = SiLU, 0 = tanh), sel[ntypes]
#     float64  table_stride, table_max, rcut, eps, degree_floor, b_head,
#              bias_atom_e[ntypes]
#     float64  table [interval_count][6 * table_width]: per interval the
#              quartet block [table_width][c0 c1 c2 c3] then the pair block
#              [table_width][c4 c5] of p(x) = sum c_k x^k, x = r - i * stride
#     float64  pair_film [ntypes * ntypes][channels][2] (scale, shift; row
#              t_centre * ntypes + t_neighbour)
#     float64  type_embedding [ntypes][channels]
#     float64  readout [8][4][4]: matrices 0, 2, 4, 6 (vector alignment,
#              tensor alignment, vector probe, tensor probe; only the first
#              two columns of matrix 6 are used) each followed by its
#              transpose, which the backward reads
#     float64  output_mean [70], output_inv_std [70]
#     float64  fitting: per layer W [d_in][d_out] row-major then b [d_out];
#              then w_head [fit[-1]]
#
# ``sel`` is not part of the reference model: it sizes the per-type neighbour
# rows of this framework's formatted list (a row holding more in-cutoff
# neighbours than sel is an overflow, reported like DeePMD's).

C8_MAGIC = b"B2DPC8L2"
C8_DIM = 70


@dataclasses.dataclass
class C8Model:
    ntypes: int
    sel: list[int]
    channels: int = 8
    lmax: int = 2
    fit: list[int] = dataclasses.field(default_factory=lambda: [96, 96, 96])
    resnets: list[int] = dataclasses.field(default_factory=lambda: [0, 1, 1])
    activation: int = 1
    interval_count: int = 600
    table_max: float = 6.0
    rcut: float = 6.0
    eps: float = 1e-3
    degree_floor: float = 1.0
    b_head: float = 0.0
    bias_atom_e: list[float] | None = None
    table: np.ndarray | None = None  # [interval_count, 6 * channels]
    pair_film: np.ndarray | None = None  # [ntypes**2, channels, 2]
    type_embedding: np.ndarray | None = None  # [ntypes, channels]
    readout: np.ndarray | None = None  # [8, 4, 4]
    output_mean: np.ndarray | None = None  # [70]
    output_inv_std: np.ndarray | None = None  # [70]
    fit_layers: list[tuple[np.ndarray, np.ndarray]] = dataclasses.field(default_factory=list)
    w_head: np.ndarray | None = None

    @property
    def table_stride(self) -> float:
        return self.table_max / self.interval_count

    @property
    def table_width(self) -> int:
        return self.channels

    @property
    def sel_total(self) -> int:
        return int(sum(self.sel))

    def fit_dims(self) -> list[int]:
        return [C8_DIM] + list(self.fit)


def quintic_table(f, df, d2f, nint: int, rmax: float) -> np.ndarray:
    """Quintic Hermite pieces of f on [0, rmax]: per interval and channel the six
    coefficients of p(x), x in [0, h], matching f, f', f'' at both knots (so the
    table is C2 across knots).  f, df, d2f map radii [n] to values [n, width]."""
    h = rmax / nint
    knots = np.arange(nint + 1) * h
    v, d, s = f(knots), df(knots), d2f(knots)
    width = v.shape[1]
    c0, c1, c2 = v[:-1], d[:-1], 0.5 * s[:-1]
    dv = v[1:] - (c0 + c1 * h + c2 * h * h)
    dd = d[1:] - (c1 + 2.0 * c2 * h)
    ds = s[1:] - 2.0 * c2
    A = np.array([[h**3, h**4, h**5], [3 * h**2, 4 * h**3, 5 * h**4], [6 * h, 12 * h**2, 20 * h**3]])
    rhs = np.stack([dv, dd, ds], axis=-1)  # [nint, width, 3]
    c345 = np.linalg.solve(A, rhs.reshape(-1, 3).T).T.reshape(nint, width, 3)
    quartet = np.stack([c0, c1, c2, c345[..., 0]], axis=-1)  # [nint, width, 4]
    pair = c345[..., 1:]  # [nint, width, 2]
    return np.concatenate([quartet.reshape(nint, 4 * width), pair.reshape(nint, 2 * width)], axis=1)


def random_c8_model(seed: int = 0, ntypes: int = 2, sel=(46, 92), **over) -> C8Model:
    """Random-init C8L2 model.  The radial branch of every channel is a sum of
    eight Gaussians (centres spread over [0, rcut], random amplitudes), fitted
    by the quintic table; the readout matrices and the fitting net are
    N(0, 1/fan_in); descriptor statistics are random but fixed."""
    m = C8Model(ntypes=ntypes, sel=list(sel), **over)
    if m.bias_atom_e is None:
        m.bias_atom_e = [0.0] * ntypes
    rng = np.random.default_rng(seed)
    C = m.channels
    mu = np.linspace(0.0, m.rcut, 8)
    sig = 0.75
    amp = rng.normal(0.0, 1.0 / np.sqrt(8.0), size=(8, C))

    def gauss(r):
        z = (r[:, None] - mu[None, :]) / sig
        return z, np.exp(-0.5 * z * z)

    f = lambda r: gauss(r)[1] @ amp
    df = lambda r: (gauss(r)[1] * (-gauss(r)[0] / sig)) @ amp
    d2f = lambda r: (gauss(r)[1] * ((gauss(r)[0] ** 2 - 1.0) / sig**2)) @ amp
    m.table = quintic_table(f, df, d2f, m.interval_count, m.table_max)
    film = np.empty((ntypes * ntypes, C, 2))
    film[..., 0] = rng.normal(1.0, 0.3, size=(ntypes * ntypes, C))
    film[..., 1] = rng.normal(0.0, 0.1, size=(ntypes * ntypes, C))
    m.pair_film = film
    m.type_embedding = rng.normal(0.0, 1.0, size=(ntypes, C))
    ro = np.zeros((8, 4, 4))
    for k in (0, 2, 4, 6):
        ro[k] = rng.normal(0.0, 0.5, size=(4, 4))
        ro[k + 1] = ro[k].T
    m.readout = ro
    m.output_mean = rng.normal(0.0, 0.1, size=C8_DIM)
    m.output_inv_std = rng.uniform(0.5, 2.0, size=C8_DIM)
    dims = m.fit_dims()
    m.fit_layers = []
    for l in range(len(dims) - 1):
        std = np.sqrt(1.0 / dims[l])
        m.fit_layers.append((rng.normal(0.0, std, size=(dims[l], dims[l + 1])),
                             rng.normal(0.0, std, size=(dims[l + 1],))))
    m.w_head = rng.normal(0.0, np.sqrt(1.0 / dims[-1]), size=dims[-1])
    m.b_head = float(rng.normal(0.0, 0.1))
    return m


def save_c8(m: C8Model, path: str) -> None:
    with open(path, "wb") as f:
        f.write(C8_MAGIC)
        ints = [1, m.ntypes, m.channels, m.lmax, m.interval_count, m.table_width, len(m.fit), *m.fit,
                *m.resnets, int(m.activation), *m.sel]
        f.write(struct.pack(f"<{len(ints)}i", *ints))
        dbl = [m.table_stride, m.table_max, m.rcut, m.eps, m.degree_floor, m.b_head, *m.bias_atom_e]
        f.write(struct.pack(f"<{len(dbl)}d", *dbl))
        for a in (m.table, m.pair_film, m.type_embedding, m.readout, m.output_mean, m.output_inv_std):
            f.write(np.ascontiguousarray(a, dtype="<f8").tobytes())
        for w, b in m.fit_layers:
            f.write(np.ascontiguousarray(w, dtype="<f8").tobytes())
            f.write(np.ascontiguousarray(b, dtype="<f8").tobytes())
        f.write(np.ascontiguousarray(m.w_head, dtype="<f8").tobytes())


def load_c8(path: str) -> C8Model:
    with open(path, "rb") as f:
        data = f.read()
    if data[:8] != C8_MAGIC:
        raise ValueError(f"{path}: not a B2DPC8L2 model file")
    off = 8

    def ints(n):
        nonlocal off
        v = struct.unpack_from(f"<{n}i", data, off)
        off += 4 * n
        return list(v)

    def dbls(n):
        nonlocal off
        v = struct.unpack_from(f"<{n}d", data, off)
        off += 8 * n
        return list(v)

    def arr(shape):
        nonlocal off
        n = int(np.prod(shape))
        a = np.frombuffer(data, dtype="<f8", count=n, offset=off).reshape(shape).copy()
        off += 8 * n
        return a

    version, ntypes, channels, lmax, nint, width, nfit = ints(7)
    if version != 1:
        raise ValueError(f"{path}: unsupported version {version}")
    fit = ints(nfit)
    res = ints(nfit)
    (act,) = ints(1)
    sel = ints(ntypes)
    stride, tmax, rcut, eps, floor_, b_head = dbls(6)
    bias = dbls(ntypes)
    m = C8Model(ntypes=ntypes, sel=sel, channels=channels, lmax=lmax, fit=fit, resnets=res, activation=act,
                interval_count=nint, table_max=tmax, rcut=rcut, eps=eps, degree_floor=floor_, b_head=b_head,
                bias_atom_e=bias)
    m.table = arr((nint, 6 * width))
    m.pair_film = arr((ntypes * ntypes, channels, 2))
    m.type_embedding = arr((ntypes, channels))
    m.readout = arr((8, 4, 4))
    m.output_mean = arr((C8_DIM,))
    m.output_inv_std = arr((C8_DIM,))
    dims = m.fit_dims()
    m.fit_layers = [(arr((dims[l], dims[l + 1])), arr((dims[l + 1],))) for l in range(len(dims) - 1)]
    m.w_head = arr((dims[-1],))
    if off != len(data):
        raise ValueError(f"{path}: {len(data) - off} trailing bytes")
    if abs(stride - m.table_stride) > 1e-12 * max(1.0, stride):
        raise ValueError(f"{path}: table stride does not match table_max / interval_count")
    return m
