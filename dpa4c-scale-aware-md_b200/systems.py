"""Seeded synthetic systems for the five DPA4C evaluation configurations.

The reference publishes no input data for these configurations, so every system
is generated here from a seed.  All coordinates are fp64 Angstrom, the box is a
3x3 row-vector matrix (rows are the cell vectors a, b, c), and types are int32.

Recipes (one function per family):

* water: O on a jittered simple-cubic lattice of spacing 3.105 A (N(0, 0.1 A)
  jitter), each O carrying two H at 0.96 A with an H-O-H angle of 104.5 deg in a
  uniformly random orientation (random unit quaternion).  Atom order is
  O, H, H per molecule.  Types O=0, H=1.  64 molecules in a 12.42 A cube is the
  192-atom CPU case; 16^3 molecules in a 49.68 A cube is the 12,288-atom case.
* copper: FCC, a = 3.615 A, N(0, 0.05 A) displacements, one type.
* bcc alloy: BCC, a = 3.2 A, types uniform over 4 (seed 1), N(0, 0.08 A) jitter.
* slab: a water block whose box is doubled along z (50 % vacuum).

The RNG is numpy's PCG64 (``np.random.default_rng(seed)``); draws happen in
the fixed order documented in each function so the systems are reproducible.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np

WATER_SPACING = 3.105
OH_BOND = 0.96
HOH_ANGLE_DEG = 104.5


@dataclasses.dataclass
class System:
    name: str
    coord: np.ndarray  # [n, 3] float64
    atype: np.ndarray  # [n] int32
    box: np.ndarray  # [3, 3] float64, rows are cell vectors

    @property
    def natoms(self) -> int:
        return int(self.coord.shape[0])


def _quat_to_rot(q: np.ndarray) -> np.ndarray:
    """Rotation matrices [n,3,3] from unit quaternions [n,4] (w, x, y, z)."""
    w, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    r = np.empty((q.shape[0], 3, 3))
    r[:, 0, 0] = 1 - 2 * (y * y + z * z)
    r[:, 0, 1] = 2 * (x * y - z * w)
    r[:, 0, 2] = 2 * (x * z + y * w)
    r[:, 1, 0] = 2 * (x * y + z * w)
    r[:, 1, 1] = 1 - 2 * (x * x + z * z)
    r[:, 1, 2] = 2 * (y * z - x * w)
    r[:, 2, 0] = 2 * (x * z - y * w)
    r[:, 2, 1] = 2 * (y * z + x * w)
    r[:, 2, 2] = 1 - 2 * (x * x + y * y)
    return r


def water(nx: int, ny: int | None = None, nz: int | None = None, seed: int = 0,
          jitter: float = 0.1, vacuum_z: float = 1.0, name: str | None = None) -> System:
    """Water box of nx*ny*nz molecules on a jittered 3.105 A lattice.

    Draw order: jitter [nmol,3] normal, then quaternions [nmol,4] normal.
    ``vacuum_z`` scales the z cell vector (2.0 gives a 50 % vacuum slab).
    """
    ny = nx if ny is None else ny
    nz = nx if nz is None else nz
    nmol = nx * ny * nz
    rng = np.random.default_rng(seed)
    jit = rng.normal(0.0, jitter, size=(nmol, 3))
    q = rng.normal(size=(nmol, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    ix, iy, iz = np.meshgrid(np.arange(nx), np.arange(ny), np.arange(nz), indexing="ij")
    lat = np.stack([ix.ravel(), iy.ravel(), iz.ravel()], axis=1).astype(np.float64)
    o = (lat + 0.5) * WATER_SPACING + jit
    half = math.radians(HOH_ANGLE_DEG) / 2.0
    h_local = np.array([[math.sin(half), math.cos(half), 0.0],
                        [-math.sin(half), math.cos(half), 0.0]]) * OH_BOND
    rot = _quat_to_rot(q)
    h = o[:, None, :] + np.einsum("nij,kj->nki", rot, h_local)
    coord = np.concatenate([o[:, None, :], h], axis=1).reshape(-1, 3)
    atype = np.tile(np.array([0, 1, 1], dtype=np.int32), nmol)
    box = np.diag([nx * WATER_SPACING, ny * WATER_SPACING, nz * WATER_SPACING * vacuum_z])
    return System(name or f"water_{3 * nmol}", np.ascontiguousarray(coord), atype, box)


def fcc(n: int, a: float = 3.615, sigma: float = 0.05, seed: int = 0, name: str | None = None) -> System:
    """FCC n^3 cells (4 atoms/cell), one type.  Draw order: displacements [N,3]."""
    basis = np.array([[0, 0, 0], [0.5, 0.5, 0], [0.5, 0, 0.5], [0, 0.5, 0.5]])
    ix, iy, iz = np.meshgrid(np.arange(n), np.arange(n), np.arange(n), indexing="ij")
    cells = np.stack([ix.ravel(), iy.ravel(), iz.ravel()], axis=1).astype(np.float64)
    pos = (cells[:, None, :] + basis[None, :, :]).reshape(-1, 3) * a
    rng = np.random.default_rng(seed)
    pos = pos + rng.normal(0.0, sigma, size=pos.shape)
    return System(name or f"cu_fcc_{pos.shape[0]}", pos, np.zeros(pos.shape[0], np.int32),
                  np.diag([n * a] * 3))


def bcc_alloy(n: int, a: float = 3.2, sigma: float = 0.08, ntypes: int = 4, seed: int = 1,
              name: str | None = None) -> System:
    """BCC n^3 cells (2 atoms/cell), types uniform over ``ntypes``.

    Draw order: types [N] integers, then jitter [N,3] normal.
    """
    basis = np.array([[0, 0, 0], [0.5, 0.5, 0.5]])
    ix, iy, iz = np.meshgrid(np.arange(n), np.arange(n), np.arange(n), indexing="ij")
    cells = np.stack([ix.ravel(), iy.ravel(), iz.ravel()], axis=1).astype(np.float64)
    pos = (cells[:, None, :] + basis[None, :, :]).reshape(-1, 3) * a
    rng = np.random.default_rng(seed)
    atype = rng.integers(0, ntypes, size=pos.shape[0]).astype(np.int32)
    pos = pos + rng.normal(0.0, sigma, size=pos.shape)
    return System(name or f"bcc_alloy_{pos.shape[0]}", pos, atype, np.diag([n * a] * 3))


# The five configurations.  Sizes follow the configuration list; shapes that a
# cube cannot give (3.1 M atoms) are fixed here.
def config0() -> System:
    return water(4, name="c0_water_192")


def config1() -> System:
    return water(16, name="c1_water_12288")


def config2() -> System:
    return fcc(32, name="c2_cu_131072")


def config3() -> System:
    return bcc_alloy(64, name="c3_bcc_524288")


def config4(size: str) -> System:
    table = {
        "1.5k": (8, 8, 8, 1.0),
        "12k": (16, 16, 16, 1.0),
        "98k": (32, 32, 32, 1.0),
        "786k": (64, 64, 64, 1.0),
        "3.1M": (128, 128, 64, 1.0),
        "786k-slab": (64, 64, 64, 2.0),
    }
    nx, ny, nz, vac = table[size]
    return water(nx, ny, nz, vacuum_z=vac, name=f"c4_water_{size}")


MODEL_FOR_SYSTEM = {"water": "water", "cu": "cu", "bcc": "alloy"}


def model_kind(system: System) -> str:
    if "water" in system.name:
        return "water"
    if "cu" in system.name:
        return "cu"
    return "alloy"
