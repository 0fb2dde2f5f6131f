"""Generates the golden fixtures in this directory.

    python tests/golden/make_golden.py

No golden vectors for this path exist in the reference, so the fixtures come
from the independent PyTorch/autograd restatement in torch_sea.py (not from
the C++ oracle), on seeded systems and seeded random-init models.  Each
fixture stores the model recipe (preset, seed, overrides) and a SHA-256 of the
regenerated model file so a drift in the generator is detected.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "dpa4c-scale-aware-md_b200"))
sys.path.insert(0, HERE)

import modelgen  # noqa: E402
import systems  # noqa: E402
import torch_sea  # noqa: E402


def sheared_water():
    s = systems.water(4, seed=3, name="water_triclinic_192")
    box = s.box.copy()
    box[1, 0] = 2.0  # b gets an x component
    box[2, 0] = -1.0
    box[2, 1] = 1.5
    frac = s.coord @ np.linalg.inv(s.box)
    s.coord = frac @ box
    s.box = box
    return s


CASES = {
    "water192": dict(system=lambda: systems.config0(), model=("water", 0, {})),
    "water192_two_side": dict(system=lambda: systems.config0(), model=("water", 1, {"type_one_side": False})),
    "water192_triclinic": dict(system=sheared_water, model=("water", 0, {})),
    "cu108": dict(system=lambda: systems.fcc(3, name="cu_fcc_108"), model=("cu", 0, {})),
    "alloy128": dict(system=lambda: systems.bcc_alloy(4, name="bcc_alloy_128"), model=("alloy", 0, {})),
}


def model_file(preset, seed, over, path):
    m = modelgen.random_model(preset, seed=seed, **over)
    modelgen.save(m, path)
    with open(path, "rb") as f:
        return m, hashlib.sha256(f.read()).hexdigest()


def main():
    for name, case in CASES.items():
        s = case["system"]()
        preset, seed, over = case["model"]
        with tempfile.TemporaryDirectory() as td:
            m, digest = model_file(preset, seed, over, os.path.join(td, "m.b2dp"))
        out = torch_sea.evaluate(m, s.coord, s.atype, s.box)
        meta = dict(case=name, system=s.name, preset=preset, seed=seed, over=over, model_sha256=digest,
                    generator="tests/golden/torch_sea.py (autograd)")
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), coord=s.coord, atype=s.atype, box=s.box,
                            energy=out["energy"], force=out["force"], virial=out["virial"],
                            atom_energy=out["atom_energy"], atom_virial=out["atom_virial"], nlist=out["nlist"],
                            image=out["image"], meta=json.dumps(meta))
        print(name, s.natoms, out["energy"], np.abs(out["force"]).max())


if __name__ == "__main__":
    main()
