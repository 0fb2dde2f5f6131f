"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "dpa4c-scale-aware-md_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

import modelgen  # noqa: E402

GOLDEN = os.path.join(ROOT, "tests", "golden")
GOLDEN_CASES = ["water192", "water192_two_side", "water192_triclinic", "cu108", "alloy128"]
TOLERANCES = {  # mixed-mode acceptance limits (reference data/numeric-tolerances.json:3-9)
    "energy_per_atom": 2e-5,
    "force_rmse": 4e-5,
    "force_max": 5e-4,
    "stress_GPa": 4e-4,
}
EV_A3_TO_GPA = 160.21766208


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: full-size configuration")


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    d = tmp_path_factory.mktemp("models")
    specs = {
        "water": ("water", 0, {}),
        "water_two_side": ("water", 1, {"type_one_side": False}),
        "cu": ("cu", 0, {}),
        "alloy": ("alloy", 0, {}),
        "water_smallsel": ("water", 0, {"sel": [12, 24]}),
    }
    for name, (preset, seed, over) in specs.items():
        modelgen.save(modelgen.random_model(preset, seed=seed, **over), str(d / f"{name}.b2dp"))
    return d


def golden(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"), allow_pickle=False)
    import json

    meta = json.loads(str(z["meta"]))
    return {k: z[k] for k in z.files if k != "meta"}, meta


def golden_model_path(model_dir, meta):
    over = meta["over"]
    if meta["preset"] == "water" and over.get("type_one_side") is False:
        return str(model_dir / "water_two_side.b2dp")
    return str(model_dir / f"{meta['preset']}.b2dp")


def image_codes(img):
    img = np.asarray(img)
    return ((img[..., 0] + 512) << 20) | ((img[..., 1] + 512) << 10) | (img[..., 2] + 512)
