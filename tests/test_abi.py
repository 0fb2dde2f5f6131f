"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and rejects bad model files before touching the device."""
import ctypes
import os
import re

import pytest

import b200dp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "b200dp.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200dp_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_functions():
    names = declared_functions()
    assert "b200dp_compute_host" in names and "b200dp_compute_device" in names
    assert len(names) >= 14


def test_library_exports_every_declared_symbol():
    L = b200dp.load_library()
    for name in declared_functions():
        assert hasattr(L, name), name
    assert set(b200dp.EXPORTS) <= set(declared_functions())


def test_create_rejects_missing_and_bad_files(tmp_path):
    with pytest.raises(b200dp.B200DPError) as e:
        b200dp.DeepPot(str(tmp_path / "missing.b2dp"))
    assert e.value.status == 2
    bad = tmp_path / "bad.b2dp"
    bad.write_bytes(b"NOTAMODEL" + bytes(100))
    with pytest.raises(b200dp.B200DPError) as e:
        b200dp.DeepPot(str(bad))
    assert e.value.status == 2


def test_create_rejects_truncated_model(tmp_path, model_dir):
    data = (model_dir / "water.b2dp").read_bytes()
    p = tmp_path / "trunc.b2dp"
    p.write_bytes(data[: len(data) // 2])
    with pytest.raises(b200dp.B200DPError) as e:
        b200dp.DeepPot(str(p))
    assert e.value.status == 2


def test_options_default():
    L = b200dp.load_library()
    o = b200dp.Options()
    L.b200dp_options_default(ctypes.byref(o))
    assert o.precision == b200dp.MIXED and o.device == 0 and o.sel_overflow_is_error == 0


def test_null_engine_is_rejected():
    L = b200dp.load_library()
    assert L.b200dp_check(None) == 1
    assert L.b200dp_compute_host(None, 0, 0, None, None, None, None, None, None, None, None) == 1
