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


def test_header_is_plain_c_and_links(tmp_path):
    """A C11 translation unit that takes the address of every declared function compiles
    with warnings as errors and links against the library (what a cgo / plain-C binding
    needs); the program runs without touching a GPU."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    names = declared_functions()
    src = tmp_path / "abi.c"
    src.write_text('#include <stdio.h>\n#include "b200dp.h"\n'
                   "typedef void (*fn)(void);\n"
                   "int main(void) {\n  fn table[] = {\n"
                   + "".join(f"    (fn){n},\n" for n in names)
                   + "  };\n  int n = 0;\n"
                   "  for (size_t i = 0; i < sizeof(table) / sizeof(table[0]); ++i) n += table[i] != 0;\n"
                   '  printf("%d\\n", n);\n  return 0;\n}\n')
    lib_dir = os.path.dirname(b200dp.LIB_PATH)
    exe = tmp_path / "abi"
    r = subprocess.run([cc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                        str(src), "-o", str(exe), "-L", lib_dir, "-lb200dp", f"-Wl,-rpath,{lib_dir}",
                        "-Wl,--allow-shlib-undefined"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    assert int(out.stdout.strip()) == len(names)
