"""The C-ABI library loads and exports every symbol include/*.h declares
(no compute calls: this runs without a GPU)."""
import ctypes
import re

from packr_b200 import _lib
from conftest import REPO


def declared_symbols():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(packr_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.lib_path()))
    names = declared_symbols()
    assert "packr_adam8_multi" in names
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_covers_declarations():
    assert declared_symbols() <= set(_lib.SIGNATURES), \
        f"no ctypes signature for {declared_symbols() - set(_lib.SIGNATURES)}"


def test_error_strings_and_version():
    lib = _lib.load()
    assert lib.packr_abi_version() >= 1
    assert lib.packr_error_string(0) == b"ok"
    assert lib.packr_error_string(7) == b"device-side wait timed out"
    assert lib.packr_error_string(999) == b"unknown status"


def test_adam_rejects_bad_arguments_before_touching_the_device():
    lib = _lib.load()
    # negative tensor count and a NULL table are argument errors
    assert lib.packr_adam8_multi(None, -1, 1e-3, .9, .999, 1e-8, .1, .001, 0., None) == 1
    assert lib.packr_adam8_multi(None, 3, 1e-3, .9, .999, 1e-8, .1, .001, 0., None) == 1
    assert lib.packr_adam8_multi(None, 0, 1e-3, .9, .999, 1e-8, .1, .001, 0., None) == 0


def test_variant_build_needs_its_own_output():
    import pytest
    from packr_b200 import build
    with pytest.raises(ValueError):
        build.build(defines=["PACKR_SKINNY_N16=1"])  # would overwrite the in-tree library
