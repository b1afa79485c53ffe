"""The C-ABI library loads on a CPU-only machine and exports every entry point
include/tokquay_b200.h declares, with a binding for each.  No kernel runs."""

import ctypes
import re
from pathlib import Path

import pytest

from tokquay_b200 import _lib
from tokquay_b200.build import LIB_PATH, is_stale

HEADER = Path(__file__).resolve().parents[1] / "include" / "tokquay_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^TQ_API\s+[\w\s\*]+?\b(tq_\w+)\s*\(", text, flags=re.M)


def test_header_declares_the_entry_points():
    names = declared_functions()
    assert len(names) == len(set(names)) >= 10
    assert set(names) == set(_lib.SIGNATURES), "every declared function needs a binding and vice versa"


def test_library_is_built_and_current():
    assert LIB_PATH.exists(), "run `python -m tokquay_b200.build`"
    assert not is_stale(), "libtokquay_b200.so is older than its sources"


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(LIB_PATH))
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_abi_version_and_error_channel():
    lib = _lib.load()
    m = re.search(r"#define TQ_ABI_VERSION (\d+)", HEADER.read_text())
    assert lib.tq_abi_version() == int(m.group(1)) == _lib.EXPECTED_ABI
    # A host-only call that fails sets the thread's message.
    layout = (ctypes.c_int32 * _lib.PLAN_LAYOUT_LEN)()
    st = lib.tq_plan_step(0, None, None, None, None, None, 16, 8, 1, 0, 1, 1, None, None, 0,
                          ctypes.addressof(layout))
    assert st == _lib.TQ_ERR_INVALID
    assert "non-empty" in _lib.last_error()


def test_status_mapping_to_python_exceptions():
    with pytest.raises(ValueError):
        _lib.check(_lib.TQ_ERR_INVALID, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.TQ_ERR_CUDA, "x")
    _lib.check(_lib.TQ_OK, "x")


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(_lib.NativeLibraryMissing):
        _lib.load(tmp_path / "nope.so")


def test_noalloc_limit_matches_the_header():
    m = re.search(r"#define TQ_NOALLOC_MAX_PARTIALS (\d+)", HEADER.read_text())
    assert int(m.group(1)) == _lib.NOALLOC_MAX_PARTIALS
