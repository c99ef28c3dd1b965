"""The C-ABI library loads without a GPU and exports every symbol the headers
declare; argument validation answers with status codes, never aborts."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from ictc_o2_hp_b200 import _lib

INCLUDE = Path(__file__).resolve().parents[1] / "include"


def declared_symbols() -> list[str]:
    names = []
    for header in sorted(INCLUDE.glob("*.h")):
        text = header.read_text()
        names += re.findall(r"ICTC_API\s+[\w\s\*]+?\b(ictc_\w+)\s*\(", text)
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "ictc_o2_tp_forward" in names and "ictc_o2_tp_backward" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)


def test_python_signatures_cover_the_header():
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_abi_version():
    assert _lib.load().ictc_o2_abi_version() >= 100


def test_invalid_arguments_return_status():
    lib = _lib.load()
    out = ctypes.c_int64()
    assert lib.ictc_o2_tp_weight_numel(0, 2, 1, ctypes.byref(out)) == _lib.ERR_INVALID
    assert "channels" in lib.ictc_o2_last_error().decode()
    assert lib.ictc_o2_tp_weight_numel(4, -1, 1, ctypes.byref(out)) == _lib.ERR_INVALID
    assert lib.ictc_o2_tp_weight_numel(4, 2, 7, ctypes.byref(out)) == _lib.ERR_INVALID
    assert lib.ictc_o2_tp_weight_numel(4, 99, 1, ctypes.byref(out)) == _lib.ERR_UNSUPPORTED
    assert lib.ictc_o2_tp_weight_numel(4, 2, 1, None) == _lib.ERR_INVALID
    # rows == 0 forward is a no-op that touches no device
    assert lib.ictc_o2_tp_forward(None, None, None, None, 0, 4, 2, 1, 0, None) == _lib.OK
    assert lib.ictc_o2_tp_forward(None, None, None, None, -1, 4, 2, 1, 0, None) == \
        _lib.ERR_INVALID
    assert lib.ictc_o2_tp_forward(None, None, None, None, 5, 4, 2, 1, 3, None) == \
        _lib.ERR_INVALID
    # the wait probe validates its limit and pointer before touching a device
    assert lib.ictc_o2_test_wait_timeout(0, None, None) == _lib.ERR_INVALID
    assert lib.ictc_o2_test_wait_timeout(2000000, None, None) == _lib.ERR_INVALID
    assert lib.ictc_o2_test_wait_timeout(100, None, None) == _lib.ERR_INVALID


def test_check_maps_status_to_exceptions():
    with pytest.raises(ValueError):
        _lib.tp_weight_numel(0, 1, "full")
    with pytest.raises(NotImplementedError):
        _lib.tp_weight_numel(3, 40, "full")
