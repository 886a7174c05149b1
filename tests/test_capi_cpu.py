"""The C-ABI library loads and exports every entry point the header declares
(no GPU needed: no compute call is made)."""

from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from tests.conftest import ROOT
from tensorshrink_b200 import _C

HEADER = ROOT / "include" / "tensorshrink_b200.h"


def header_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"TS_API\s+[\w\s\*]+?\b(ts_\w+)\s*\(", text)))


def test_header_declares_functions():
    fns = header_functions()
    assert "ts_qlinear" in fns and "ts_quantize_pack" in fns
    assert len(fns) >= 10


def test_library_exports_every_declared_symbol():
    lib = _C.load()
    for name in header_functions():
        assert hasattr(lib, name), name
    assert set(header_functions()) == set(_C.EXPORTED_SYMBOLS)


def test_library_exports_nothing_else():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_C.lib_path())], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert {s for s in exported if s.startswith("ts_")} == set(header_functions())


def test_version_and_errors_without_gpu():
    lib = _C.load()
    assert b"sm_100a" in lib.ts_version()
    # argument validation happens before any CUDA call
    rc = lib.ts_qlinear(None, None, 0, 1, 1, None, 0, None, 0, 1, None, 0, None)
    assert rc == -1
    assert b"NULL" in lib.ts_last_error()
    with pytest.raises(ValueError):
        _C.check(rc, "ts_qlinear")
    q = _C.TsQWeight()
    q.bits = 3
    rc = lib.ts_qlinear(ctypes.byref(q), None, 0, 1, 1, None, 0, None, 0, 1, None, 0, None)
    assert rc == -2
    with pytest.raises(NotImplementedError):
        _C.check(rc, "ts_qlinear")


def test_struct_layouts_match_header():
    # sizes fixed by the header's field order (all 8-byte aligned members)
    assert ctypes.sizeof(_C.TsQWeight) == 8 * 5 + 4 * 2 + 8 * 7 + 4 * 2 + 8 + 8 + 8 * 4
    assert ctypes.sizeof(_C.TsQuantParams) == 8 * 2 + 4 * 2 + 8 + 4 * 4 + 8 * 2 + 8
    assert ctypes.sizeof(_C.TsQuantOutputs) == 8 * 16
