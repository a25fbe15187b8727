"""The C-ABI library loads on a CPU-only host and exports every entry point include/specdec_b200.h
declares (no compute calls without a GPU)."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "specdec_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"SD_API\s+[\w\s\*]*?\b(sd_\w+)\s*\(", src)))


def test_header_parses_and_lists_symbols():
    syms = declared_symbols()
    assert "sd_matvec_q4_0_q8_0_dev" in syms and "sd_generate" in syms and len(syms) >= 30


def test_library_exports_every_declared_symbol():
    from anetransformers_b200 import _lib
    L = _lib.lib()
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing
    assert L.sd_abi_version() == 1
    # binding table covers the header
    assert set(declared_symbols()) <= set(_lib.exported_symbols())


def test_no_device_is_reported_not_crashed():
    from anetransformers_b200 import _lib
    L = _lib.lib()
    n = L.sd_device_count()
    assert n >= 0


def test_header_compiles_as_c():
    out = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", "-x", "c", HEADER],
                         capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
