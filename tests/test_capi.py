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


ROOT_LIB = os.path.join(ROOT, "anetransformers_b200")


def build_compat_check(tmp_path):
    exe = str(tmp_path / "compat_check")
    cmd = ["gcc", "-std=gnu11", "-Wall", "-Wno-unused-function", "-I" + os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "compat_check.c"), "-o", exe, "-L" + ROOT_LIB, "-lspecdec_b200",
           "-Wl,-rpath," + ROOT_LIB, "-lm"]
    out = subprocess.run(cmd, capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    return exe


def test_compat_headers_compile_and_link(tmp_path):
    exe = build_compat_check(tmp_path)
    from tests.conftest import gpu_available
    if not gpu_available():
        out = subprocess.run([exe], capture_output=True, text=True)
        assert out.returncode == 0 and "no-device" in out.stdout, out.stdout + out.stderr


def test_cli_usage_and_errors():
    cli = os.path.join(ROOT_LIB, "mistral")
    assert os.path.exists(cli)
    out = subprocess.run([cli], capture_output=True, text=True)
    assert out.returncode == 1 and "--prompt-ids" in out.stderr
    out = subprocess.run([cli, "--model", "/nonexistent", "--prompt", "hi"], capture_output=True, text=True)
    assert out.returncode == 1 and "No such file" in out.stderr
    out = subprocess.run([cli, "--model", "/nonexistent"], capture_output=True, text=True)
    assert out.returncode == 1 and "--prompt" in out.stderr   # no prompt: usage
