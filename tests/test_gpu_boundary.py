"""GPU checks of the drop-in boundary: the reference-signature C headers and the mistral CLI."""
import os
import subprocess

import numpy as np
import pytest

from tests.conftest import gpu_available
from tests.test_capi import ROOT, ROOT_LIB, build_compat_check

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a CUDA GPU")]


@pytest.fixture(scope="module")
def mini_path(tmp_path_factory):
    from anetransformers_b200 import gguf as G
    p = str(tmp_path_factory.mktemp("b") / "mini.gguf")
    G.write_synthetic_gguf(p, G.MINI, seed=9)
    return p


def test_compat_headers_run(tmp_path, mini_path):
    exe = build_compat_check(tmp_path)
    out = subprocess.run([exe, mini_path], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    lines = out.stdout.splitlines()
    assert any(l.startswith("ngram n=1 first=4") or l.startswith("ngram n=") for l in lines)
    assert "batch5=0 batch9=0 batch17=-1" in out.stdout   # verify batches up to SD_MAX_VERIFY = 16
    assert "verify rc=0 accepted=5" in out.stdout      # drafts = argmax of each row -> all accepted + bonus


def test_compat_quantize_matches_oracle(tmp_path, oracle):
    exe = build_compat_check(tmp_path)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0
    n = 4096
    x = (np.sin(np.float32(0.37) * np.arange(n, dtype=np.float32)) * (1 + np.arange(n) % 7)).astype(np.float32)
    ref = oracle.quantize_q8_0(x)
    line = next(l for l in out.stdout.splitlines() if l.startswith("q8 "))
    d0 = float(line.split()[1].split("=")[1])
    q0 = int(line.split()[2].split("=")[1])
    assert np.float32(d0) == ref[0]["d"] and q0 == ref[0]["qs"][0]


def test_cli_ngram_decode(mini_path):
    cli = os.path.join(ROOT_LIB, "mistral")
    ids = ",".join(str(t) for t in [5, 6, 7, 8, 9, 10, 5, 6, 7, 8, 9, 10, 5, 6, 7])
    out = subprocess.run([cli, "--model", mini_path, "--prompt-ids", ids, "--tokens", "12", "--temp", "0",
                          "--rep-penalty", "1", "--ignore-eos", "--speculative", "--draft", "ngram",
                          "--context", "512"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert "Generated tokens:" in out.stderr and "Acceptance rate" in out.stderr
    # greedy run of the same prompt prints the same text (temp-0 speculation is exact)
    out2 = subprocess.run([cli, "--model", mini_path, "--prompt-ids", ids, "--tokens", "12", "--temp", "0",
                           "--rep-penalty", "1", "--ignore-eos", "--context", "512"], capture_output=True, text=True,
                          timeout=300)
    assert out2.returncode == 0, out2.stderr
    a, b = out.stdout.strip(), out2.stdout.strip()
    assert a[:min(len(a), len(b))] == b[:min(len(a), len(b))]
