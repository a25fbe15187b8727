"""Synthetic GGUF writer / reader vs the reference's own parser (mistral/gguf_loader.h compiled into
oracle/_ref/gguf_dump by oracle/Makefile)."""
import dataclasses
import json
import os
import subprocess

import numpy as np
import pytest

from anetransformers_b200 import gguf as G

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DUMP = os.path.join(ROOT, "oracle", "_ref", "gguf_dump")
REF_SRC = os.path.join(os.environ.get("ANETRANSFORMERS_REFERENCE", "/root/reference"), "mistral", "gguf_loader.h")


@pytest.fixture(scope="module")
def mini_path(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("gguf") / "mini.gguf")
    G.write_synthetic_gguf(p, G.MINI, seed=11)
    return p


def _ref_dump():
    if not os.path.exists(REF_DUMP):
        if not os.path.exists(REF_SRC):
            pytest.skip("reference tree not present and oracle/_ref/gguf_dump not built")
        subprocess.check_call(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref"])
    return REF_DUMP


def test_reader_roundtrip(mini_path):
    g = G.GGUFFile(mini_path)
    got, exp = dataclasses.asdict(g.config()), dataclasses.asdict(G.MINI)
    for k in exp:
        assert got[k] == pytest.approx(exp[k], rel=1e-6), k
    names = [n for n, _, _ in G.tensor_names(G.MINI)]
    assert list(g.tensors) == names
    w = g.array("blk.0.attn_q.weight")
    assert w.shape == (1024, 32) and w.dtype == G.Q4_0_DTYPE
    d = w["d"].astype(np.float32)
    assert (d >= 0).all() and 0.005 < d.mean() < 0.03        # |N(0, 0.02)|
    assert np.all(g.array("blk.1.ffn_norm.weight") == 1.0)
    g.close()


def test_deterministic(tmp_path):
    a = G.synthetic_gguf_bytes(G.MINI, seed=5)
    b = G.synthetic_gguf_bytes(G.MINI, seed=5)
    c = G.synthetic_gguf_bytes(G.MINI, seed=6)
    assert a == b and a != c


def test_reference_parser_reads_synthetic_model(mini_path):
    out = json.loads(subprocess.check_output([_ref_dump(), mini_path]))
    cfg = G.MINI
    assert out["version"] == 3
    for k in ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size"):
        assert out[k] == getattr(cfg, k), k
    assert out["head_dim"] == cfg.head_dim
    assert abs(out["rope_theta"] - cfg.rope_theta) < 1e-3 and abs(out["rms_eps"] - cfg.rms_eps) < 1e-12
    assert out["bos_id"] == 1 and out["eos_id"] == 2
    g = G.GGUFFile(mini_path)
    assert out["data_start"] == g.data_start
    assert len(out["tensors"]) == len(g.tensors)
    for t in out["tensors"]:
        mine = g.tensors[t["name"]]
        assert t["type"] == mine.ttype
        assert tuple(reversed(t["ne"][: len(mine.shape)])) == mine.shape
        assert g.data_start + t["offset"] == mine.offset
        assert t["bytes"] == G.tensor_nbytes(mine.ttype, mine.shape)
    assert out["token0"] == "<unk>"
    g.close()
