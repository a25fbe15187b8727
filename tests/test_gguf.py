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


def test_reference_parser_reads_kquant_model(tmp_path):
    """A model with a Q4_K embedding and a Q6_K LM head (the real Mistral Q4_0 files ship a Q6_K head): the
    reference's parser finds every tensor at the writer's offsets with the writer's types; its own size table
    (gguf_loader.h:335-344) knows Q4_K (144 bytes per 256 values) but not Q6_K, whose 210-byte block is
    block_q6_K of mistral/dequant.h:283-289 (checked here through the offsets of the tensors that follow)."""
    cfg = dataclasses.replace(G.MINI, lm_head_type="q6_k", embd_type="q4_k")
    path = str(tmp_path / "kq.gguf")
    G.write_synthetic_gguf(path, cfg, seed=12)
    out = json.loads(subprocess.check_output([_ref_dump(), path]))
    g = G.GGUFFile(path)
    types = {t["name"]: t["type"] for t in out["tensors"]}
    assert types["token_embd.weight"] == 12 and types["output.weight"] == 14
    for t in out["tensors"]:
        mine = g.tensors[t["name"]]
        assert t["type"] == mine.ttype and g.data_start + t["offset"] == mine.offset
        if mine.ttype != 14:
            assert t["bytes"] == G.tensor_nbytes(mine.ttype, mine.shape)
    assert G.tensor_nbytes(14, (2048, 1024)) == 2048 * 4 * 210
    assert g.array("output.weight").dtype.itemsize == 210 and g.array("token_embd.weight").dtype.itemsize == 144
    g.close()


def test_kquant_oracle_dequant_properties():
    """Q6_K / Q4_K dequant of the oracle (mistral/dequant.h:47-113, :292-306): Q6_K values are (d*sc)*q with q in
    -32..31; Q4_K values are fp16 and lie within [-dmin*63, d*63*15]; the K-quant matvec equals the float64 dot
    of the dequantised rows to fp32 accumulation error."""
    from oracle import oracle as O
    rng = np.random.default_rng(3)
    W6 = G.random_q6_k(rng, 16, 512)
    d6 = O.dequant_q6_k(W6)
    q = d6 / (W6["d"].astype(np.float32)[..., None].repeat(256, axis=-1).reshape(16, 512) *
              np.repeat(W6["scales"].astype(np.float32), 16, axis=-1).reshape(16, 512))
    qi = q[np.isfinite(q)]
    assert np.allclose(qi, np.round(qi)) and qi.min() >= -32 and qi.max() <= 31
    W4 = G.random_q4_k(rng, 16, 512)
    d4 = O.dequant_q4_k(W4).astype(np.float32)
    assert np.all(np.abs(d4) <= 63 * 15 * W4["d"].astype(np.float32).max() + 63 * W4["dmin"].astype(np.float32).max())
    x = rng.standard_normal(512).astype(np.float32)
    for W, d, t in ((W6, d6, O.TYPE_Q6_K), (W4, d4, O.TYPE_Q4_K)):
        y = O.matvec_kq(W, x, t)
        ref = d.astype(np.float64) @ x
        assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(d) @ np.abs(x))
