"""GPU parity of the K-quant paths against the CPU oracle: the fp32-activation Q6_K / Q4_K matvec (the LM head of
the real Mistral Q4_0 GGUFs is Q6_K) and a whole model with a Q6_K LM head and a Q4_K embedding.

The device and the oracle compute the same weights (Q6_K: (d * sc) * q, exact in fp32; Q4_K: the reference's fp16
dequant) and accumulate in the same order (value n into lane n % 4 by fused multiply-add, lanes added pairwise), so
the matvec is bit-identical.  The model's logits are held to the north_star bar (1e-2 relative), and the persistent
and kernel-per-op forwards to bit equality.
"""
import dataclasses

import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a CUDA GPU")]

TYPE_Q4_K, TYPE_Q6_K = 12, 14


@pytest.mark.parametrize("ttype", [TYPE_Q6_K, TYPE_Q4_K])
@pytest.mark.parametrize("rows,cols", [(1000, 4096), (32000, 1024), (257, 14336)])
def test_kq_matvec_bit_exact_vs_oracle(oracle, ttype, rows, cols):
    from anetransformers_b200 import dequant as dq, gguf as G
    rng = np.random.default_rng(rows + cols + ttype)
    W = (G.random_q6_k if ttype == TYPE_Q6_K else G.random_q4_k)(rng, rows, cols)
    for trial in range(2):
        x = (rng.standard_normal(cols) * rng.uniform(0.5, 4)).astype(np.float32)
        y = dq.kq_matvec(W, x, ttype)
        ref = oracle.matvec_kq(W, x, ttype)
        np.testing.assert_array_equal(y.view(np.uint32), ref.view(np.uint32))


@pytest.fixture(scope="module")
def kq_model(tmp_path_factory):
    from anetransformers_b200 import gguf as G
    cfg = dataclasses.replace(G.MINI, lm_head_type="q6_k", embd_type="q4_k")
    path = str(tmp_path_factory.mktemp("kq") / "mini_kq.gguf")
    G.write_synthetic_gguf(path, cfg, seed=6)
    return path


def test_model_with_q6k_head_and_q4k_embedding_matches_oracle(kq_model, oracle):
    from anetransformers_b200 import gguf as G
    from anetransformers_b200.engine import Context
    ctx = Context(kq_model, max_seq=256)
    om = oracle.OracleModel(G.GGUFFile(kq_model), max_seq=256)
    kv = om.new_kv()
    try:
        toks = np.random.default_rng(81).integers(3, ctx.vocab, 10).tolist()
        for i, t in enumerate(toks):
            ref = om.forward(kv, t, i)
            lg, am = ctx.forward([t], i)
            assert np.max(np.abs(lg[0] - ref)) <= 1e-2 * np.max(np.abs(ref)), i
            s = np.sort(ref)
            if s[-1] - s[-2] > 1e-3 * np.max(np.abs(ref)):
                assert am[0] == int(np.argmax(ref)), i
        # the embedding is Q4_K: its rows are the reference's fp16 dequant, exactly
        np.testing.assert_array_equal(ctx.embed_token(toks[0]), om.embed(toks[0]))
    finally:
        om.free_kv(kv)
        om.close()
        ctx.close()


def test_kq_model_paths_bitwise_and_spec_equals_greedy(kq_model):
    from anetransformers_b200 import _lib
    from anetransformers_b200.engine import BatchContext, Context
    fused = Context(kq_model, max_seq=256, forward_kernel=1)
    perop = Context(kq_model, max_seq=256, forward_kernel=0)
    try:
        rng = np.random.default_rng(82)
        prompt = rng.integers(3, fused.vocab, 12).tolist()
        for c in (fused, perop):
            c.prefill(prompt, 0)
        toks = rng.integers(3, fused.vocab, 5).tolist()
        a, am_a = fused.forward(toks, 12)
        b, am_b = perop.forward(toks, 12)
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
        np.testing.assert_array_equal(am_a, am_b)
        pool = [rng.integers(3, fused.vocab, 8).tolist() for _ in range(3)]
        p2 = sum((pool[i % 3] for i in range(6)), [])
        kw = dict(max_tokens=24, temp=0.0, rep_penalty=1.0, ignore_eos=True)
        greedy, _ = fused.generate(p2, mode="greedy", **kw)
        spec, st = fused.generate(p2, mode="ngram", spec_k=4, ngram_n=3, **kw)
        n = min(len(greedy), len(spec))
        assert n >= 24 and spec[:n] == greedy[:n]
        with pytest.raises(_lib.SpecDecError):
            BatchContext(fused, 2, max_seq=64, width=5)   # batched serving needs a Q4_0 head
    finally:
        fused.close()
        perop.close()
