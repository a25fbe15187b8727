"""Single-stream prompt prefill through the batched engine's tensor-core GEMMs (sd_ctx_opts.prefill_gemm).

A prompt of at least 256 tokens is written into the context's own K/V ring by batched forwards of 64 slices of
8 tokens; the decode that follows is the context's usual path.  Bars: the logits after such a prefill stay within
the north_star's 1e-2 relative of the CPU oracle and within 5e-3 of the same context prefilled by 8-token matvec
forwards (the bar of the batched path against the single-stream one: its attention runs on single fp16 Q and P);
the K/V rows of the first layer, which no attention precedes, agree to fp16 rounding.
"""
import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a CUDA GPU")]

LOGIT_RTOL = 1e-2
PATH_RTOL = 5e-3


@pytest.fixture(scope="module")
def mini(tmp_path_factory):
    from anetransformers_b200 import gguf as G
    path = str(tmp_path_factory.mktemp("pf") / "mini.gguf")
    G.write_synthetic_gguf(path, G.MINI, seed=7)
    return path


@pytest.fixture(scope="module")
def ctxs(mini):
    from anetransformers_b200.engine import Context
    a = Context(mini, max_seq=1024, prefill_gemm=False)
    b = Context(mini, max_seq=1024)
    yield a, b
    a.close()
    b.close()


def rel_err(x, ref):
    return float(np.max(np.abs(x.astype(np.float64) - ref)) / max(np.max(np.abs(ref)), 1e-30))


@pytest.mark.parametrize("n", [300, 513])
def test_gemm_prefill_logits_match_matvec_prefill_and_oracle(mini, ctxs, oracle, n):
    """n = 300: one GEMM forward with a short last slice; 513: two forwards (the second with one token)."""
    from anetransformers_b200 import gguf as G
    a, b = ctxs
    rng = np.random.default_rng(n)
    prompt = rng.integers(3, a.vocab, n).tolist()
    nxt = rng.integers(3, a.vocab, 5).tolist()
    a.prefill(prompt, 0)
    la, _ = a.forward(nxt, n)
    b.prefill(prompt, 0)
    lb, _ = b.forward(nxt, n)
    assert np.isfinite(lb).all()
    assert rel_err(lb, la.astype(np.float64)) < PATH_RTOL
    om = oracle.OracleModel(G.GGUFFile(mini), max_seq=1024)
    kv = om.new_kv()
    for i, t in enumerate(prompt):
        om.forward(kv, int(t), i)
    for j, t in enumerate(nxt):
        ref = om.forward(kv, int(t), n + j)
        assert rel_err(lb[j], ref) < LOGIT_RTOL, j
    om.free_kv(kv)


def test_gemm_prefill_first_layer_kv_and_offset_start(ctxs):
    """A 40-token matvec prefill, then 280 tokens from position 40 through the GEMMs: the first layer's K/V rows
    (whose inputs are the embeddings alone) equal the matvec path's to fp16 rounding of K-split sums."""
    a, b = ctxs
    rng = np.random.default_rng(3)
    prompt = rng.integers(3, a.vocab, 320).tolist()
    for c in (a, b):
        c.prefill(prompt[:40], 0)
        c.prefill(prompt[40:], 40)
    ka, va = a.kv_read(0, 0, 320)
    kb, vb = b.kv_read(0, 0, 320)
    for x, y in ((ka, kb), (va, vb)):
        x = x.view(np.float16).astype(np.float32)
        y = y.view(np.float16).astype(np.float32)
        assert np.max(np.abs(x - y)) <= 2e-3 * max(np.max(np.abs(x)), 1.0)
    # the positions the second call wrote are the GEMM path's: not all equal to the matvec path's deeper layers,
    # but within the path tolerance through the logits
    nxt = rng.integers(3, a.vocab, 5).tolist()
    la, _ = a.forward(nxt, 320)
    lb, _ = b.forward(nxt, 320)
    assert rel_err(lb, la.astype(np.float64)) < PATH_RTOL


def test_gemm_prefill_generate_matches_matvec_generate(ctxs):
    """sd_generate from a 400-token prompt (GEMM prefill of the first 392 tokens, the last chunk with logits on
    the matvec path): the greedy continuation agrees with the matvec-prefill context's until the first step
    whose top-2 logit gap is below the path tolerance."""
    a, b = ctxs
    rng = np.random.default_rng(11)
    prompt = rng.integers(3, a.vocab, 400).tolist()
    kw = dict(mode="greedy", max_tokens=12, temp=0.0, rep_penalty=1.0, ignore_eos=True)
    ta, _ = a.generate(prompt, **kw)
    tb, _ = b.generate(prompt, **kw)
    n = 0
    while n < min(len(ta), len(tb)) and ta[n] == tb[n]:
        n += 1
    if n < min(len(ta), len(tb)):
        # a divergence must start at a near-tie of the matvec path's logits at that step
        a.prefill(prompt + ta[:n], 0)
        lg, _ = a.forward([(prompt + ta[:n])[-1]], len(prompt) + n - 1)
        top = np.sort(lg[0].astype(np.float64))[-2:]
        assert top[1] - top[0] <= PATH_RTOL * np.max(np.abs(lg[0])), (n, ta, tb)
