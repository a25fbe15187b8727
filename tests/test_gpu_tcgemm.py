"""The tcgen05 GEMM of batched forwards (sd_tcgemm.cu: tcgen05.mma kind::i8, accumulators in TMEM) against
the mma.sync GEMM (sd_wgemm.cu) and the CPU oracle.

Both GEMMs take exact int32 block sums and run the same fp32 operations per block in the same K order, so
a forward through either gives the same logits bit for bit (sd_batch_set_gemm switches between them); the
logits also stay within the north_star's 1e-2 relative bar of the oracle.  Shapes cover a token count that
is not a multiple of 8 (ragged last n8 tile, N padded to 16), more than one token tile, the gate|up SiLU
epilogue and a K-split o-proj / down (partial slices).
"""
import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a CUDA GPU")]

LOGIT_RTOL = 1e-2


@pytest.fixture(scope="module")
def mini(tmp_path_factory):
    from anetransformers_b200 import gguf as G
    path = str(tmp_path_factory.mktemp("tc") / "mini.gguf")
    G.write_synthetic_gguf(path, G.MINI, seed=5)
    return path


@pytest.fixture(scope="module")
def ctx(mini):
    from anetransformers_b200.engine import Context
    c = Context(mini, max_seq=512)
    yield c
    c.close()


def rel_err(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b)) / max(np.max(np.abs(b)), 1e-30))


def _forward_both(ctx, n_streams, T, seed, n0=24):
    from anetransformers_b200.engine import BatchContext
    rng = np.random.default_rng(seed)
    prom = rng.integers(3, ctx.vocab, (n_streams, n0)).astype(np.int32)
    nxt = rng.integers(3, ctx.vocab, (n_streams, T)).astype(np.int32)
    pos = (n0 - rng.integers(0, 4, n_streams)).astype(np.int32)
    out = {}
    bc = BatchContext(ctx, n_streams, max_seq=256, width=8)
    try:
        for mode in (BatchContext.GEMM_MMA, BatchContext.GEMM_TC):
            bc.set_gemm(mode)
            bc.prefill(prom)
            out[mode] = bc.forward(nxt, pos)
    finally:
        bc.close()
    return prom, nxt, pos, out[BatchContext.GEMM_MMA], out[BatchContext.GEMM_TC]


@pytest.mark.parametrize("n_streams,T", [(3, 5), (13, 5), (16, 8), (40, 5)])
def test_tcgen05_forward_bit_identical_to_mma_sync(ctx, n_streams, T):
    """M = 15 (one 16-token tile), 65 (ragged n8 tile), 128 (one full 128-token tile), 200 (two tiles)."""
    _, _, _, lg_mma, lg_tc = _forward_both(ctx, n_streams, T, seed=n_streams * 10 + T)
    assert np.isfinite(lg_tc).all()
    np.testing.assert_array_equal(lg_tc.view(np.uint32), lg_mma.view(np.uint32))


def test_tcgen05_forward_matches_oracle(mini, ctx, oracle):
    from anetransformers_b200 import gguf as G
    prom, nxt, pos, _, lg = _forward_both(ctx, 13, 5, seed=77)
    om = oracle.OracleModel(G.GGUFFile(mini), max_seq=256)
    for s in (0, 6, 12):
        kv = om.new_kv()
        for i in range(pos[s]):
            om.forward(kv, int(prom[s, i]), i)
        for j in range(5):
            ref = om.forward(kv, int(nxt[s, j]), int(pos[s]) + j)
            assert rel_err(lg[s, j], ref) < LOGIT_RTOL, (s, j)
        om.free_kv(kv)


def test_tcgen05_default_from_64_tokens(ctx):
    """AUTO picks tcgen05 at 13 streams x 5 tokens (65 >= 64) and mma.sync for one token per stream; the
    width-1 and width-5 logits of a stream stay bit-identical across the switch (same K splits)."""
    from anetransformers_b200.engine import BatchContext
    rng = np.random.default_rng(5)
    n, T, n0 = 13, 5, 16
    prom = rng.integers(3, ctx.vocab, (n, n0)).astype(np.int32)
    nxt = rng.integers(3, ctx.vocab, (n, T)).astype(np.int32)
    pos = np.full(n, n0, np.int32)
    bc = BatchContext(ctx, n, max_seq=256, width=8)
    try:
        bc.prefill(prom)
        lg5 = bc.forward(nxt, pos)
        bc.prefill(prom)
        for j in range(T):
            lg1 = bc.forward(nxt[:, j:j + 1], pos + j)
            np.testing.assert_array_equal(lg1[:, 0].view(np.uint32), lg5[:, j].view(np.uint32))
    finally:
        bc.close()


def test_tcgen05_ngram_decode_equals_mma_decode(ctx):
    """Temp-0 n-gram speculative decode of 16 streams (verify M = 80 on tcgen05) emits the same tokens as the
    same decode on mma.sync."""
    from anetransformers_b200.engine import BatchContext
    rng = np.random.default_rng(21)
    n = 16
    seg = rng.integers(3, ctx.vocab, (4, 16))
    prom = np.stack([np.concatenate([seg[(s + i) % 4] for i in range(4)]) for s in range(n)]).astype(np.int32)
    kw = dict(mode="ngram", spec_k=4, ngram_n=3, max_tokens=40, temp=0.0, rep_penalty=1.0, ignore_eos=True)
    res = {}
    bc = BatchContext(ctx, n, max_seq=256, width=5)
    try:
        for mode in (BatchContext.GEMM_MMA, BatchContext.GEMM_TC):
            bc.set_gemm(mode)
            res[mode] = bc.generate(prom, **kw)
    finally:
        bc.close()
    (a, sa), (b, sb) = res[BatchContext.GEMM_MMA], res[BatchContext.GEMM_TC]
    for s in range(n):
        assert a[s] == b[s], s
    assert sa["total_accepted"] == sb["total_accepted"]
