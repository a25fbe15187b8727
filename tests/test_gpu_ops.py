"""GPU parity of the single-op layer against the CPU oracle, through the C ABI.

Bars (north_star): Q8_0 codes + scales and per-block int32 SDOT sums bit-exact; matvec fp32 outputs
within a bound derived from the exact block sums: |y_gpu - y_ref| <= 2e-6 * sum_b |wd*xd*isum| + 1e-30
(fp32 re-association of the same terms; the reference's own order is unpinned under -ffast-math).
"""
import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a CUDA GPU")]

MV_RTOL = 2e-6


@pytest.fixture(scope="module")
def dq():
    from anetransformers_b200 import dequant
    return dequant


def rand_q4(rng, rows, cols):
    from anetransformers_b200.gguf import random_q4_0
    return random_q4_0(rng, rows, cols)


def term_bound(oracle, W, xq):
    isum = oracle.block_sums(W, xq).astype(np.float64)
    s = W["d"].astype(np.float64) * xq["d"].astype(np.float64)[None, :]
    return np.abs(s * isum).sum(axis=1)


def edge_inputs(n=4096, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n).astype(np.float32)
    x[0:32] = 0.0                                     # amax == 0 block -> d = 0, q = 0
    x[32:64] = 0.0
    x[32] = -1e-38                                    # denormal-sized amax
    x[64:96] = np.float32(127.0)                      # all at amax
    x[96:128] = np.linspace(-1, 1, 32, dtype=np.float32) * np.float32(3e30)   # huge
    blk = np.arange(32, dtype=np.float32) - 15.5      # x*id lands on .5 boundaries
    x[128:160] = blk * np.float32(1.0)
    x[160:192] = -0.0
    x[192:224] = np.float32(1e-3) * np.sign(rng.standard_normal(32)).astype(np.float32)
    return x


@pytest.mark.parametrize("S", [1, 5, 8])
def test_quantizer_bit_exact(oracle, dq, S):
    import torch
    rng = np.random.default_rng(100 + S)
    n = 4096
    x = rng.standard_normal((S, n)).astype(np.float32) * rng.uniform(0.01, 50, (S, 1)).astype(np.float32)
    x[0] = edge_inputs(n, S)
    act = dq.quantize_dev(torch.from_numpy(x).cuda())
    blocks = dq.q8_to_blocks_dev(act).cpu().numpy().view(oracle.Q8_0_DTYPE).reshape(S, n // 32)
    for s in range(S):
        ref = oracle.quantize_q8_0(x[s])
        np.testing.assert_array_equal(blocks[s]["d"].view(np.uint32), ref["d"].view(np.uint32))
        np.testing.assert_array_equal(blocks[s]["qs"], ref["qs"])
        # code sums plane
        np.testing.assert_array_equal(act.sum[s].cpu().numpy(), ref["qs"].astype(np.int32).sum(axis=1))


def test_host_quantize_dropin(oracle, dq):
    x = edge_inputs(14336, 9)
    got = dq.quantize_f32_to_q8_0(x)
    ref = oracle.quantize_q8_0(x)
    np.testing.assert_array_equal(got["d"].view(np.uint32), ref["d"].view(np.uint32))
    np.testing.assert_array_equal(got["qs"], ref["qs"])


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1024, 14336), (1000, 1024)])
def test_block_sums_bit_exact(oracle, dq, rows, cols):
    rng = np.random.default_rng(rows + cols)
    W = rand_q4(rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    xq = oracle.quantize_q8_0(x)
    ref = oracle.block_sums(W, xq)
    rows16 = rows // 16 * 16
    if rows16 != rows:
        with pytest.raises(Exception):
            dq.block_sums_dev(dq.QMat(W), dq.blocks_to_q8_dev(xq, 1, cols))
        return
    got = dq.block_sums_dev(dq.QMat(W), dq.blocks_to_q8_dev(xq, 1, cols)).cpu().numpy()
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("rows,cols,S", [(4096, 4096, 1), (4096, 4096, 5), (14336, 4096, 5), (4096, 14336, 5),
                                         (32000, 4096, 1), (1000, 2048, 3), (6144, 4096, 8)])
def test_matvec_matches_oracle(oracle, dq, rows, cols, S):
    import torch
    rng = np.random.default_rng(rows * 7 + cols + S)
    W = rand_q4(rng, rows, cols)
    x = rng.standard_normal((S, cols)).astype(np.float32)
    xq = np.stack([oracle.quantize_q8_0(x[s]) for s in range(S)])
    qm = dq.QMat(W)
    act = dq.blocks_to_q8_dev(xq, S, cols)
    y = dq.matvec_dev(qm, act).cpu().numpy()
    for s in range(S):
        ref = oracle.matvec(W, xq[s])
        bound = MV_RTOL * term_bound(oracle, W, xq[s]) + 1e-30
        err = np.abs(y[s].astype(np.float64) - ref.astype(np.float64))
        assert np.all(err <= bound), (s, float(err.max()), float(bound[np.argmax(err)]))
        # the two reference accumulation forms bracket the same tolerance
        ref2 = oracle.matvec(W, xq[s], oracle.ACC_MULADD)
        assert np.all(np.abs(ref2 - ref) <= bound)


@pytest.mark.parametrize("rows,cols,S", [(4096, 4096, 5), (4096, 14336, 8), (1024, 14336, 5), (2048, 4096, 2),
                                         (2048, 4096, 3)])
def test_matvec_batch_invariant(oracle, dq, rows, cols, S):
    """A token's result does not depend on the other tokens of the batch (S=1 vs S, bitwise), also for
    long rows whose K range is split across CTAs at the larger S, and on both sides of the staging's switch
    from per-thread 16-byte pieces (S <= 2) to one warp per block (S >= 3)."""
    import torch
    rng = np.random.default_rng(42 + cols)
    W = rand_q4(rng, rows, cols)
    x = rng.standard_normal((S, cols)).astype(np.float32)
    qm = dq.QMat(W)
    actS = dq.quantize_dev(torch.from_numpy(x).cuda())
    yS = dq.matvec_dev(qm, actS).cpu().numpy()
    for s in range(S):
        act1 = dq.quantize_dev(torch.from_numpy(x[s:s + 1]).cuda())
        y1 = dq.matvec_dev(qm, act1).cpu().numpy()
        np.testing.assert_array_equal(y1[0].view(np.uint32), yS[s].view(np.uint32))


def test_host_matvec_dropin(oracle, dq):
    rng = np.random.default_rng(5)
    W = rand_q4(rng, 2048, 4096)
    xq = oracle.quantize_q8_0(rng.standard_normal(4096).astype(np.float32))
    y = dq.q4_0_q8_0_matvec_sdot_parallel(W, xq, 2048, 4096)
    ref = oracle.matvec(W, xq)
    assert np.all(np.abs(y - ref) <= MV_RTOL * term_bound(oracle, W, xq) + 1e-30)
    # cached second call gives identical bits
    y2 = dq.q4_0_q8_0_matvec_sdot_parallel(W, xq, 2048, 4096)
    np.testing.assert_array_equal(y, y2)


def test_bad_shapes_rejected(dq):
    from anetransformers_b200 import SpecDecError
    rng = np.random.default_rng(1)
    with pytest.raises(SpecDecError):
        dq.QMat(rand_q4(rng, 64, 992))          # cols not a multiple of 1024
