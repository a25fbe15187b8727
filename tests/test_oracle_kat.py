"""Pin the CPU oracle to the reference's own known-answer tests (tests/test_mistral.m).

These replay, on the oracle restatement, every KAT the reference's test-suite holds for the decode
path: Q4_0 dequant values (test_mistral.m:742-779), RoPE pos-0 identity and norm preservation
(:414-471), GQA head broadcast vs expanded MHA (:474-518), RMSNorm / SiLU / softmax KATs (:921-983).
"""
import numpy as np
import pytest


def _f16(x):
    return np.float16(x).view(np.uint16)


def test_q4_0_dequant_kat(oracle):
    # test_mistral.m:742-779: d = 0.1*(b+1), qs[j] = (j%16) | ((j+1)%16)<<4 -> val[0] = -0.8, val[16] = -0.7
    nb = 8
    blocks = np.zeros(nb, dtype=oracle.Q4_0_DTYPE)
    for b in range(nb):
        blocks[b]["d"] = np.float16(0.1 * (b + 1))
        blocks[b]["qs"] = [(j % 16) | (((j + 1) % 16) << 4) for j in range(16)]
    out = oracle.dequant(blocks)
    assert abs(out[0] - (-0.8)) < 0.01 and abs(out[16] - (-0.7)) < 0.01
    # exact: d is the fp16 value, products are exact in fp32
    d0 = float(np.float16(0.1))
    assert out[0] == np.float32(d0 * -8) and out[16] == np.float32(d0 * -7)
    # full expected table
    exp = []
    for b in range(nb):
        d = float(np.float16(0.1 * (b + 1)))
        lo = [d * ((j % 16) - 8) for j in range(16)]
        hi = [d * (((j + 1) % 16) - 8) for j in range(16)]
        exp += lo + hi
    np.testing.assert_array_equal(out, np.array(exp, np.float32))


def test_rope_pos0_identity_and_norm(oracle):
    # test_mistral.m:414-471: S=4, nh=8, hd=32, theta 1e4, q[i]=0.1*(i%17-8), k[i]=0.1*(i%13-6)
    S, nh, hd = 4, 8, 32
    q = (0.1 * (np.arange(S * nh * hd) % 17 - 8)).astype(np.float32).reshape(S, nh * hd)
    k = (0.1 * (np.arange(S * nh * hd) % 13 - 6)).astype(np.float32).reshape(S, nh * hd)
    th = oracle.rope_theta(hd, 10000.0)
    qr = np.stack([oracle.apply_rope(q[t], k[t], t, th, nh, nh, hd)[0] for t in range(S)])
    assert np.max(np.abs(qr[0] - q[0])) <= 1e-6                      # pos 0 is the identity
    nb, na = np.linalg.norm(q[1]), np.linalg.norm(qr[1])              # rotation preserves norm
    assert abs(nb - na) / nb < 1e-5


def test_gqa_broadcast_matches_expanded_mha(oracle):
    # test_mistral.m:474-518: nh=8, nkv=2 (ratio 4) vs expanded KV heads, tol 1e-5
    rng = np.random.default_rng(7)
    S, nh, nkv, hd = 8, 8, 2, 32
    max_seq = 16
    q = rng.uniform(-0.5, 0.5, (S, nh * hd)).astype(np.float32)
    k = rng.uniform(-0.5, 0.5, (S, nkv * hd)).astype(np.float32).astype(np.float16).view(np.uint16)
    v = rng.uniform(-0.5, 0.5, (S, nkv * hd)).astype(np.float32).astype(np.float16).view(np.uint16)
    kc = np.zeros((max_seq, nkv * hd), np.uint16); kc[:S] = k
    vc = np.zeros((max_seq, nkv * hd), np.uint16); vc[:S] = v
    ke = np.zeros((max_seq, nh * hd), np.uint16)
    ve = np.zeros((max_seq, nh * hd), np.uint16)
    for h in range(nh):
        ke[:S, h * hd:(h + 1) * hd] = k[:, (h // 4) * hd:(h // 4 + 1) * hd]
        ve[:S, h * hd:(h + 1) * hd] = v[:, (h // 4) * hd:(h // 4 + 1) * hd]
    for t in range(S):
        a = oracle.attention(q[t], kc, vc, nh, 4, hd, max_seq, t)
        b = oracle.attention(q[t], ke, ve, nh, 1, hd, max_seq, t)
        assert np.max(np.abs(a - b)) <= 1e-5


def test_rmsnorm_silu_softmax_kats(oracle):
    # test_mistral.m:921-983
    out = oracle.rmsnorm(np.ones(4, np.float32), np.ones(4, np.float32), 1e-5)
    assert np.max(np.abs(out - 1.0)) < 1e-4
    x = np.array([0.0, 1.0, -1.0, 10.0, -10.0], np.float32)
    exp = x / (1.0 + np.exp(-x.astype(np.float64)))
    got = oracle.silu_mul(x, np.ones_like(x))
    assert np.max(np.abs(got - exp)) < 1e-4
    assert np.max(np.abs(oracle.softmax(np.ones(4, np.float32)) - 0.25)) < 1e-6
    sm = oracle.softmax(np.array([100, 0, 0, 0], np.float32))
    assert sm[0] > 0.999 and sm[1] < 0.001


def test_quantizer_follows_dequant_h(oracle):
    # dequant.h:545-599 semantics: d = amax/127, amax == 0 -> zeros, RNE, saturate
    x = np.zeros(64, np.float32)
    x[32:] = np.linspace(-3, 3, 32, dtype=np.float32)
    q = oracle.quantize_q8_0(x)
    assert q[0]["d"] == 0 and not q[0]["qs"].any()
    d = np.float32(3.0) / np.float32(127.0)
    assert q[1]["d"] == d
    idv = np.float32(1.0) / d
    exp = np.rint((x[32:] * idv).astype(np.float32)).astype(np.int64).clip(-128, 127)
    np.testing.assert_array_equal(q[1]["qs"], exp)
    assert q[1]["qs"][0] == -127 and q[1]["qs"][-1] == 127


def test_quantizer_recip_variant_mismatch_rate(oracle):
    """-ffast-math may rewrite amax/127 as amax*(1/127); report how often codes differ."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal(4096 * 64).astype(np.float32)
    a = oracle.quantize_q8_0(x, oracle.QUANT_IEEE)
    b = oracle.quantize_q8_0(x, oracle.QUANT_RECIP)
    code_mismatch = np.mean(a["qs"] != b["qs"])
    d_mismatch = np.mean(a["d"] != b["d"])
    assert code_mismatch < 1e-3      # rare: only ties at a rounding boundary move
    assert d_mismatch < 0.6
