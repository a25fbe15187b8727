"""The parity oracle's speculative-decoding functions against the reference's own mistral/speculative.h.

The reference header compiles here against stand-ins for its Apple-only dependencies (oracle/ref_stub/, built by
`make -C oracle ref` into oracle/_ref/libspec_ref.so): the n-gram drafter and spec_accept's control flow run as the
reference wrote them; vDSP / vForce calls are restated with libm as the oracle restates them, and arc4random is fed
the same Philox draws the oracle and the device consume.

  - golden: tests/golden/spec_golden.json, written by tests/golden/make_spec_golden.py from that build, held against
    the oracle everywhere (the reference tree is not needed);
  - live: seeded random cases against the build itself, where it exists.
Bars: drafts (tokens and 0.9 probabilities), accepted tokens and the number of draws consumed are identical;
spec_softmax probabilities are bit-identical.
"""
import base64
import json
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden", "spec_golden.json")


def f32(s: str) -> np.ndarray:
    return np.frombuffer(base64.b64decode(s), "<f4").astype(np.float32)


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def ref():
    from oracle import ref_spec as R
    if not R.available():
        pytest.skip("oracle/_ref/libspec_ref.so not built (needs the reference tree: make -C oracle ref)")
    return R


def test_ngram_drafter_matches_reference_golden(oracle, golden):
    cases = golden["ngram"]
    assert len(cases) >= 60 and sum(1 for c in cases if c["tokens"]) >= 20
    for c in cases:
        toks, probs = oracle.ngram_draft(c["prompt"], c["pushed"], c["ngram_n"], c["max_draft"], c["current"])
        assert toks == c["tokens"], c
        assert np.array_equal(np.float32(probs), f32(c["probs"])), c


def test_spec_accept_matches_reference_golden(oracle, golden):
    V = golden["vocab"]
    cases = golden["accept"]
    assert len(cases) >= 64
    assert any(c["temp"] <= 0 for c in cases) and any(c["temp"] > 0 and len(c["accepted"]) > 1 for c in cases)
    for c in cases:
        lg = f32(c["logits"]).reshape(c["n_draft"], V)
        acc, counter = oracle.spec_accept(f32(c["draft_probs"]), lg, c["draft_tokens"], c["temp"], seed=c["seed"])
        assert acc == c["accepted"], c
        assert counter == c["draws_used"], c


def test_spec_softmax_and_sample_match_reference_golden(oracle, golden):
    for c in golden["softmax"]:
        p = oracle.spec_softmax(f32(c["logits"]), c["temp"])
        assert np.array_equal(p, f32(c["probs"]))
        idx, counter = oracle.spec_sample_probs(p, seed=c["seed"])
        assert (idx, counter) == (c["sample"], c["draws_used"])


def test_ngram_drafter_matches_reference_live(oracle, ref):
    rng = np.random.default_rng(41)
    nonempty = 0
    for _ in range(600):
        hlen = int(rng.integers(0, 200))
        alpha = int(rng.integers(2, 12))
        hist = rng.integers(0, alpha, hlen).tolist()
        cut = int(rng.integers(0, hlen + 1))
        n, md = int(rng.integers(-1, 19)), int(rng.integers(-2, 14))
        cur = int(rng.integers(0, alpha))
        want = ref.ngram_draft(hist[:cut], hist[cut:], n, md, cur)
        got = oracle.ngram_draft(hist[:cut], hist[cut:], n, md, cur)
        assert got[0] == want[0] and np.array_equal(np.float32(got[1]), np.float32(want[1])), (hist, cut, n, md, cur)
        nonempty += bool(want[0])
    assert nonempty > 100


@pytest.mark.parametrize("temp", [0.0, 0.5, 1.0, 2.0])
def test_spec_accept_matches_reference_live(oracle, ref, temp):
    rng = np.random.default_rng(int(temp * 10) + 3)
    V = 48
    for i in range(150):
        nd = int(rng.integers(1, 9))
        if temp <= 0:
            lg = rng.integers(0, 3, (nd, V)).astype(np.float32)
        else:
            lg = (rng.standard_normal((nd, V)) * rng.uniform(0.3, 5.0)).astype(np.float32)
        toks = [int(np.argmax(lg[j])) if rng.random() < 0.8 else int(rng.integers(0, V)) for j in range(nd)]
        dp = rng.choice([0.0, 0.05, 0.5, 0.9, 1.0], nd).astype(np.float32)
        seed = int(rng.integers(0, 2**31))
        want, used = ref.spec_accept(dp, lg, toks, temp, [oracle.philox(seed, c) for c in range(64)])
        got, counter = oracle.spec_accept(dp, lg, toks, temp, seed=seed)
        assert got == want and counter == used, (i, temp, toks, dp.tolist())
