"""Writes tests/golden/spec_golden.json from the reference's own mistral/speculative.h (built by `make -C oracle ref`
into oracle/_ref/libspec_ref.so against the stand-ins in oracle/ref_stub/).

Cases, all seeded:
  - n-gram drafter (speculative.h:395-464): histories over a small alphabet (so n-grams repeat), split into a prompt
    and pushed tokens, every ngram_n / max_draft edge the code handles (defaults for <= 0, the SPEC_MAX_DRAFT clip,
    the 16-token pattern cap, history shorter than n, a match only in the skipped tail);
  - spec_accept (:121-198) at temperature <= 0 (argmax acceptance, logits with ties) and > 0 (Leviathan
    acceptance and resampling), with arc4random fed the Philox draws philox(seed, 0), philox(seed, 1), ...;
  - spec_softmax (:37-57) and spec_sample_probs (:60-68).
Float arrays are stored as base64 of little-endian float32 bytes.

usage: python tests/golden/make_spec_golden.py   (from the repository root, after `make -C oracle ref`)
"""
import base64
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from oracle import ref_spec as R  # noqa: E402

OUT = os.path.join(ROOT, "tests", "golden", "spec_golden.json")
VOCAB = 32
N_DRAWS = 40


def f32b64(a) -> str:
    return base64.b64encode(np.ascontiguousarray(a, "<f4").tobytes()).decode()


def ngram_cases(rng):
    cases = []
    for ngram_n, max_draft in [(3, 4), (2, 8), (4, 12), (1, 4), (0, 4), (-1, 0), (5, -3), (17, 8), (20, 4), (3, 1)]:
        for k in range(6):
            hlen = int(rng.integers(0, 120)) if k else int(rng.integers(0, 4))
            alpha = int(rng.integers(2, 9))
            hist = rng.integers(0, alpha, hlen).tolist()
            if k in (2, 3, 4) and hlen > 24:
                # plant a repeat: the last tokens (and the current one) copy an earlier stretch
                a = int(rng.integers(0, hlen // 2))
                span = min(int(rng.integers(4, 24)), hlen - a - 1)
                hist = hist[:hlen - span] + hist[a:a + span]
            if k == 5 and hlen > 8:
                # the only match of the pattern is the tail itself, which the scan skips
                hist = list(range(100, 100 + hlen))
            cut = int(rng.integers(0, hlen + 1))
            current = int(rng.integers(0, alpha)) if k != 5 else (hist[-1] + 1 if hist else 0)
            if k in (2, 3) and hlen > 24:
                current = hist[a + span] if a + span < len(hist) else current
            toks, probs = R.ngram_draft(hist[:cut], hist[cut:], ngram_n, max_draft, current)
            cases.append({"prompt": hist[:cut], "pushed": hist[cut:], "ngram_n": ngram_n, "max_draft": max_draft,
                          "current": current, "tokens": toks, "probs": f32b64(probs)})
    return cases


def accept_cases(rng):
    cases = []
    temps = [0.0, -1.0, 0.0, 0.3, 0.7, 1.0, 1.5, 0.7]
    for i in range(64):
        temp = temps[i % len(temps)]
        n_draft = int(rng.integers(1, 9))
        if temp <= 0:
            logits = rng.integers(0, 4, (n_draft, VOCAB)).astype(np.float32)  # many ties: first index wins
        else:
            logits = (rng.standard_normal((n_draft, VOCAB)) * rng.uniform(0.5, 4.0)).astype(np.float32)
        tokens = []
        for j in range(n_draft):
            am = int(np.argmax(logits[j]))
            tokens.append(am if rng.random() < 0.85 else int(rng.integers(0, VOCAB)))
        kind = i % 3
        if kind == 0:
            probs = np.full(n_draft, 0.9, np.float32)
        elif kind == 1:
            probs = rng.uniform(0.01, 1.0, n_draft).astype(np.float32)
        else:
            probs = np.where(rng.random(n_draft) < 0.3, 0.0, 0.5).astype(np.float32)
        seed = int(rng.integers(0, 2**31))
        draws = [O.philox(seed, c) for c in range(N_DRAWS)]
        acc, used = R.spec_accept(probs, logits, tokens, temp, draws)
        cases.append({"temp": temp, "logits": f32b64(logits), "n_draft": n_draft, "draft_tokens": tokens,
                      "draft_probs": f32b64(probs), "seed": seed, "accepted": acc, "draws_used": used})
    return cases


def softmax_cases(rng):
    cases = []
    for i in range(12):
        temp = [0.7, 1.0, 0.3, 2.0][i % 4]
        logits = (rng.standard_normal(64) * 3).astype(np.float32)
        probs = R.spec_softmax(logits, temp)
        seed = int(rng.integers(0, 2**31))
        idx, used = R.spec_sample_probs(probs, [O.philox(seed, c) for c in range(4)])
        cases.append({"temp": temp, "logits": f32b64(logits), "probs": f32b64(probs), "seed": seed, "sample": idx,
                      "draws_used": used})
    return cases


def main():
    if not R.available():
        sys.exit("oracle/_ref/libspec_ref.so is missing: run `make -C oracle ref` where the reference tree is present")
    rng = np.random.default_rng(20261202)
    data = {"source": "mistral/speculative.h compiled by oracle/Makefile (_ref/libspec_ref.so)", "vocab": VOCAB,
            "ngram": ngram_cases(rng), "accept": accept_cases(rng), "softmax": softmax_cases(rng)}
    with open(OUT, "w") as f:
        json.dump(data, f, separators=(",", ":"))
    print(OUT, len(data["ngram"]), len(data["accept"]), len(data["softmax"]))


if __name__ == "__main__":
    main()
