"""Regenerate tests/golden/tokenizer_golden.json: the reference's own tokenizer (mistral/tokenizer.h, compiled
from the reference tree into oracle/_ref/tok_dump by `make -C oracle ref`) run on the seeded bpe test vocabulary
(anetransformers_b200.gguf.bpe_vocab, written into a small synthetic model) and a fixed set of texts.

    python tests/golden/make_tokenizer_golden.py [--ref-bin oracle/_ref/tok_dump]

The fixture stores, per text, the ids of tokenizer_encode(text, add_bos=1) and the bytes of tokenizer_decode(ids);
tests/test_tokenizer.py checks the library's tokenizer against it without the reference tree.
"""
import argparse
import dataclasses
import json
import os
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

VOCAB_SEED = 0


def texts():
    """Inputs covering the encoder's paths: merges (with equal-score runs), capitals, digits, punctuation,
    multi-byte characters inside and outside the vocabulary (byte fallback), spaces in every position,
    repeated characters, a long word, the chat template, and the empty text."""
    import numpy as np
    from anetransformers_b200 import gguf as G
    words = G.bpe_corpus_words(VOCAB_SEED)
    rng = np.random.default_rng(99)
    out = ["", " ", "  ", "a", "ab", "hello world", "Hello, World!", "  leading and trailing  ",
           "aaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaa", "bababababababababa", "kékükéküké ßñ 中文中文 😀😀",
           "qxz QX €λ — unknown characters", "digits 0123456789 and 3.14159", "tab\tand\nnewline",
           "[INST] Tell me a story about a dragon. [/INST]", "x" * 300, "ba" * 200]
    for _ in range(40):
        n = int(rng.integers(1, 16))
        out.append(" ".join(str(w) for w in rng.choice(words, n)))
    for _ in range(10):  # words glued together (long merge chains) with outside characters mixed in
        out.append("".join(str(w) for w in rng.choice(words, 6)) + str(rng.choice(list(G.BPE_OUTSIDE))))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-bin", default=os.path.join(ROOT, "oracle", "_ref", "tok_dump"))
    ap.add_argument("--out", default=os.path.join(ROOT, "tests", "golden", "tokenizer_golden.json"))
    args = ap.parse_args()
    from anetransformers_b200 import gguf as G
    cfg = dataclasses.replace(G.MINI, tokenizer="bpe", tokenizer_seed=VOCAB_SEED)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "tok.gguf")
        G.write_synthetic_gguf(path, cfg, seed=1)
        tx = texts()
        inp = "".join(t.encode().hex() + "\n" for t in tx)
        res = subprocess.run([args.ref_bin, path], input=inp, capture_output=True, text=True, check=True)
    cases = []
    for t, line in zip(tx, res.stdout.splitlines()):
        ids_s, dec = line.split("|")
        cases.append({"text_hex": t.encode().hex(), "ids": [int(v) for v in ids_s.split()], "decode_hex": dec})
    assert len(cases) == len(tx)
    json.dump({"generator": "tests/golden/make_tokenizer_golden.py", "reference": "mistral/tokenizer.h",
               "model": {"config": "MINI", "tokenizer": "bpe", "tokenizer_seed": VOCAB_SEED, "vocab_size": cfg.vocab_size},
               "cases": cases}, open(args.out, "w"), indent=0)
    print(f"wrote {len(cases)} cases to {args.out}")


if __name__ == "__main__":
    main()
