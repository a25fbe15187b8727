"""The library's tokenizer (sd_tokenizer_*, host code) against the reference's own (mistral/tokenizer.h).

Pinned by tests/golden/tokenizer_golden.json, which tests/golden/make_tokenizer_golden.py produced by running
the reference's tokenizer, compiled from the reference tree, on the seeded bpe test vocabulary: ids and decoded
bytes must be identical for every case (merges with equal-score runs, byte fallback, multi-byte characters,
spaces, the empty text).  When the compiled reference probe is present, random texts are compared live too.
"""
import dataclasses
import json
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden", "tokenizer_golden.json")
REF_BIN = os.path.join(ROOT, "oracle", "_ref", "tok_dump")


@pytest.fixture(scope="module")
def golden():
    return json.load(open(GOLDEN))


@pytest.fixture(scope="module")
def bpe_model(tmp_path_factory, golden):
    from anetransformers_b200 import gguf as G
    m = golden["model"]
    cfg = dataclasses.replace(G.MINI, tokenizer=m["tokenizer"], tokenizer_seed=m["tokenizer_seed"])
    assert cfg.vocab_size == m["vocab_size"]
    path = str(tmp_path_factory.mktemp("tok") / "bpe.gguf")
    G.write_synthetic_gguf(path, cfg, seed=1)
    return path


@pytest.fixture(scope="module")
def tok(bpe_model):
    from anetransformers_b200.tokenizer import Tokenizer
    t = Tokenizer(bpe_model)
    yield t
    t.close()


def test_encode_decode_match_reference_golden(tok, golden):
    assert len(golden["cases"]) >= 60
    for case in golden["cases"]:
        text = bytes.fromhex(case["text_hex"]).decode()
        assert tok.encode(text, add_bos=True) == case["ids"], text
        assert tok.decode(case["ids"]).encode("utf-8", errors="surrogateescape") == bytes.fromhex(case["decode_hex"]), text


def test_vocabulary_and_special_pieces(tok):
    assert tok.vocab_size == 2048 and tok.bos_id == 1 and tok.eos_id == 2
    assert tok.decode_token(tok.bos_id) == b"" and tok.decode_token(tok.eos_id) == b""
    assert tok.decode_token(-1) == b"" and tok.decode_token(tok.vocab_size) == b""
    # byte tokens decode to their byte; <0x00> gives the empty string (a C string ends at NUL)
    assert tok.decode_token(3 + 0x41) == b"A" and tok.decode_token(3) == b""
    piece, score, ty = tok.entry(3 + 0xE2)
    assert piece == b"<0xE2>" and ty == 6
    assert tok.encode("", add_bos=True) == [1] and tok.encode("", add_bos=False) == []


def test_max_tokens_truncates(tok):
    full = tok.encode("bada kéku sada pelo", add_bos=True)
    for m in range(len(full) + 2):
        from anetransformers_b200 import _lib
        out = np.zeros(max(m, 1), np.int32)
        n = _lib.lib().sd_tokenizer_encode(tok.h, "bada kéku sada pelo".encode(), out.ctypes.data, m, 1)
        assert n == min(m, len(full)) and out[:n].tolist() == full[:n]


def test_chat_template():
    from anetransformers_b200.tokenizer import apply_chat
    assert apply_chat("Hello") == "[INST] Hello [/INST]"
    assert apply_chat("") == "[INST]  [/INST]"


def test_plain_vocabulary_round_trip(tmp_path):
    """The benchmark models' vocabulary (specials, bytes, filler pieces, zero scores): every character takes the
    byte fallback and the text decodes back (spaces as U+2581 byte triples, as the reference prints them)."""
    from anetransformers_b200 import gguf as G
    from anetransformers_b200.tokenizer import Tokenizer
    path = str(tmp_path / "plain.gguf")
    G.write_synthetic_gguf(path, G.MINI, seed=1)
    t = Tokenizer(path)
    ids = t.encode("hello world")
    assert ids[0] == 1 and all(3 <= i < 259 for i in ids[1:])
    assert t.decode(ids) == "▁hello▁world"
    t.close()


@pytest.mark.skipif(not os.path.exists(REF_BIN), reason="reference tokenizer probe not built (make -C oracle ref)")
def test_random_texts_match_reference_live(tok, bpe_model):
    from anetransformers_b200 import gguf as G
    rng = np.random.default_rng(5)
    words = G.bpe_corpus_words(0)
    alphabet = G.BPE_CHARS + G.BPE_OUTSIDE + [" ", "  ", "▁"]
    texts = []
    for _ in range(60):
        if rng.random() < 0.5:
            texts.append(" ".join(str(w) for w in rng.choice(words, int(rng.integers(1, 12)))))
        else:
            texts.append("".join(str(c) for c in rng.choice(alphabet, int(rng.integers(1, 40)))))
    res = subprocess.run([REF_BIN, bpe_model], input="".join(t.encode().hex() + "\n" for t in texts),
                         capture_output=True, text=True, check=True)
    for t, line in zip(texts, res.stdout.splitlines()):
        ids = [int(v) for v in line.split("|")[0].split()]
        assert tok.encode(t) == ids, t
