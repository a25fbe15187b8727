"""TEST INFRASTRUCTURE.  ctypes view of oracle/_ref/libspec_ref.so: the reference's own mistral/speculative.h
(n-gram drafter, spec_softmax, spec_sample_probs, spec_accept), compiled by `make -C oracle ref` from the reference
tree against the stand-ins in oracle/ref_stub/ (see oracle/ref_spec.c).  Only tests and the fixture script in
tests/golden/ use it.  The reference's arc4random draws from the table passed in `draws` (uint32 values), so a
caller can hand it the same Philox draws the oracle and the device consume.
"""
import ctypes as C
import os
from typing import Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(_HERE, "_ref", "libspec_ref.so")
_lib: Optional[C.CDLL] = None


def available() -> bool:
    return os.path.exists(LIB)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        L = C.CDLL(LIB)
        vp, i32, f32 = C.c_void_p, C.c_int, C.c_float
        sig = {
            "ref_set_draws": (None, [vp, i32]), "ref_draws_used": (i32, []),
            "ref_ngram_draft": (i32, [vp, i32, i32, i32, i32, vp, vp]),
            "ref_ngram_draft_pushed": (i32, [vp, i32, vp, i32, i32, i32, i32, vp, vp]),
            "ref_spec_softmax": (None, [vp, vp, i32, f32]),
            "ref_spec_sample_probs": (i32, [vp, i32]),
            "ref_spec_accept": (i32, [vp, vp, vp, i32, i32, f32, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data if a.size else None


def ngram_draft(prompt: Sequence[int], pushed: Sequence[int], ngram_n: int, max_draft: int, current: int):
    """ngram_draft_init(prompt) + ngram_draft_push_n(pushed) + ngram_draft_fn(current): (tokens, probs)."""
    pr = np.ascontiguousarray(prompt, np.int32)
    pu = np.ascontiguousarray(pushed, np.int32)
    dt = np.zeros(16, np.int32)
    dp = np.zeros(16, np.float32)
    n = lib().ref_ngram_draft_pushed(_p(pr), pr.size, _p(pu), pu.size, ngram_n, max_draft, current, _p(dt), _p(dp))
    return dt[:n].tolist(), dp[:n].tolist()


class _Draws:
    def __init__(self, draws):
        self.a = np.ascontiguousarray(draws, np.uint32)

    def __enter__(self):
        lib().ref_set_draws(_p(self.a), self.a.size)
        return self

    def __exit__(self, *exc):
        lib().ref_set_draws(None, 0)

    @staticmethod
    def used() -> int:
        return lib().ref_draws_used()


def spec_softmax(logits, temp: float) -> np.ndarray:
    lg = np.ascontiguousarray(logits, np.float32)
    out = np.empty_like(lg)
    lib().ref_spec_softmax(_p(lg), _p(out), lg.size, temp)
    return out


def spec_sample_probs(probs, draws):
    """(index, draws consumed)."""
    p = np.ascontiguousarray(probs, np.float32)
    with _Draws(draws) as d:
        t = lib().ref_spec_sample_probs(_p(p), p.size)
        return t, d.used()


def spec_accept(draft_probs, logits, draft_tokens, temp: float, draws):
    """(accepted tokens, draws consumed)."""
    lg = np.ascontiguousarray(logits, np.float32)
    n_draft = len(draft_tokens)
    dp = np.ascontiguousarray(draft_probs, np.float32)
    dt = np.ascontiguousarray(draft_tokens, np.int32)
    acc = np.zeros(n_draft + 1, np.int32)
    with _Draws(draws) as d:
        n = lib().ref_spec_accept(_p(dp), _p(lg), _p(dt), n_draft, lg.shape[-1], temp, _p(acc))
        return acc[:n].tolist(), d.used()
