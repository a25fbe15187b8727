"""ctypes binding for the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU baseline /
reference arm.  The product package never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import List, Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "liboracle.so")

Q4_0_DTYPE = np.dtype([("d", "<f2"), ("qs", "u1", (16,))])
Q8_0_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (32,))])

QUANT_IEEE, QUANT_RECIP = 0, 1
ACC_FMA, ACC_MULADD = 0, 1
BONUS_ARGMAX, BONUS_REFERENCE = 0, 1


def build(force: bool = False) -> str:
    src = os.path.join(_HERE, "oracle.c")
    if force or not os.path.exists(_LIB) or os.path.getmtime(_LIB) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE, "liboracle.so"])
    return _LIB


class Config(C.Structure):
    _fields_ = [("dim", C.c_int), ("hidden_dim", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
                ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("vocab_size", C.c_int),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float)]


class Layer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "w1", "w2", "w3")] + \
               [("rms_att", C.c_void_p), ("rms_ffn", C.c_void_p)]


class Model(C.Structure):
    _fields_ = [("cfg", Config), ("layers", Layer * 64), ("tok_embd", C.c_void_p), ("rms_final", C.c_void_p),
                ("lm_head", C.c_void_p), ("tok_embd_type", C.c_int), ("lm_head_type", C.c_int),
                ("theta_inv", C.c_void_p)] + \
               [(n, C.c_void_p) for n in ("xb", "xb2", "q", "k", "v", "att", "hb", "hb2", "logits",
                                         "xb_q8", "hb_q8")] + [("att_cap", C.c_int)]


class KV(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("max_seq", C.c_int),
                ("kv_dim", C.c_int), ("k", C.c_void_p), ("v", C.c_void_p), ("pos", C.c_int), ("len", C.c_int)]


class GenOpts(C.Structure):
    _fields_ = [("max_tokens", C.c_int), ("temp", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int),
                ("rep_penalty", C.c_float), ("rep_window", C.c_int), ("ignore_eos", C.c_int),
                ("eos_id", C.c_int), ("spec_k", C.c_int), ("ngram_n", C.c_int), ("draft_layers", C.c_int),
                ("history_has_current", C.c_int), ("bonus_mode", C.c_int), ("seed", C.c_uint64),
                ("max_seq", C.c_int)]


class GenStats(C.Structure):
    _fields_ = [("n_generated", C.c_int), ("total_draft", C.c_int64), ("total_accepted", C.c_int64),
                ("total_iterations", C.c_int64)]


class Rng(C.Structure):
    _fields_ = [("seed", C.c_uint64), ("counter", C.c_uint64)]


class SampleParams(C.Structure):
    _fields_ = [("temp", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float), ("rep_penalty", C.c_float),
                ("prev_tokens", C.c_void_p), ("n_prev", C.c_int)]


_lib: Optional[C.CDLL] = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(_LIB)
        vp, i32, f32 = C.c_void_p, C.c_int, C.c_float
        sig = {
            "or_set_threads": (None, [i32]), "or_get_threads": (i32, []),
            "or_quantize_q8_0": (None, [vp, vp, i32, i32]),
            "or_q4q8_block_sums": (None, [vp, vp, vp, i32, i32]),
            "or_matvec_q4_0_q8_0": (None, [vp, vp, vp, i32, i32]),
            "or_set_acc_mode": (None, [i32]),
            "or_dequant_q4_0": (None, [vp, vp, i32]),
            "or_rmsnorm": (None, [vp, vp, vp, i32, f32]),
            "or_rope_theta": (None, [vp, i32, f32]),
            "or_apply_rope": (None, [vp, vp, i32, vp, i32, i32, i32]),
            "or_silu_mul": (None, [vp, vp, i32]),
            "or_softmax": (None, [vp, i32]),
            "or_attention": (None, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32]),
            "or_model_init": (i32, [vp, i32]), "or_model_free": (None, [vp]),
            "or_kv_alloc": (i32, [vp, i32, i32, i32, i32]), "or_kv_free": (None, [vp]),
            "or_embed_token": (None, [vp, i32, vp]),
            "or_layer_decode": (None, [vp, vp, vp, i32, i32]),
            "or_logits": (None, [vp, vp]),
            "or_forward_token": (None, [vp, vp, i32, i32, i32]),
            "or_prefill": (None, [vp, vp, vp, i32, i32, vp]),
            "or_philox_u32": (C.c_uint32, [C.c_uint64, C.c_uint64]),
            "or_sample_argmax": (i32, [vp, i32]),
            "or_sample_token": (i32, [vp, i32, vp, vp]),
            "or_spec_softmax": (None, [vp, vp, i32, f32]),
            "or_spec_sample_probs": (i32, [vp, i32, vp]),
            "or_spec_accept": (i32, [vp, vp, vp, i32, i32, f32, vp, vp]),
            "or_ngram_scan": (i32, [vp, i32, i32, i32, i32, vp, vp]),
            "or_ngram_init": (i32, [vp, vp, i32, i32, i32]), "or_ngram_push": (None, [vp, i32]),
            "or_ngram_free": (None, [vp]), "or_ngram_draft": (i32, [vp, i32, vp, vp]),
            "or_generate_greedy": (i32, [vp, vp, i32, vp, vp, vp]),
            "or_generate_ngram": (i32, [vp, vp, i32, vp, vp, vp]),
            "or_generate_self_spec": (i32, [vp, vp, i32, vp, vp, vp]),
            "or_f16_to_f32": (f32, [C.c_uint16]), "or_f32_to_f16": (C.c_uint16, [f32]),
            "or_dequant_q6_K": (None, [vp, vp, i32]), "or_dequant_q4_K_f16": (None, [vp, vp, i32]),
            "or_matvec_kq_f32": (None, [i32, vp, vp, vp, i32, i32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def set_threads(n: int):
    lib().or_set_threads(n)


def quantize_q8_0(x: np.ndarray, variant: int = QUANT_IEEE) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 32, dtype=Q8_0_DTYPE)
    lib().or_quantize_q8_0(_p(x), _p(out), x.size, variant)
    return out


def block_sums(W: np.ndarray, xq: np.ndarray) -> np.ndarray:
    rows, bpr = W.shape
    out = np.zeros((rows, bpr), dtype=np.int32)
    Wc, xc = np.ascontiguousarray(W), np.ascontiguousarray(xq)  # alive across the call
    lib().or_q4q8_block_sums(_p(Wc), _p(xc), _p(out), rows, bpr * 32)
    return out


def matvec(W: np.ndarray, xq: np.ndarray, acc_mode: int = ACC_FMA) -> np.ndarray:
    rows, bpr = W.shape
    y = np.zeros(rows, dtype=np.float32)
    L = lib()
    L.or_set_acc_mode(acc_mode)
    Wc, xc = np.ascontiguousarray(W), np.ascontiguousarray(xq)
    L.or_matvec_q4_0_q8_0(_p(Wc), _p(xc), _p(y), rows, bpr * 32)
    L.or_set_acc_mode(ACC_FMA)
    return y


def dequant(W: np.ndarray) -> np.ndarray:
    W = np.ascontiguousarray(W)
    out = np.zeros(W.size * 32, dtype=np.float32)
    lib().or_dequant_q4_0(_p(W), _p(out), W.size * 32)
    return out.reshape(W.shape[0], -1) if W.ndim == 2 else out


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros_like(x)
    lib().or_rmsnorm(_p(out), _p(x), _p(w), x.size, eps)
    return out


def rope_theta(head_dim: int, theta: float) -> np.ndarray:
    out = np.zeros(head_dim // 2, np.float32)
    lib().or_rope_theta(_p(out), head_dim, theta)
    return out


def apply_rope(q: np.ndarray, k: np.ndarray, pos: int, theta_inv: np.ndarray, n_heads: int, n_kv: int,
               head_dim: int):
    q = np.array(q, np.float32, copy=True)
    k = np.array(k, np.float32, copy=True)
    ti = np.ascontiguousarray(theta_inv, np.float32)
    lib().or_apply_rope(_p(q), _p(k), pos, _p(ti), n_heads, n_kv, head_dim)
    return q, k


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.array(g, np.float32, copy=True)
    uc = np.ascontiguousarray(u, np.float32)
    lib().or_silu_mul(_p(g), _p(uc), g.size)
    return g


def softmax(x: np.ndarray) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    lib().or_softmax(_p(x), x.size)
    return x


def attention(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, n_heads: int, heads_per_kv: int, hd: int,
              max_seq: int, pos: int) -> np.ndarray:
    """q: [n_heads*hd] fp32 (not pre-scaled); kc/vc: [max_seq, kv_dim] fp16 bit patterns (uint16)."""
    q = np.array(q, np.float32, copy=True)
    att = np.zeros(n_heads * max_seq, np.float32)
    out = np.zeros(n_heads * hd, np.float32)
    kcc, vcc = np.ascontiguousarray(kc), np.ascontiguousarray(vc)
    lib().or_attention(_p(q), _p(att), _p(out), _p(kcc), _p(vcc),
                       n_heads, heads_per_kv, hd, max_seq, pos)
    return out


def philox(seed: int, counter: int) -> int:
    return lib().or_philox_u32(seed, counter)


def sample_argmax(logits: np.ndarray) -> int:
    lc = np.ascontiguousarray(logits, np.float32)
    return lib().or_sample_argmax(_p(lc), logits.size)


def sample_token(logits, temp: float, top_k: int = 40, top_p: float = 0.9, rep_penalty: float = 1.0, prev_tokens=(),
                 seed: int = 0, counter: int = 0):
    """mistral_model.h:1145-1240 on a copy of logits; returns (token, counter, logits after the penalty)."""
    lg = np.array(logits, dtype=np.float32, copy=True)
    prev = np.ascontiguousarray(prev_tokens, np.int32)
    sp = SampleParams(temp, top_k, top_p, rep_penalty, _p(prev) if prev.size else None, prev.size)
    rng = Rng(seed, counter)
    t = lib().or_sample_token(_p(lg), lg.size, C.addressof(sp), C.addressof(rng))
    return t, rng.counter, lg


def spec_softmax(logits, temp: float) -> np.ndarray:
    """speculative.h:37-57."""
    lg = np.ascontiguousarray(logits, np.float32)
    out = np.empty_like(lg)
    lib().or_spec_softmax(_p(lg), _p(out), lg.size, temp)
    return out


def spec_sample_probs(probs, seed: int = 0, counter: int = 0):
    """speculative.h:60-68 with the Philox draw; returns (index, counter)."""
    p = np.ascontiguousarray(probs, np.float32)
    rng = Rng(seed, counter)
    t = lib().or_spec_sample_probs(_p(p), p.size, C.addressof(rng))
    return t, rng.counter


def uniform(seed: int, counter: int) -> float:
    """The draw the oracle and the device use in place of (float)arc4random() / (float)UINT32_MAX."""
    return float(np.float32(philox(seed, counter)) / np.float32(4294967295.0))


TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K = 2, 12, 14


def dequant_q6_k(W: np.ndarray) -> np.ndarray:
    """dequant_q6_K_block (mistral/dequant.h:292-306) of [rows, cols/256] Q6_K blocks -> [rows, cols] fp32."""
    W = np.ascontiguousarray(W)
    out = np.empty(W.size * 256, np.float32)
    lib().or_dequant_q6_K(_p(W), _p(out), out.size)
    return out.reshape(W.shape[0], -1)


def dequant_q4_k(W: np.ndarray) -> np.ndarray:
    """dequant_q4_K_block_neon (mistral/dequant.h:63-113) -> fp16 values (as float16), [rows, cols]."""
    W = np.ascontiguousarray(W)
    out = np.empty(W.size * 256, np.uint16)
    lib().or_dequant_q4_K_f16(_p(W), _p(out), out.size)
    return out.view(np.float16).reshape(W.shape[0], -1)


def matvec_kq(W: np.ndarray, x: np.ndarray, ttype: int) -> np.ndarray:
    """The reference's fp32 K-quant matvec (q4_matvec -> q6_K_matvec_f32_neon / Q4_K dequant + sgemv)."""
    W = np.ascontiguousarray(W)
    xs = np.ascontiguousarray(x, np.float32)
    y = np.empty(W.shape[0], np.float32)
    lib().or_matvec_kq_f32(ttype, _p(W), _p(xs), _p(y), W.shape[0], xs.size)
    return y


def spec_accept(draft_probs, logits, draft_tokens, temp: float, seed: int = 0, counter: int = 0):
    logits = np.ascontiguousarray(logits, np.float32)
    n_draft = len(draft_tokens)
    vocab = logits.shape[-1]
    dp = np.ascontiguousarray(draft_probs, np.float32)
    dt = np.ascontiguousarray(draft_tokens, np.int32)
    acc = np.zeros(n_draft + 1, np.int32)
    rng = Rng(seed, counter)
    n = lib().or_spec_accept(_p(dp), _p(logits), _p(dt), n_draft, vocab, temp, _p(acc), C.addressof(rng))
    return acc[:n].tolist(), rng.counter


def ngram_scan(history, ngram_n: int, max_draft: int, current: int):
    h = np.ascontiguousarray(history, np.int32)
    dt = np.zeros(max(max_draft, 1), np.int32)
    mp = C.c_int(-1)
    n = lib().or_ngram_scan(_p(h) if h.size else None, h.size, ngram_n, max_draft, current, _p(dt), C.addressof(mp))
    return dt[:n].tolist(), mp.value


class NGram(C.Structure):
    _fields_ = [("history", C.c_void_p), ("history_len", C.c_int), ("history_cap", C.c_int), ("ngram_n", C.c_int),
                ("max_draft", C.c_int)]


def ngram_draft(prompt, pushed, ngram_n: int, max_draft: int, current: int):
    """speculative.h:395-464 through the oracle's drafter object: init on prompt (ngram_n / max_draft defaults and
    the SPEC_MAX_DRAFT clip applied there), push each of pushed, draft after current.  Returns (tokens, probs)."""
    L = lib()
    pr = np.ascontiguousarray(prompt, np.int32)
    d = NGram()
    if L.or_ngram_init(C.addressof(d), _p(pr) if pr.size else None, pr.size, ngram_n, max_draft):
        raise MemoryError("or_ngram_init")
    try:
        for t in pushed:
            L.or_ngram_push(C.addressof(d), int(t))
        dt = np.zeros(16, np.int32)
        dp = np.zeros(16, np.float32)
        n = L.or_ngram_draft(C.addressof(d), current, _p(dt), _p(dp))
        return dt[:n].tolist(), dp[:n].tolist()
    finally:
        L.or_ngram_free(C.addressof(d))


class OracleModel:
    """Oracle view of a GGUF model (pointers into the mapped file)."""

    def __init__(self, gguf, max_seq: int = 4096):
        self.g = gguf
        cfg = gguf.config()
        self.cfg = cfg
        self.m = Model()
        c = self.m.cfg
        c.dim, c.hidden_dim, c.n_layers = cfg.dim, cfg.hidden_dim, cfg.n_layers
        c.n_heads, c.n_kv_heads, c.head_dim, c.vocab_size = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.vocab_size
        c.rope_theta, c.rms_eps = cfg.rope_theta, cfg.rms_eps
        self._keep: List[np.ndarray] = []

        def ptr(name):
            a = gguf.array(name)
            self._keep.append(a)
            return a.ctypes.data
        for l in range(cfg.n_layers):
            L = self.m.layers[l]
            L.wq, L.wk, L.wv = ptr(f"blk.{l}.attn_q.weight"), ptr(f"blk.{l}.attn_k.weight"), ptr(f"blk.{l}.attn_v.weight")
            L.wo = ptr(f"blk.{l}.attn_output.weight")
            L.w1, L.w3, L.w2 = ptr(f"blk.{l}.ffn_gate.weight"), ptr(f"blk.{l}.ffn_up.weight"), ptr(f"blk.{l}.ffn_down.weight")
            L.rms_att, L.rms_ffn = ptr(f"blk.{l}.attn_norm.weight"), ptr(f"blk.{l}.ffn_norm.weight")
        self.m.tok_embd = ptr("token_embd.weight")
        self.m.rms_final = ptr("output_norm.weight")
        self.m.lm_head = ptr("output.weight")
        self.m.tok_embd_type = gguf.tensors["token_embd.weight"].ttype
        self.m.lm_head_type = gguf.tensors["output.weight"].ttype
        self.max_seq = max_seq
        if lib().or_model_init(C.addressof(self.m), max_seq) != 0:
            raise MemoryError("oracle model init failed")

    def close(self):
        if self.m.att:
            lib().or_model_free(C.addressof(self.m))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def new_kv(self, n_layers: Optional[int] = None) -> KV:
        kv = KV()
        lib().or_kv_alloc(C.addressof(kv), n_layers or self.cfg.n_layers, self.cfg.n_kv_heads, self.cfg.head_dim,
                          self.max_seq)
        return kv

    def free_kv(self, kv: KV):
        lib().or_kv_free(C.addressof(kv))

    def kv_arrays(self, kv: KV, layer: int):
        n = self.max_seq * kv.kv_dim
        k = np.ctypeslib.as_array(C.cast(kv.k, C.POINTER(C.c_uint16)), shape=(kv.n_layers * n,))
        v = np.ctypeslib.as_array(C.cast(kv.v, C.POINTER(C.c_uint16)), shape=(kv.n_layers * n,))
        return (k[layer * n:(layer + 1) * n].reshape(self.max_seq, kv.kv_dim),
                v[layer * n:(layer + 1) * n].reshape(self.max_seq, kv.kv_dim))

    def embed(self, token: int) -> np.ndarray:
        out = np.zeros(self.cfg.dim, np.float32)
        lib().or_embed_token(C.addressof(self.m), token, _p(out))
        return out

    def layer(self, kv: KV, x: np.ndarray, layer: int, pos: int) -> np.ndarray:
        x = np.array(x, np.float32, copy=True)
        lib().or_layer_decode(C.addressof(self.m), C.addressof(kv), _p(x), layer, pos)
        return x

    def logits(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        lib().or_logits(C.addressof(self.m), _p(x))
        return np.ctypeslib.as_array(C.cast(self.m.logits, C.POINTER(C.c_float)), shape=(self.cfg.vocab_size,)).copy()

    def forward(self, kv: KV, token: int, pos: int, n_layers: Optional[int] = None) -> np.ndarray:
        lib().or_forward_token(C.addressof(self.m), C.addressof(kv), token, pos, n_layers or self.cfg.n_layers)
        return np.ctypeslib.as_array(C.cast(self.m.logits, C.POINTER(C.c_float)), shape=(self.cfg.vocab_size,)).copy()

    def prefill(self, kv: KV, tokens, n_layers: Optional[int] = None) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int32)
        x = np.zeros(self.cfg.dim, np.float32)
        lib().or_prefill(C.addressof(self.m), C.addressof(kv), _p(t), t.size, n_layers or self.cfg.n_layers, _p(x))
        return x

    def generate(self, mode: str, prompt, max_tokens: int, *, temp=0.0, top_k=40, top_p=0.9, rep_penalty=1.0,
                 rep_window=64, ignore_eos=True, spec_k=4, ngram_n=3, draft_layers=8, history_has_current=False,
                 bonus_mode=BONUS_ARGMAX, seed=0):
        o = GenOpts(max_tokens=max_tokens, temp=temp, top_p=top_p, top_k=top_k, rep_penalty=rep_penalty,
                    rep_window=rep_window, ignore_eos=int(ignore_eos), eos_id=self.cfg.eos_id, spec_k=spec_k,
                    ngram_n=ngram_n, draft_layers=draft_layers, history_has_current=int(history_has_current),
                    bonus_mode=bonus_mode, seed=seed, max_seq=self.max_seq)
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max_tokens + 2 * 8 + 4, np.int32)
        st = GenStats()
        fn = {"greedy": lib().or_generate_greedy, "ngram": lib().or_generate_ngram,
              "self": lib().or_generate_self_spec}[mode]
        n = fn(C.addressof(self.m), _p(p), p.size, C.addressof(o), _p(out), C.addressof(st))
        if n < 0:
            raise RuntimeError("oracle generate failed")
        return out[:n].tolist(), {"n_generated": st.n_generated, "total_draft": st.total_draft,
                                  "total_accepted": st.total_accepted, "total_iterations": st.total_iterations}
