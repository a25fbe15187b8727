"""Model-level host mirror of the reference's metal_matvec.h / speculative.h / mistral CLI loops.

``Context`` wraps an sd_ctx (metal_context_init + mistral_load: weights repacked in HBM, fp16 KV ring);
``forward`` is metal_forward / metal_forward_batch + logits (spec_verify); ``generate`` runs the decode
loops of mistral_infer.m (greedy, n-gram speculative, self-speculative) on the device.  Free functions
``ngram_draft`` and ``spec_accept`` mirror speculative.h's ngram_draft_fn and spec_accept.
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib

GEN_GREEDY, GEN_NGRAM, GEN_SELF_SPEC = 0, 1, 2
BONUS_ARGMAX, BONUS_REFERENCE = 0, 1
_MODES = {"greedy": GEN_GREEDY, "ngram": GEN_NGRAM, "self": GEN_SELF_SPEC}
MAX_VERIFY = 16  # SD_MAX_VERIFY: tokens per verify forward (current + up to 15 drafts)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


NCCL_ID_BYTES = 128


def nccl_unique_id() -> bytes:
    """A new NCCL unique id (created by one rank, sent to the others)."""
    buf = C.create_string_buffer(NCCL_ID_BYTES)
    _lib.check(_lib.lib().sd_nccl_unique_id(buf), "sd_nccl_unique_id")
    return buf.raw


class NcclComm:
    """One rank's NCCL communicator for tensor-parallel contexts (pass .handle as nccl_comm)."""

    def __init__(self, unique_id: bytes, nranks: int, rank: int, device: int):
        if len(unique_id) != NCCL_ID_BYTES:
            raise ValueError("unique id must be %d bytes" % NCCL_ID_BYTES)
        h = C.c_void_p()
        _lib.check(_lib.lib().sd_nccl_comm_create(unique_id, nranks, rank, device, C.byref(h)), "sd_nccl_comm_create")
        self.h = h

    @property
    def handle(self) -> int:
        return self.h.value or 0

    def close(self):
        if getattr(self, "h", None):
            _lib.lib().sd_nccl_comm_destroy(self.h)
            self.h = None


class Context:
    """A model on one GPU (or one tensor-parallel rank)."""

    def __init__(self, model, device: int = 0, max_seq: int = 0, max_batch: int = 0, use_graphs: bool = True,
                 use_pdl: bool = True, tp_rank: int = 0, tp_size: int = 1, nccl_comm: int = 0,
                 forward_kernel: Optional[int] = None, prefill_gemm: Optional[bool] = None):
        L = _lib.lib()
        o = _lib.CtxOpts()
        L.sd_ctx_opts_default(C.byref(o))
        o.device, o.max_seq, o.max_batch = device, max_seq, max_batch
        o.use_graphs, o.use_pdl = int(use_graphs), int(use_pdl)
        if forward_kernel is not None:
            o.forward_kernel = int(forward_kernel)
        if prefill_gemm is not None:
            o.prefill_gemm = int(prefill_gemm)
        o.tp_rank, o.tp_size, o.nccl_comm = tp_rank, tp_size, nccl_comm or None
        h = C.c_void_p()
        if isinstance(model, (bytes, bytearray, memoryview)):
            buf = (C.c_char * len(model)).from_buffer_copy(model) if not isinstance(model, bytearray) else \
                (C.c_char * len(model)).from_buffer(model)
            rc = L.sd_ctx_create(C.addressof(buf), len(model), C.byref(o), C.byref(h))
        else:
            rc = L.sd_ctx_create_file(str(model).encode(), C.byref(o), C.byref(h))
        _lib.check(rc, "sd_ctx_create")
        self.h = h
        info = _lib.ModelInfo()
        _lib.check(L.sd_ctx_info(h, C.byref(info)), "sd_ctx_info")
        self.info = info
        self.vocab = info.vocab_size
        self.max_batch = max_batch if 0 < max_batch <= 8 else 8

    # -- tensor parallel over peer memory -------------------------------------------------------------
    def tp_handle(self) -> bytes:
        """This rank's exchange-region handle (CUDA IPC), to be sent to the other ranks."""
        buf = C.create_string_buffer(64)
        _lib.check(_lib.lib().sd_ctx_tp_handle(self.h, buf), "sd_ctx_tp_handle")
        return buf.raw

    def tp_connect(self, handles: Sequence[bytes]):
        """Connect to every rank's exchange region (handles in rank order); the all-reduces then run
        inside the norm kernels over NVLink instead of NCCL."""
        blob = b"".join(handles)
        _lib.check(_lib.lib().sd_ctx_tp_connect(self.h, blob, len(handles)), "sd_ctx_tp_connect")
        info = _lib.ModelInfo()
        _lib.check(_lib.lib().sd_ctx_info(self.h, C.byref(info)), "sd_ctx_info")
        self.info = info  # forward_kernel may change once the peers are connected

    # -- lifetime --------------------------------------------------------------------------------
    def close(self):
        if getattr(self, "h", None):
            _lib.lib().sd_ctx_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def stream(self) -> int:
        return _lib.lib().sd_ctx_stream(self.h) or 0

    def device_error(self) -> int:
        return _lib.lib().sd_ctx_device_error(self.h)

    # -- forward ---------------------------------------------------------------------------------
    def forward(self, tokens: Sequence[int], pos: int, want_logits: bool = True) -> Tuple[np.ndarray, np.ndarray]:
        """Forward len(tokens) <= MAX_VERIFY tokens at positions pos.. (writes their K/V; batches wider than
        max_batch run as consecutive forwards); returns (logits [S, vocab] or None, argmax [S])."""
        t = _i32(tokens)
        S = t.size
        logits = np.empty((S, self.vocab), np.float32) if want_logits else None
        am = np.empty(S, np.int32)
        _lib.check(_lib.lib().sd_forward(self.h, t.ctypes.data, S, pos,
                                         logits.ctypes.data if want_logits else None, am.ctypes.data), "sd_forward")
        return logits, am

    def forward_layers(self, n_layers: int, tokens: Sequence[int], pos: int) -> Tuple[np.ndarray, np.ndarray]:
        t = _i32(tokens)
        logits = np.empty((t.size, self.vocab), np.float32)
        am = np.empty(t.size, np.int32)
        _lib.check(_lib.lib().sd_forward_layers(self.h, n_layers, t.ctypes.data, t.size, pos, logits.ctypes.data,
                                                am.ctypes.data), "sd_forward_layers")
        return logits, am

    def forward_dev(self, tokens_dev, pos: int, logits_dev=None, argmax_dev=None, stream: int = 0):
        """Device-pointer form (torch tensors), stream-ordered."""
        S = tokens_dev.numel()
        _lib.check(_lib.lib().sd_forward_dev(self.h, tokens_dev.data_ptr(), S, pos,
                                             logits_dev.data_ptr() if logits_dev is not None else None,
                                             argmax_dev.data_ptr() if argmax_dev is not None else None,
                                             stream or None), "sd_forward_dev")

    def prefill(self, tokens: Sequence[int], start_pos: int = 0):
        t = _i32(tokens)
        _lib.check(_lib.lib().sd_prefill(self.h, t.ctypes.data if t.size else None, t.size, start_pos), "sd_prefill")

    def kv_read(self, layer: int, pos0: int, n: int) -> Tuple[np.ndarray, np.ndarray]:
        kvd = self.info.n_kv_heads * self.info.head_dim // self.info.tp_size
        k = np.empty((n, kvd), np.uint16)
        v = np.empty((n, kvd), np.uint16)
        _lib.check(_lib.lib().sd_kv_read(self.h, layer, pos0, n, k.ctypes.data, v.ctypes.data), "sd_kv_read")
        return k, v

    # -- generation ------------------------------------------------------------------------------
    @staticmethod
    def gen_params(mode="greedy", max_tokens=128, temp=0.7, top_p=0.9, top_k=40, rep_penalty=1.1, rep_window=64,
                   ignore_eos=False, spec_k=4, ngram_n=3, draft_layers=8, history_has_current=False,
                   bonus_mode=BONUS_ARGMAX, seed=0, reuse_draft_kv=False) -> _lib.GenParams:
        p = _lib.GenParams()
        _lib.lib().sd_gen_params_default(C.byref(p))
        p.mode = _MODES[mode] if isinstance(mode, str) else mode
        p.max_tokens, p.temp, p.top_p, p.top_k = max_tokens, temp, top_p, top_k
        p.rep_penalty, p.rep_window, p.ignore_eos = rep_penalty, rep_window, int(ignore_eos)
        p.spec_k, p.ngram_n, p.draft_layers = spec_k, ngram_n, draft_layers
        p.history_has_current, p.bonus_mode, p.seed = int(history_has_current), bonus_mode, seed
        p.reuse_draft_kv = int(reuse_draft_kv)
        return p

    def generate(self, prompt: Sequence[int], **kw) -> Tuple[List[int], Dict]:
        """Prefill + first token + decode loop (mistral_infer.m main).  Returns (tokens, stats)."""
        p = self.gen_params(**kw)
        t = _i32(prompt)
        out = np.empty(p.max_tokens + 2 * MAX_VERIFY + 4, np.int32)
        st = _lib.GenStats()
        n = _lib.lib().sd_generate(self.h, C.byref(p), t.ctypes.data, t.size, out.ctypes.data, out.size, C.byref(st))
        if n < 0:
            _lib.check(n, "sd_generate")
        return out[:n].tolist(), _stats(st)

    def decode(self, history: Sequence[int], first_token: int, **kw) -> Tuple[List[int], Dict]:
        """Decode loop only; positions [0, len(history)-1) must already hold the prompt's K/V."""
        p = self.gen_params(**kw)
        h = _i32(history)
        out = np.empty(p.max_tokens + 2 * MAX_VERIFY + 4, np.int32)
        st = _lib.GenStats()
        n = _lib.lib().sd_decode(self.h, C.byref(p), h.ctypes.data, h.size, first_token, out.ctypes.data, out.size,
                                 C.byref(st))
        if n < 0:
            _lib.check(n, "sd_decode")
        return out[:n].tolist(), _stats(st)

    def spec_accept(self, draft_probs, logits, draft, temp: float, bonus_mode=BONUS_ARGMAX, seed=0, counter=0):
        """speculative.h spec_accept on the device.  logits: [n_draft+1, vocab].  Returns (accepted, counter)."""
        lg = np.ascontiguousarray(logits, np.float32)
        d = _i32(draft)
        dp = np.ascontiguousarray(draft_probs, np.float32) if draft_probs is not None else None
        acc = np.empty(d.size + 1, np.int32)
        ctr = C.c_uint64(counter)
        n = _lib.lib().sd_spec_accept(self.h, dp.ctypes.data if dp is not None else None, lg.ctypes.data, d.ctypes.data,
                                      d.size, temp, bonus_mode, seed, C.byref(ctr), acc.ctypes.data)
        if n < 0:
            _lib.check(n, "sd_spec_accept")
        return acc[:n].tolist(), ctr.value

    # -- single-op model layer (mistral_model.h / speculative.h helpers) ---------------------------------
    def sample_token(self, logits, temp: float, top_k: int = 40, top_p: float = 0.9, rep_penalty: float = 1.0,
                     prev_tokens=(), seed: int = 0, counter: int = 0):
        """mistral_model.h sample_token on the device.  Returns (token, counter, logits after the in-place
        repetition penalty)."""
        lg = np.array(logits, dtype=np.float32, copy=True)
        prev = _i32(prev_tokens)
        ctr = C.c_uint64(counter)
        n = _lib.lib().sd_sample_token(self.h, lg.ctypes.data, lg.size, temp, top_k, top_p, rep_penalty,
                                       prev.ctypes.data if prev.size else None, prev.size, seed, C.byref(ctr))
        if n < 0:
            _lib.check(n, "sd_sample_token")
        return n, ctr.value, lg

    def spec_softmax(self, logits, temp: float) -> np.ndarray:
        lg = np.ascontiguousarray(logits, np.float32)
        out = np.empty_like(lg)
        _lib.check(_lib.lib().sd_spec_softmax(self.h, lg.ctypes.data, out.ctypes.data, lg.size, temp), "sd_spec_softmax")
        return out

    def spec_sample_probs(self, probs, seed: int = 0, counter: int = 0):
        p = np.ascontiguousarray(probs, np.float32)
        ctr = C.c_uint64(counter)
        n = _lib.lib().sd_spec_sample_probs(self.h, p.ctypes.data, p.size, seed, C.byref(ctr))
        if n < 0:
            _lib.check(n, "sd_spec_sample_probs")
        return n, ctr.value

    def embed_token(self, token: int) -> np.ndarray:
        out = np.empty(self.info.dim, np.float32)
        _lib.check(_lib.lib().sd_embed_token(self.h, token, out.ctypes.data), "sd_embed_token")
        return out

    def layer_decode(self, x, layer: int, pos: int) -> np.ndarray:
        """mistral_layer_decode_parallel: x [dim] through one layer at pos (writes that layer's K/V)."""
        xv = np.array(x, dtype=np.float32, copy=True)
        _lib.check(_lib.lib().sd_layer_decode(self.h, xv.ctypes.data, layer, pos), "sd_layer_decode")
        return xv

    def logits_of(self, x) -> np.ndarray:
        """mistral_logits: final RMSNorm + Q8_0 + LM head of hidden states x [S, dim] (or [dim])."""
        xv = np.ascontiguousarray(np.atleast_2d(np.asarray(x, np.float32)))
        out = np.empty((xv.shape[0], self.vocab), np.float32)
        _lib.check(_lib.lib().sd_logits(self.h, xv.ctypes.data, xv.shape[0], out.ctypes.data), "sd_logits")
        return out


class BatchContext:
    """Many independent streams on one GPU sharing a Context's weights (sd_batch_* of the C ABI).  Every
    stream has its own KV ring and generation state; one forward carries `width` tokens of every stream."""

    def __init__(self, ctx: Context, n_streams: int, max_seq: int, width: int = _lib.BATCH_MAX_WIDTH):
        self.ctx = ctx  # keeps the weights alive
        self.n_streams, self.max_seq, self.width, self.vocab = n_streams, max_seq, width, ctx.vocab
        h = C.c_void_p()
        _lib.check(_lib.lib().sd_batch_create(ctx.h, n_streams, max_seq, width, C.byref(h)), "sd_batch_create")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            _lib.lib().sd_batch_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return _lib.lib().sd_batch_stream(self.h) or 0

    GEMM_AUTO, GEMM_MMA, GEMM_TC = 0, 1, 2

    def set_gemm(self, mode: int):
        """Tensor-core GEMM of the forwards: GEMM_AUTO (tcgen05 from 64 tokens per forward), GEMM_MMA
        (mma.sync always) or GEMM_TC (tcgen05 always); the results are bit-identical."""
        _lib.check(_lib.lib().sd_batch_set_gemm(self.h, int(mode)), "sd_batch_set_gemm")

    def forward(self, tokens, pos, want_logits: bool = True) -> np.ndarray:
        """tokens [n_streams, T] at positions pos[s] ..; returns logits [n_streams, T, vocab] (or None)."""
        t = np.ascontiguousarray(tokens, np.int32)
        assert t.ndim == 2 and t.shape[0] == self.n_streams
        ps = _i32(pos)
        lg = np.empty((t.shape[0], t.shape[1], self.vocab), np.float32) if want_logits else None
        _lib.check(_lib.lib().sd_batch_forward(self.h, t.ctypes.data, t.shape[1], ps.ctypes.data,
                                               lg.ctypes.data if want_logits else None), "sd_batch_forward")
        return lg

    def prefill(self, tokens):
        t = np.ascontiguousarray(tokens, np.int32)
        _lib.check(_lib.lib().sd_batch_prefill(self.h, t.ctypes.data, t.shape[1]), "sd_batch_prefill")

    def _out(self, p):
        return np.empty((self.n_streams, p.max_tokens + 2 * MAX_VERIFY + 4), np.int32), np.empty(self.n_streams, np.int32)

    def generate(self, prompts, **kw) -> Tuple[List[List[int]], Dict]:
        """Prefill + first token + decode of every stream (prompts [n_streams, n_prompt])."""
        p = Context.gen_params(**kw)
        t = np.ascontiguousarray(prompts, np.int32)
        out, n = self._out(p)
        st = _lib.BatchStats()
        _lib.check(_lib.lib().sd_batch_generate(self.h, C.byref(p), t.ctypes.data, t.shape[1], out.ctypes.data,
                                                out.shape[1], n.ctypes.data, C.byref(st)), "sd_batch_generate")
        return [out[i, :n[i]].tolist() for i in range(self.n_streams)], _batch_stats(st)

    def decode(self, history, first, **kw) -> Tuple[List[List[int]], Dict]:
        """Decode only: history [n_streams, n_hist] (ends with first), K/V of positions < n_hist - 1 in place."""
        p = Context.gen_params(**kw)
        h = np.ascontiguousarray(history, np.int32)
        f = _i32(first)
        out, n = self._out(p)
        st = _lib.BatchStats()
        _lib.check(_lib.lib().sd_batch_decode(self.h, C.byref(p), h.ctypes.data, h.shape[1], f.ctypes.data,
                                              out.ctypes.data, out.shape[1], n.ctypes.data, C.byref(st)),
                   "sd_batch_decode")
        return [out[i, :n[i]].tolist() for i in range(self.n_streams)], _batch_stats(st)


def _batch_stats(st: _lib.BatchStats) -> Dict:
    it = st.total_iterations
    return {"n_generated": st.n_generated, "total_draft": st.total_draft, "total_accepted": st.total_accepted,
            "total_iterations": it, "verify_forwards": st.verify_forwards, "ms_prefill": st.ms_prefill,
            "ms_decode": st.ms_decode,
            "acceptance_rate": ((st.total_accepted - it) / st.total_draft) if st.total_draft else 0.0}


def _stats(st: _lib.GenStats) -> Dict:
    it = st.total_iterations
    return {"n_generated": st.n_generated, "total_draft": st.total_draft, "total_accepted": st.total_accepted,
            "total_iterations": it, "ms_prefill": st.ms_prefill, "ms_decode": st.ms_decode,
            # (accepted - iterations) / drafted: the reference's definition (speculative.h:360-366)
            "acceptance_rate": ((st.total_accepted - it) / st.total_draft) if st.total_draft else 0.0}


def ngram_draft(history: Sequence[int], ngram_n: int, max_draft: int, current: int) -> Tuple[List[int], int]:
    """speculative.h ngram_draft_fn as a device scan: (drafts, match position) for the given history."""
    h = _i32(history)
    out = np.empty(max(max_draft, 1), np.int32)
    mp = C.c_int(-1)
    n = _lib.lib().sd_ngram_draft(h.ctypes.data if h.size else None, h.size, ngram_n, max_draft, current,
                                  out.ctypes.data, C.byref(mp))
    if n < 0:
        _lib.check(n, "sd_ngram_draft")
    return out[:n].tolist(), mp.value
