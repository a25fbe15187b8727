"""ctypes binding of libspecdec_b200.so (the C ABI declared in include/specdec_b200.h).

There is no CPU fallback: if the shared library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
SO_PATH = os.path.join(_HERE, "libspecdec_b200.so")

SD_OK = 0
STATUS_NAMES = {0: "SD_OK", -1: "SD_ERR_INVALID", -2: "SD_ERR_OOM", -3: "SD_ERR_CUDA", -4: "SD_ERR_TIMEOUT",
                -5: "SD_ERR_FORMAT", -6: "SD_ERR_UNSUPPORTED", -7: "SD_ERR_NO_DEVICE"}


class SpecDecError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class Q8Dev(C.Structure):
    _fields_ = [("qs", C.c_void_p), ("d", C.c_void_p), ("sum", C.c_void_p)]


class ModelInfo(C.Structure):
    _fields_ = [("dim", C.c_int), ("hidden_dim", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
                ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("vocab_size", C.c_int), ("max_seq", C.c_int),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float), ("bos_id", C.c_int), ("eos_id", C.c_int),
                ("tp_rank", C.c_int), ("tp_size", C.c_int), ("weight_bytes", C.c_size_t), ("kv_bytes", C.c_size_t),
                ("forward_kernel", C.c_int)]


class CtxOpts(C.Structure):
    _fields_ = [("device", C.c_int), ("max_seq", C.c_int), ("max_batch", C.c_int), ("tp_rank", C.c_int),
                ("tp_size", C.c_int), ("nccl_comm", C.c_void_p), ("use_graphs", C.c_int), ("use_pdl", C.c_int),
                ("forward_kernel", C.c_int), ("prefill_gemm", C.c_int)]


class GenParams(C.Structure):
    _fields_ = [("mode", C.c_int), ("max_tokens", C.c_int), ("temp", C.c_float), ("top_p", C.c_float),
                ("top_k", C.c_int), ("rep_penalty", C.c_float), ("rep_window", C.c_int), ("ignore_eos", C.c_int),
                ("spec_k", C.c_int), ("ngram_n", C.c_int), ("draft_layers", C.c_int),
                ("history_has_current", C.c_int), ("bonus_mode", C.c_int), ("seed", C.c_uint64),
                ("reuse_draft_kv", C.c_int)]


class GenStats(C.Structure):
    _fields_ = [("n_generated", C.c_int), ("total_draft", C.c_int64), ("total_accepted", C.c_int64),
                ("total_iterations", C.c_int64), ("ms_prefill", C.c_double), ("ms_decode", C.c_double)]


class BatchStats(C.Structure):
    _fields_ = [("n_generated", C.c_int64), ("total_draft", C.c_int64), ("total_accepted", C.c_int64),
                ("total_iterations", C.c_int64), ("verify_forwards", C.c_int64), ("ms_prefill", C.c_double),
                ("ms_decode", C.c_double)]


BATCH_MAX_WIDTH = 8

vp, i32, f32, sz, u64 = C.c_void_p, C.c_int, C.c_float, C.c_size_t, C.c_uint64
_SIGS = {
    "sd_last_error": (C.c_char_p, []),
    "sd_abi_version": (i32, []),
    "sd_device_count": (i32, []),
    "sd_qmat_create": (i32, [vp, i32, i32, i32, vp]),
    "sd_qmat_free": (None, [vp]),
    "sd_qmat_shape": (i32, [vp, vp, vp, vp]),
    "sd_quantize_q8_0_dev": (i32, [vp, Q8Dev, i32, i32, vp]),
    "sd_q8_to_blocks_dev": (i32, [Q8Dev, vp, i32, i32, vp]),
    "sd_blocks_to_q8_dev": (i32, [vp, Q8Dev, i32, i32, vp]),
    "sd_matvec_q4_0_q8_0_dev": (i32, [vp, Q8Dev, vp, i32, vp]),
    "sd_block_sums_dev": (i32, [vp, Q8Dev, vp, vp]),
    "sd_matvec_q4_0_q8_0_noalloc_dev": (i32, [vp, Q8Dev, vp, i32, vp]),
    "sd_device_error": (i32, [i32]),
    "sd_host_quantize_f32_to_q8_0": (None, [vp, vp, i32]),
    "sd_host_q4_0_q8_0_matvec": (None, [vp, vp, vp, i32, i32]),
    "sd_host_kq_matvec": (None, [i32, vp, vp, vp, i32, i32]),
    "sd_host_cache_clear": (None, []),
    "sd_ctx_opts_default": (None, [vp]),
    "sd_nccl_unique_id": (i32, [vp]),
    "sd_nccl_comm_create": (i32, [vp, i32, i32, i32, vp]),
    "sd_nccl_comm_destroy": (None, [vp]),
    "sd_ctx_tp_handle": (i32, [vp, vp]),
    "sd_ctx_tp_connect": (i32, [vp, vp, i32]),
    "sd_gguf_describe": (i32, [vp, sz, vp]),
    "sd_ctx_create": (i32, [vp, sz, vp, vp]),
    "sd_ctx_create_file": (i32, [C.c_char_p, vp, vp]),
    "sd_ctx_free": (None, [vp]),
    "sd_ctx_info": (i32, [vp, vp]),
    "sd_ctx_device_error": (i32, [vp]),
    "sd_ctx_stream": (vp, [vp]),
    "sd_forward": (i32, [vp, vp, i32, i32, vp, vp]),
    "sd_forward_dev": (i32, [vp, vp, i32, i32, vp, vp, vp]),
    "sd_forward_layers": (i32, [vp, i32, vp, i32, i32, vp, vp]),
    "sd_prefill": (i32, [vp, vp, i32, i32]),
    "sd_kv_read": (i32, [vp, i32, i32, i32, vp, vp]),
    "sd_ngram_draft": (i32, [vp, i32, i32, i32, i32, vp, vp]),
    "sd_spec_accept": (i32, [vp, vp, vp, vp, i32, f32, i32, u64, vp, vp]),
    "sd_sample_token": (i32, [vp, vp, i32, f32, i32, f32, f32, vp, i32, u64, vp]),
    "sd_spec_softmax": (i32, [vp, vp, vp, i32, f32]),
    "sd_spec_sample_probs": (i32, [vp, vp, i32, u64, vp]),
    "sd_embed_token": (i32, [vp, i32, vp]),
    "sd_layer_decode": (i32, [vp, vp, i32, i32]),
    "sd_logits": (i32, [vp, vp, i32, vp]),
    "sd_gen_params_default": (None, [vp]),
    "sd_generate": (i32, [vp, vp, vp, i32, vp, i32, vp]),
    "sd_decode": (i32, [vp, vp, vp, i32, i32, vp, i32, vp]),
    "sd_tokenizer_create": (i32, [vp, sz, vp]),
    "sd_tokenizer_free": (None, [vp]),
    "sd_tokenizer_info": (i32, [vp, vp, vp, vp]),
    "sd_tokenizer_entry": (i32, [vp, i32, vp, vp, vp]),
    "sd_tokenizer_encode": (i32, [vp, C.c_char_p, vp, i32, i32]),
    "sd_tokenizer_piece": (C.c_char_p, [vp, i32]),
    "sd_tokenizer_decode": (vp, [vp, vp, i32]),
    "sd_tokenizer_apply_chat": (vp, [C.c_char_p]),
    "sd_free": (None, [vp]),
    "sd_batch_create": (i32, [vp, i32, i32, i32, vp]),
    "sd_batch_free": (None, [vp]),
    "sd_batch_stream": (vp, [vp]),
    "sd_batch_set_gemm": (i32, [vp, i32]),
    "sd_batch_forward": (i32, [vp, vp, i32, vp, vp]),
    "sd_batch_prefill": (i32, [vp, vp, i32]),
    "sd_batch_decode": (i32, [vp, vp, vp, i32, vp, vp, i32, vp, vp]),
    "sd_batch_generate": (i32, [vp, vp, vp, i32, vp, i32, vp, vp]),
}

_lib = None
_lock = threading.Lock()


def build():
    subprocess.check_call(["make", "-s", "-j8", "-C", _HERE])


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(SO_PATH):
                    raise RuntimeError(f"{SO_PATH} is not built (run __graft_entry__.build()); "
                                       "there is no CPU fallback")
                L = C.CDLL(SO_PATH)
                for name, (res, args) in _SIGS.items():
                    try:
                        fn = getattr(L, name)
                    except AttributeError:
                        continue  # reported by tests/test_capi.py
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def last_error() -> str:
    return lib().sd_last_error().decode(errors="replace")


def check(rc: int, what: str = ""):
    if rc != SD_OK:
        raise SpecDecError(rc, f"{what}: {last_error()}" if what else last_error())
    return rc


def exported_symbols():
    """Names of every sd_* entry point declared in include/specdec_b200.h."""
    return sorted(_SIGS.keys())
