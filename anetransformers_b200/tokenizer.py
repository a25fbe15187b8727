"""Host mirror of the reference's mistral/tokenizer.h over the library's tokenizer (sd_tokenizer_*).

``Tokenizer(path_or_bytes)`` is tokenizer_init on a GGUF; ``encode`` / ``decode_token`` / ``decode`` /
``apply_chat`` are tokenizer_encode / tokenizer_decode_token / tokenizer_decode / tokenizer_apply_chat.
"""
from __future__ import annotations

import ctypes as C
from typing import List, Sequence

import numpy as np

from . import _lib


def apply_chat(user_msg: str) -> str:
    """mistral/tokenizer.h tokenizer_apply_chat: the Mistral instruct template."""
    p = _lib.lib().sd_tokenizer_apply_chat(user_msg.encode())
    try:
        return C.string_at(p).decode("utf-8", errors="surrogateescape")
    finally:
        _lib.lib().sd_free(p)


class Tokenizer:
    def __init__(self, model):
        if isinstance(model, (bytes, bytearray)):
            buf = bytes(model)
        else:
            with open(str(model), "rb") as f:   # the metadata (vocabulary) sits at the start of the file
                buf = f.read(64 << 20)
        self._buf = C.create_string_buffer(buf, len(buf))
        base, n = C.addressof(self._buf), len(buf)
        h = C.c_void_p()
        _lib.check(_lib.lib().sd_tokenizer_create(base, n, C.byref(h)), "sd_tokenizer_create")
        self.h = h
        vs, bos, eos = C.c_int(), C.c_int(), C.c_int()
        _lib.check(_lib.lib().sd_tokenizer_info(h, C.byref(vs), C.byref(bos), C.byref(eos)), "sd_tokenizer_info")
        self.vocab_size, self.bos_id, self.eos_id = vs.value, bos.value, eos.value

    def close(self):
        if getattr(self, "h", None):
            _lib.lib().sd_tokenizer_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode(self, text: str, add_bos: bool = True, max_tokens: int = 1 << 20) -> List[int]:
        raw = text.encode("utf-8", errors="surrogateescape")
        out = np.empty(max(1, min(max_tokens, 3 * len(raw) + 4)), np.int32)  # a space can fall back to 3 byte tokens
        n = _lib.lib().sd_tokenizer_encode(self.h, raw, out.ctypes.data, out.size, int(add_bos))
        if n < 0:
            _lib.check(n, "sd_tokenizer_encode")
        return out[:n].tolist()

    def decode_token(self, token: int) -> bytes:
        return _lib.lib().sd_tokenizer_piece(self.h, token) or b""

    def decode(self, tokens: Sequence[int]) -> str:
        t = np.ascontiguousarray(tokens, np.int32)
        p = _lib.lib().sd_tokenizer_decode(self.h, t.ctypes.data if t.size else None, t.size)
        if not p:
            raise MemoryError("sd_tokenizer_decode")
        try:
            return C.string_at(p).decode("utf-8", errors="surrogateescape")
        finally:
            _lib.lib().sd_free(p)

    def entry(self, token: int):
        s, sc, ty = C.c_char_p(), C.c_float(), C.c_int()
        _lib.check(_lib.lib().sd_tokenizer_entry(self.h, token, C.byref(s), C.byref(sc), C.byref(ty)), "sd_tokenizer_entry")
        return s.value, sc.value, ty.value
