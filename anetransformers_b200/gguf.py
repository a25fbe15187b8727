"""GGUF v3 reader and seeded synthetic-model writer for Mistral-architecture Q4_0 models.

The on-disk format is the one the reference's loader parses (mistral/gguf_loader.h:148-325):
little-endian header ``GGUF`` / version 3 / tensor count / KV count, typed metadata KV pairs, a tensor
table (name, dims with ne[0] = columns, ggml type, offset) and a data section aligned to 32 bytes
(gguf_loader.h:280-281).  Model hyper-parameters use the ``llama.*`` keys the reference reads
(gguf_loader.h:201-233); head_dim is dim / n_heads and the vocabulary size is the length of
``tokenizer.ggml.tokens`` (gguf_loader.h:256-259).

Synthetic weights (all 2-D tensors Q4_0, including token_embd and output): every 18-byte block holds
an fp16 scale d = |N(0, 0.02)| and 16 bytes of uniformly random nibbles.  RMSNorm weights are 1.0.
Each tensor draws from its own PCG64 stream seeded by (seed, tensor index), so any tensor can be
regenerated independently and the file is identical for a given seed.
"""
from __future__ import annotations

import dataclasses
import mmap
import os
import struct
from typing import Dict, Iterator, List, Optional, Tuple

import numpy as np

GGUF_MAGIC = 0x46554747
GGML_TYPE_F32 = 0
GGML_TYPE_F16 = 1
GGML_TYPE_Q4_0 = 2
GGML_TYPE_Q4_K = 12
GGML_TYPE_Q6_K = 14
# K-quant super-blocks of 256 values (mistral/dequant.h:23-30, :283-289)
Q4_K_DTYPE = np.dtype([("d", "<f2"), ("dmin", "<f2"), ("scales", "u1", (12,)), ("qs", "u1", (128,))])
Q6_K_DTYPE = np.dtype([("ql", "u1", (128,)), ("qh", "u1", (64,)), ("scales", "i1", (16,)), ("d", "<f2")])
assert Q4_K_DTYPE.itemsize == 144 and Q6_K_DTYPE.itemsize == 210
_TYPE_NAMES = {"q4_0": 2, "q4_k": 12, "q6_k": 14}
ALIGN = 32

# GGUF metadata value types (gguf_loader.h:20-28)
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)

Q4_0_DTYPE = np.dtype([("d", "<f2"), ("qs", "u1", (16,))])
assert Q4_0_DTYPE.itemsize == 18
Q8_0_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (32,))])
assert Q8_0_DTYPE.itemsize == 36


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    dim: int = 4096
    hidden_dim: int = 14336
    n_layers: int = 32
    n_heads: int = 32
    n_kv_heads: int = 8
    vocab_size: int = 32000
    rope_theta: float = 1e6
    rms_eps: float = 1e-5
    context_length: int = 32768
    bos_id: int = 1
    eos_id: int = 2
    # vocabulary written to tokenizer.ggml.*: "plain" (specials, byte tokens, distinct filler pieces, all scores
    # 0) or "bpe" (a SentencePiece-style vocabulary with learned merges, for tokenizer tests; bpe_vocab)
    tokenizer: str = "plain"
    tokenizer_seed: int = 0
    # types of output.weight ("q4_0", "q6_k" as in the real Mistral Q4_0 GGUFs, or "q4_k") and of
    # token_embd.weight ("q4_0" or "q4_k"); every other 2-D tensor is Q4_0
    lm_head_type: str = "q4_0"
    embd_type: str = "q4_0"

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim


# Mistral-7B-v0.2 architecture.
MISTRAL_7B = ModelConfig()
# Small configs with the same head_dim (128) and 4:1 GQA, for parity tests the CPU oracle finishes fast.
MINI = ModelConfig(dim=1024, hidden_dim=3072, n_layers=2, n_heads=8, n_kv_heads=2, vocab_size=2048,
                   context_length=4096)
SMALL = ModelConfig(dim=2048, hidden_dim=5120, n_layers=4, n_heads=16, n_kv_heads=4, vocab_size=4096,
                    context_length=4096)


def tensor_names(cfg: ModelConfig) -> List[Tuple[str, int, Tuple[int, ...]]]:
    """(name, ggml type, shape as (rows, cols) or (n,)) in file order, using the reference's names
    (mistral/mistral_model.h:290-318)."""
    out: List[Tuple[str, int, Tuple[int, ...]]] = [("token_embd.weight", _TYPE_NAMES[cfg.embd_type],
                                                    (cfg.vocab_size, cfg.dim))]
    for l in range(cfg.n_layers):
        out += [
            (f"blk.{l}.attn_q.weight", GGML_TYPE_Q4_0, (cfg.dim, cfg.dim)),
            (f"blk.{l}.attn_k.weight", GGML_TYPE_Q4_0, (cfg.kv_dim, cfg.dim)),
            (f"blk.{l}.attn_v.weight", GGML_TYPE_Q4_0, (cfg.kv_dim, cfg.dim)),
            (f"blk.{l}.attn_output.weight", GGML_TYPE_Q4_0, (cfg.dim, cfg.dim)),
            (f"blk.{l}.ffn_gate.weight", GGML_TYPE_Q4_0, (cfg.hidden_dim, cfg.dim)),
            (f"blk.{l}.ffn_up.weight", GGML_TYPE_Q4_0, (cfg.hidden_dim, cfg.dim)),
            (f"blk.{l}.ffn_down.weight", GGML_TYPE_Q4_0, (cfg.dim, cfg.hidden_dim)),
            (f"blk.{l}.attn_norm.weight", GGML_TYPE_F32, (cfg.dim,)),
            (f"blk.{l}.ffn_norm.weight", GGML_TYPE_F32, (cfg.dim,)),
        ]
    out += [("output_norm.weight", GGML_TYPE_F32, (cfg.dim,)),
            ("output.weight", _TYPE_NAMES[cfg.lm_head_type], (cfg.vocab_size, cfg.dim))]
    return out


def tensor_nbytes(ttype: int, shape: Tuple[int, ...]) -> int:
    n = int(np.prod(shape))
    if ttype == GGML_TYPE_Q4_0:
        return n // 32 * 18
    if ttype == GGML_TYPE_F32:
        return n * 4
    if ttype == GGML_TYPE_F16:
        return n * 2
    if ttype == GGML_TYPE_Q4_K:
        return n // 256 * 144
    if ttype == GGML_TYPE_Q6_K:
        return n // 256 * 210
    raise ValueError(f"unsupported ggml type {ttype}")


def random_q4_0(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    """[rows, cols/32] Q4_0 blocks: d = fp16(|N(0, 0.02)|), nibbles uniform on 0..15."""
    nb = rows * (cols // 32)
    blk = np.empty(nb, dtype=Q4_0_DTYPE)
    blk["d"] = np.abs(rng.standard_normal(nb, dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    blk["qs"] = rng.integers(0, 256, size=(nb, 16), dtype=np.uint8)
    return blk.reshape(rows, cols // 32)


def random_q6_k(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    """[rows, cols/256] Q6_K super-blocks: ql / qh uniform bytes, sub-block scales int8 uniform on -32..31,
    d = fp16(|N(0, 0.02)| / 128), so that weights are of the Q4_0 tensors' magnitude."""
    nb = rows * (cols // 256)
    blk = np.empty(nb, dtype=Q6_K_DTYPE)
    blk["ql"] = rng.integers(0, 256, size=(nb, 128), dtype=np.uint8)
    blk["qh"] = rng.integers(0, 256, size=(nb, 64), dtype=np.uint8)
    blk["scales"] = rng.integers(-32, 32, size=(nb, 16), dtype=np.int8)
    blk["d"] = (np.abs(rng.standard_normal(nb, dtype=np.float32) * np.float32(0.02)) / np.float32(128)).astype(np.float16)
    return blk.reshape(rows, cols // 256)


def random_q4_k(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    """[rows, cols/256] Q4_K super-blocks: d = fp16(|N(0, 0.02)| / 256), dmin = fp16(|N(0, 0.02)| / 256), packed
    6-bit scales / mins and nibbles uniform bytes."""
    nb = rows * (cols // 256)
    blk = np.empty(nb, dtype=Q4_K_DTYPE)
    blk["d"] = (np.abs(rng.standard_normal(nb, dtype=np.float32) * np.float32(0.02)) / np.float32(256)).astype(np.float16)
    blk["dmin"] = (np.abs(rng.standard_normal(nb, dtype=np.float32) * np.float32(0.02)) / np.float32(256)).astype(np.float16)
    blk["scales"] = rng.integers(0, 256, size=(nb, 12), dtype=np.uint8)
    blk["qs"] = rng.integers(0, 256, size=(nb, 128), dtype=np.uint8)
    return blk.reshape(rows, cols // 256)


def _tensor_data(cfg: ModelConfig, seed: int, idx: int, name: str, ttype: int, shape) -> np.ndarray:
    if ttype == GGML_TYPE_F32:
        return np.ones(shape, dtype=np.float32)
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, idx])))
    if ttype == GGML_TYPE_Q6_K:
        return random_q6_k(rng, shape[0], shape[1])
    if ttype == GGML_TYPE_Q4_K:
        return random_q4_k(rng, shape[0], shape[1])
    return random_q4_0(rng, shape[0], shape[1])


def _vocab(cfg: ModelConfig) -> List[bytes]:
    toks = [b"<unk>", b"<s>", b"</s>"]
    toks += [b"<0x%02X>" % i for i in range(256)]
    i = len(toks)
    while len(toks) < cfg.vocab_size:
        toks.append(("▁t%d" % i).encode())
        i += 1
    return toks[: cfg.vocab_size]


# Characters of the bpe test vocabulary's corpus; those in BPE_OUTSIDE are left out of the vocabulary so
# that encoding them takes the byte fallback.
BPE_CHARS = list("abcdefghijklmnoprstuvwyABCDEFGHIJKLMNOPRSTUVWY0123456789.,;:!?'-()") + ["é", "ü", "ß", "ñ", "中", "文", "😀"]
BPE_OUTSIDE = ["q", "x", "z", "Q", "X", "€", "λ"]


def bpe_corpus_words(seed: int, n_words: int = 2000) -> List[str]:
    """Seeded pseudo-words (consonant-vowel syllables, some capitalised, some with digits, punctuation or
    multi-byte characters) for the bpe test vocabulary and the tokenizer tests."""
    rng = np.random.default_rng(seed)
    cons = list("bcdfghklmnprstvw")
    vows = list("aeiouy") + ["é", "ü"]
    syll = [c + v for c in cons for v in vows] + ["ß", "ñ", "中文", "😀"]
    words = []
    for _ in range(n_words):
        w = "".join(rng.choice(syll, int(rng.integers(1, 5))))
        r = rng.random()
        if r < 0.15:
            w = w[0].upper() + w[1:]
        elif r < 0.2:
            w += str(int(rng.integers(0, 100)))
        elif r < 0.3:
            w += str(rng.choice(list(".,;:!?")))
        words.append(w)
    return words


def bpe_vocab(size: int, seed: int = 0, max_merges: int = 900) -> Tuple[List[bytes], np.ndarray, np.ndarray]:
    """A SentencePiece-style vocabulary of `size` pieces for tokenizer tests: <unk> (UNKNOWN), <s> and </s>
    (CONTROL), the 256 byte tokens <0xNN> (BYTE), U+2581 and the single characters of BPE_CHARS, then merges
    learned by pair counting on the words of bpe_corpus_words (each word prefixed by U+2581), in merge order
    (at most max_merges).
    A merged piece's score is -(rank // 3), so runs of three merges share a score (equal-score merges must
    resolve in the reference's order).  Pieces are unique; the rest is filled with unmergeable <fN> pieces."""
    pieces: List[str] = ["<unk>", "<s>", "</s>"] + ["<0x%02X>" % i for i in range(256)]
    types = [2, 3, 3] + [6] * 256
    scores = [0.0] * len(pieces)
    singles = ["\u2581"] + BPE_CHARS
    for ch in singles:
        pieces.append(ch)
        types.append(1)
        scores.append(-1e6)
    have = set(pieces)
    counts: dict = {}
    for w in bpe_corpus_words(seed):
        key = tuple(["\u2581"] + [c for c in w])
        counts[key] = counts.get(key, 0) + 1
    words = [(list(k), n) for k, n in counts.items()]
    rank = 0
    while len(pieces) < size and rank < max_merges:
        pc: dict = {}
        for syms, n in words:
            for a, b in zip(syms, syms[1:]):
                pc[(a, b)] = pc.get((a, b), 0) + n
        if not pc:
            break
        (a, b), _ = max(pc.items(), key=lambda kv: (kv[1], kv[0]))
        m = a + b
        for i, (syms, n) in enumerate(words):
            j, out = 0, []
            while j < len(syms):
                if j + 1 < len(syms) and syms[j] == a and syms[j + 1] == b:
                    out.append(m)
                    j += 2
                else:
                    out.append(syms[j])
                    j += 1
            words[i] = (out, n)
        if m not in have:
            have.add(m)
            pieces.append(m)
            types.append(1)
            scores.append(-float(rank // 3))
            rank += 1
    k = 0
    while len(pieces) < size:
        pieces.append("<f%d>" % k)
        types.append(1)
        scores.append(-1e9)
        k += 1
    return [p.encode() for p in pieces[:size]], np.array(scores[:size], "<f4"), np.array(types[:size], "<i4")


def _kv_str(key: str, val: str) -> bytes:
    k = key.encode()
    v = val.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<I", _STR) + struct.pack("<Q", len(v)) + v


def _kv_u32(key: str, val: int) -> bytes:
    k = key.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<II", _U32, val)


def _kv_f32(key: str, val: float) -> bytes:
    k = key.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<If", _F32, val)


def _header(cfg: ModelConfig) -> Tuple[bytes, List[Tuple[str, int, Tuple[int, ...], int]]]:
    kvs = [
        _kv_str("general.architecture", "llama"),
        _kv_u32("llama.embedding_length", cfg.dim),
        _kv_u32("llama.feed_forward_length", cfg.hidden_dim),
        _kv_u32("llama.block_count", cfg.n_layers),
        _kv_u32("llama.attention.head_count", cfg.n_heads),
        _kv_u32("llama.attention.head_count_kv", cfg.n_kv_heads),
        _kv_u32("llama.context_length", cfg.context_length),
        _kv_f32("llama.rope.freq_base", cfg.rope_theta),
        _kv_f32("llama.attention.layer_norm_rms_epsilon", cfg.rms_eps),
        _kv_u32("tokenizer.ggml.bos_token_id", cfg.bos_id),
        _kv_u32("tokenizer.ggml.eos_token_id", cfg.eos_id),
        _kv_u32("tokenizer.ggml.unknown_token_id", 0),
    ]
    if cfg.tokenizer == "bpe":
        vocab, scores, types = bpe_vocab(cfg.vocab_size, cfg.tokenizer_seed)
    else:
        vocab = _vocab(cfg)
        scores = np.zeros(len(vocab), "<f4")
        types = np.ones(len(vocab), "<i4")
        types[:3] = 3
        types[3:259] = 6
    k = b"tokenizer.ggml.tokens"
    arr = struct.pack("<Q", len(k)) + k + struct.pack("<IIQ", _ARR, _STR, len(vocab))
    arr += b"".join(struct.pack("<Q", len(t)) + t for t in vocab)
    kvs.append(arr)
    k = b"tokenizer.ggml.scores"
    kvs.append(struct.pack("<Q", len(k)) + k + struct.pack("<IIQ", _ARR, _F32, len(vocab)) + scores.tobytes())
    k = b"tokenizer.ggml.token_type"
    kvs.append(struct.pack("<Q", len(k)) + k + struct.pack("<IIQ", _ARR, _I32, len(vocab)) + types.tobytes())

    table = []
    off = 0
    tinfo = b""
    for name, ttype, shape in tensor_names(cfg):
        nbytes = tensor_nbytes(ttype, shape)
        ne = tuple(reversed(shape))  # ggml: ne[0] = columns
        nm = name.encode()
        tinfo += struct.pack("<Q", len(nm)) + nm + struct.pack("<I", len(ne))
        tinfo += b"".join(struct.pack("<Q", d) for d in ne)
        tinfo += struct.pack("<IQ", ttype, off)
        table.append((name, ttype, shape, off))
        off += (nbytes + ALIGN - 1) // ALIGN * ALIGN
    head = struct.pack("<IIQQ", GGUF_MAGIC, 3, len(table), len(kvs)) + b"".join(kvs) + tinfo
    pad = (-len(head)) % ALIGN
    return head + b"\0" * pad, table


def iter_synthetic_gguf(cfg: ModelConfig, seed: int) -> Iterator[bytes]:
    """Yield the synthetic model file in pieces (header, then each tensor + padding)."""
    head, table = _header(cfg)
    yield head
    for idx, (name, ttype, shape, _off) in enumerate(table):
        data = _tensor_data(cfg, seed, idx, name, ttype, shape).tobytes()
        yield data
        pad = (-len(data)) % ALIGN
        if pad:
            yield b"\0" * pad


def write_synthetic_gguf(path: str, cfg: ModelConfig = MISTRAL_7B, seed: int = 0) -> str:
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        for chunk in iter_synthetic_gguf(cfg, seed):
            f.write(chunk)
    os.replace(tmp, path)
    return path


def synthetic_gguf_bytes(cfg: ModelConfig, seed: int = 0) -> bytes:
    return b"".join(iter_synthetic_gguf(cfg, seed))


def _write_tensor_job(args):
    path, cfg, seed, idx, name, ttype, shape, abs_off = args
    data = _tensor_data(cfg, seed, idx, name, ttype, shape)
    fd = os.open(path, os.O_WRONLY)
    try:
        os.pwrite(fd, data.tobytes(), abs_off)
    finally:
        os.close(fd)
    return idx


def write_synthetic_gguf_parallel(path: str, cfg: ModelConfig = MISTRAL_7B, seed: int = 0,
                                  workers: Optional[int] = None) -> str:
    """Same bytes as write_synthetic_gguf, tensors generated by a spawn-started process pool and written
    at their offsets (each tensor depends only on (seed, tensor index))."""
    import concurrent.futures as cf
    import multiprocessing as mp
    head, table = _header(cfg)
    last_name, last_type, last_shape, last_off = table[-1]
    total = len(head) + last_off + tensor_nbytes(last_type, last_shape)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(head)
        f.truncate(total)
    jobs = [(tmp, cfg, seed, i, n, t, sh, len(head) + off) for i, (n, t, sh, off) in enumerate(table)]
    jobs.sort(key=lambda j: -tensor_nbytes(j[5], j[6]))
    workers = workers or max(1, min(16, os.cpu_count() or 1))
    with cf.ProcessPoolExecutor(max_workers=workers, mp_context=mp.get_context("spawn")) as ex:
        list(ex.map(_write_tensor_job, jobs, chunksize=1))
    os.replace(tmp, path)
    return path


# ----------------------------------------------------------------------------------------------
# Reader
# ----------------------------------------------------------------------------------------------
@dataclasses.dataclass
class GGUFTensorInfo:
    name: str
    ttype: int
    shape: Tuple[int, ...]     # (rows, cols) for 2-D
    offset: int                # absolute file offset


class GGUFFile:
    """Minimal GGUF v3 reader over a file path or an in-memory buffer (mirrors gguf_loader.h:148-325)."""

    def __init__(self, src):
        if isinstance(src, (bytes, bytearray, memoryview)):
            self._mm = None
            self.buf = memoryview(src)
        else:
            fd = os.open(src, os.O_RDONLY)
            try:
                self._mm = mmap.mmap(fd, 0, access=mmap.ACCESS_READ)
            finally:
                os.close(fd)
            self.buf = memoryview(self._mm)
        self.meta: Dict[str, object] = {}
        self.tensors: Dict[str, GGUFTensorInfo] = {}
        self._parse()

    def _parse(self):
        b = self.buf
        pos = 0

        def rd(fmt):
            nonlocal pos
            v = struct.unpack_from(fmt, b, pos)
            pos += struct.calcsize(fmt)
            return v[0] if len(v) == 1 else v

        def rstr():
            n = rd("<Q")
            nonlocal pos
            s = bytes(b[pos:pos + n])
            pos += n
            return s

        scalar = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f",
                  _BOOL: "<B", _U64: "<Q", _I64: "<q", _F64: "<d"}

        def rval(t):
            if t in scalar:
                return rd(scalar[t])
            if t == _STR:
                return rstr()
            if t == _ARR:
                at = rd("<I")
                n = rd("<Q")
                if at in scalar:
                    nonlocal pos
                    dt = np.dtype(scalar[at])
                    arr = np.frombuffer(b, dtype=dt, count=n, offset=pos)
                    pos += n * dt.itemsize
                    return arr
                return [rval(at) for _ in range(n)]
            raise ValueError(f"bad GGUF value type {t}")

        magic, self.version, n_t, n_kv = rd("<IIQQ")
        if magic != GGUF_MAGIC:
            raise ValueError("not a GGUF file")
        for _ in range(n_kv):
            key = rstr().decode()
            t = rd("<I")
            self.meta[key] = rval(t)
        infos = []
        for _ in range(n_t):
            name = rstr().decode()
            nd = rd("<I")
            ne = [rd("<Q") for _ in range(nd)]
            ttype = rd("<I")
            off = rd("<Q")
            infos.append((name, ttype, tuple(reversed(ne)), off))
        self.data_start = (pos + ALIGN - 1) // ALIGN * ALIGN
        for name, ttype, shape, off in infos:
            self.tensors[name] = GGUFTensorInfo(name, ttype, shape, self.data_start + off)

    def config(self) -> ModelConfig:
        m = self.meta

        def g(k, d=None):
            for pre in ("llama.", "mistral."):
                if pre + k in m:
                    return m[pre + k]
            return d
        return ModelConfig(dim=int(g("embedding_length")), hidden_dim=int(g("feed_forward_length")),
                           n_layers=int(g("block_count")), n_heads=int(g("attention.head_count")),
                           n_kv_heads=int(g("attention.head_count_kv")),
                           vocab_size=len(m.get("tokenizer.ggml.tokens", [])) or 32000,
                           rope_theta=float(g("rope.freq_base", 10000.0)),
                           rms_eps=float(g("attention.layer_norm_rms_epsilon", 1e-5)),
                           context_length=int(g("context_length", 4096)),
                           bos_id=int(m.get("tokenizer.ggml.bos_token_id", 1)),
                           eos_id=int(m.get("tokenizer.ggml.eos_token_id", 2)))

    def array(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        if t.ttype == GGML_TYPE_Q4_0:
            rows, cols = t.shape
            return np.frombuffer(self.buf, dtype=Q4_0_DTYPE, count=rows * cols // 32,
                                 offset=t.offset).reshape(rows, cols // 32)
        if t.ttype == GGML_TYPE_F32:
            return np.frombuffer(self.buf, dtype="<f4", count=int(np.prod(t.shape)), offset=t.offset)
        if t.ttype in (GGML_TYPE_Q4_K, GGML_TYPE_Q6_K):
            rows, cols = t.shape
            dt = Q4_K_DTYPE if t.ttype == GGML_TYPE_Q4_K else Q6_K_DTYPE
            return np.frombuffer(self.buf, dtype=dt, count=rows * cols // 256, offset=t.offset).reshape(rows, cols // 256)
        raise ValueError(f"unsupported type {t.ttype}")

    def close(self):
        """Drop the mapping (arrays handed out keep it alive until they are released)."""
        try:
            self.buf.release()
            if self._mm is not None:
                self._mm.close()
        except BufferError:
            pass
