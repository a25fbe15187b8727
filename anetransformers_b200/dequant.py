"""Host mirror of the reference's dequant.h entry points on the B200 kernels.

Names and argument meaning follow mistral/dequant.h: ``quantize_f32_to_q8_0`` (:545-599) and
``q4_0_q8_0_matvec_sdot_parallel`` (:1022-1137) on host arrays, plus device-tensor forms used by the
verify forward (S activation rows share one weight read).  Every call goes through libspecdec_b200.so.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .gguf import Q4_0_DTYPE, Q8_0_DTYPE

QK = 32


def quantize_f32_to_q8_0(x: np.ndarray) -> np.ndarray:
    """Reference signature (host in, host out): fp32 [n] -> n/32 Q8_0 blocks (fp32 d + 32 int8)."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    if x.size % QK:
        raise ValueError("n must be a multiple of 32")
    out = np.zeros(x.size // QK, dtype=Q8_0_DTYPE)
    L = _lib.lib()
    L.sd_host_quantize_f32_to_q8_0(x.ctypes.data, out.ctypes.data, x.size)
    err = _lib.last_error()
    if err:
        raise _lib.SpecDecError(-3, err)
    return out


def q4_0_q8_0_matvec_sdot_parallel(W: np.ndarray, x_q8: np.ndarray, out_dim: int, in_dim: int) -> np.ndarray:
    """Reference signature: y[out_dim] = W (Q4_0 [out_dim][in_dim/32]) x x_q8 (Q8_0 [in_dim/32])."""
    W = np.ascontiguousarray(W)
    x_q8 = np.ascontiguousarray(x_q8)
    if W.dtype != Q4_0_DTYPE or x_q8.dtype != Q8_0_DTYPE:
        raise TypeError("W must be Q4_0 blocks and x_q8 Q8_0 blocks")
    if W.size != out_dim * in_dim // QK or x_q8.size != in_dim // QK:
        raise ValueError("shape mismatch")
    y = np.zeros(out_dim, dtype=np.float32)
    L = _lib.lib()
    L.sd_host_q4_0_q8_0_matvec(W.ctypes.data, x_q8.ctypes.data, y.ctypes.data, out_dim, in_dim)
    err = _lib.last_error()
    if err:
        raise _lib.SpecDecError(-3, err)
    return y


class QMat:
    """Device-resident repacked Q4_0 matrix (sd_qmat)."""

    def __init__(self, W: np.ndarray, device: int = 0):
        W = np.ascontiguousarray(W)
        if W.dtype != Q4_0_DTYPE or W.ndim != 2:
            raise TypeError("W must be a 2-D array of Q4_0 blocks")
        self.rows, self.cols = W.shape[0], W.shape[1] * QK
        h = C.c_void_p()
        _lib.check(_lib.lib().sd_qmat_create(W.ctypes.data, self.rows, self.cols, device, C.byref(h)), "sd_qmat_create")
        self.h = h

    def close(self):
        if self.h:
            _lib.lib().sd_qmat_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Q8Act:
    """Q8_0 activation planes for S rows of n values, in torch device tensors."""

    def __init__(self, S: int, n: int, device="cuda"):
        import torch
        self.S, self.n = S, n
        self.qs = torch.zeros(S, n, dtype=torch.int8, device=device)
        self.d = torch.zeros(S, n // QK, dtype=torch.float32, device=device)
        self.sum = torch.zeros(S, n // QK, dtype=torch.int32, device=device)

    def ptrs(self) -> _lib.Q8Dev:
        return _lib.Q8Dev(self.qs.data_ptr(), self.d.data_ptr(), self.sum.data_ptr())


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def quantize_dev(x, act: Q8Act = None) -> Q8Act:
    """x: torch cuda float32 [S, n] -> Q8Act (bit-exact reference codes and scales)."""
    S, n = x.shape
    act = act or Q8Act(S, n, x.device)
    _lib.check(_lib.lib().sd_quantize_q8_0_dev(x.contiguous().data_ptr(), act.ptrs(), S, n, _stream()), "quantize")
    return act


def q8_to_blocks_dev(act: Q8Act):
    import torch
    out = torch.zeros(act.S * act.n // QK * 36, dtype=torch.uint8, device=act.qs.device)
    _lib.check(_lib.lib().sd_q8_to_blocks_dev(act.ptrs(), out.data_ptr(), act.S, act.n, _stream()), "q8_to_blocks")
    return out


def blocks_to_q8_dev(blocks: np.ndarray, S: int, n: int, device="cuda") -> Q8Act:
    import torch
    raw = torch.from_numpy(np.ascontiguousarray(blocks).view(np.uint8).copy()).to(device)
    act = Q8Act(S, n, device)
    _lib.check(_lib.lib().sd_blocks_to_q8_dev(raw.data_ptr(), act.ptrs(), S, n, _stream()), "blocks_to_q8")
    return act


def matvec_dev(W: QMat, act: Q8Act, y=None):
    import torch
    y = y if y is not None else torch.empty(act.S, W.rows, dtype=torch.float32, device=act.qs.device)
    _lib.check(_lib.lib().sd_matvec_q4_0_q8_0_dev(W.h, act.ptrs(), y.data_ptr(), act.S, _stream()), "matvec")
    return y


def block_sums_dev(W: QMat, act: Q8Act):
    import torch
    out = torch.zeros(W.rows, W.cols // QK, dtype=torch.int32, device=act.qs.device)
    _lib.check(_lib.lib().sd_block_sums_dev(W.h, act.ptrs(), out.data_ptr(), _stream()), "block_sums")
    return out


def kq_matvec(W: np.ndarray, x: np.ndarray, ttype: int) -> np.ndarray:
    """The reference's fp32 K-quant matvec (q4_matvec for Q6_K = 14 / Q4_K = 12, mistral/mistral_model.h:211-242):
    y = W x for W [out_dim, in_dim/256] GGUF super-blocks and fp32 x."""
    W = np.ascontiguousarray(W)
    x = np.ascontiguousarray(x, np.float32)
    out_dim, in_dim = W.shape[0], x.size
    if W.shape[1] * 256 != in_dim:
        raise ValueError("shape mismatch")
    y = np.zeros(out_dim, dtype=np.float32)
    L = _lib.lib()
    L.sd_host_kq_matvec(ttype, W.ctypes.data, x.ctypes.data, y.ctypes.data, out_dim, in_dim)
    err = _lib.last_error()
    if err:
        raise _lib.SpecDecError(-3, err)
    return y
