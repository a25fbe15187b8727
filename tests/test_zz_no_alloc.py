"""The allocation-free matvec entry point against the regular one, through the C ABI.

sd_matvec_q4_0_q8_0_noalloc_dev serves callers that cannot have device memory allocated for them: a
process that gives all free HBM to its own pool at start-up, or a latency loop that cannot take the
device-wide synchronisation of a cudaFree.  It keeps K-split partial outputs in a fixed array of
SD_NOALLOC_SCRATCH_BYTES per GPU instead of a workspace that grows with cudaMalloc, and must give the
same outputs as sd_matvec_q4_0_q8_0_dev.  Both run the same kernel with the same plan, so the bar is
bit-equality (tighter than the oracle tolerance of the other matvec tests).

The file name sorts last so that a run stopping at its first failure has run every other test.
"""
import ctypes as C

import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a CUDA GPU")]

SCRATCH_BYTES = 1 << 20  # SD_NOALLOC_SCRATCH_BYTES in include/specdec_b200.h


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def _act(dq, rng, S, cols):
    import torch
    x = rng.standard_normal((S, cols)).astype(np.float32) * rng.uniform(0.1, 10, (S, 1)).astype(np.float32)
    return dq.quantize_dev(torch.from_numpy(x).cuda())


def _noalloc(lib, W, act, S):
    import torch
    y = torch.full((S, W.rows), float("nan"), dtype=torch.float32, device="cuda")
    rc = lib.sd_matvec_q4_0_q8_0_noalloc_dev(W.h, act.ptrs(), C.c_void_p(y.data_ptr()), S, C.c_void_p(_stream()))
    return rc, y


def _regular(lib, W, act, S):
    import torch
    y = torch.full((S, W.rows), float("nan"), dtype=torch.float32, device="cuda")
    rc = lib.sd_matvec_q4_0_q8_0_dev(W.h, act.ptrs(), C.c_void_p(y.data_ptr()), S, C.c_void_p(_stream()))
    return rc, y


# (rows, cols, S of the first call, S of the second call).  14336 columns at S >= 5 take the K-split
# plan (partials in the fixed array); 4096 columns at S = 1 write y directly.
CASES = [
    (4096, 14336, 8, 5),    # Mistral-7B down projection: 7 K parts, 896 KiB of partials at S = 8
    (1000, 14336, 6, 8),    # ragged rows (not a multiple of 16)
    (4096, 4096, 1, 3),
]


@pytest.mark.parametrize("rows,cols,s1,s2", CASES)
def test_noalloc_matches_regular_two_calls(rows, cols, s1, s2):
    import torch
    from anetransformers_b200 import _lib, dequant as dq
    from anetransformers_b200.gguf import random_q4_0

    lib = _lib.lib()
    rng = np.random.default_rng(rows * 7 + cols + s1)
    W = dq.QMat(random_q4_0(rng, rows, cols))
    a1 = _act(dq, rng, s1, cols)
    a2 = _act(dq, rng, s2, cols)
    # two no-alloc calls in a row: the second one finds the first one's partials in the shared array
    rc1, y1 = _noalloc(lib, W, a1, s1)
    assert rc1 == 0, _lib.lib().sd_last_error().decode()
    rc2, y2 = _noalloc(lib, W, a2, s2)
    assert rc2 == 0, _lib.lib().sd_last_error().decode()
    torch.cuda.synchronize()
    r1 = _regular(lib, W, a1, s1)[1]
    r2 = _regular(lib, W, a2, s2)[1]
    torch.cuda.synchronize()
    assert torch.isfinite(y1).all() and torch.isfinite(y2).all()
    np.testing.assert_array_equal(y1.cpu().numpy().view(np.uint32), r1.cpu().numpy().view(np.uint32))
    np.testing.assert_array_equal(y2.cpu().numpy().view(np.uint32), r2.cpu().numpy().view(np.uint32))
    W.close()


def test_noalloc_rejects_oversize():
    from anetransformers_b200 import _lib, dequant as dq
    from anetransformers_b200.gguf import random_q4_0

    lib = _lib.lib()
    rng = np.random.default_rng(5)
    rows, cols, S = 5120, 14336, 8   # 7 K parts x 8 tokens x 5120 rows x 4 B = 1.09 MiB > 1 MiB
    assert rows * S * 7 * 4 > SCRATCH_BYTES
    W = dq.QMat(random_q4_0(rng, rows, cols))
    act = _act(dq, rng, S, cols)
    rc, _ = _noalloc(lib, W, act, S)
    assert rc == -1  # SD_ERR_INVALID
    assert "limit" in lib.sd_last_error().decode()
    # the regular entry point still serves the shape
    assert _regular(lib, W, act, S)[0] == 0
    W.close()
