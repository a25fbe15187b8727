"""Host-side logic of the multi-GPU paths, on CPU with two gloo ranks (no GPU).

1. The tensor-parallel shard rule: o-proj / down-proj are split by input columns on 32-column block
   boundaries, so each rank's Q8_0 codes and per-block int32 dot sums are exactly the matching blocks of
   the unsharded matvec (bit-exact), and the rank-order sum of the ranks' partial outputs equals the full
   output up to fp32 re-association.  Ranks compute with the CPU oracle and reduce with gloo.
2. bench.py's whole-job aggregation: the slowest rank's time, and one stream's tokens under tensor
   parallelism or every stream's tokens under data parallelism.
"""
import os
import socket

import numpy as np
import pytest

ROWS, COLS = 96, 2048


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs():
    from anetransformers_b200.gguf import random_q4_0
    rng = np.random.default_rng(17)
    W = random_q4_0(rng, ROWS, COLS)
    x = rng.standard_normal(COLS).astype(np.float32)
    return W, x


def _rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        import bench
        W, x = _inputs()
        xq = O.quantize_q8_0(x)
        per = (COLS // 32) // world
        Wr, xr = W[:, rank * per:(rank + 1) * per], xq[rank * per:(rank + 1) * per]
        isum = O.block_sums(Wr, xr)
        y = torch.from_numpy(O.matvec(Wr, xr).astype(np.float32))
        # rank-order sum, as the device reduction adds the ranks' slices
        parts = [torch.zeros_like(y) for _ in range(world)]
        dist.all_gather(parts, y)
        total = torch.zeros_like(y)
        for p in parts:
            total += p
        agg_dp = bench.aggregate_ranks(dist, 10.0 + rank, 100 + rank, tp=False, device="cpu")
        agg_tp = bench.aggregate_ranks(dist, 10.0 + rank, 100 + rank, tp=True, device="cpu")
        q.put((rank, isum, total.numpy(), agg_dp, agg_tp, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, None, None, None, repr(e)))
    finally:
        dist.destroy_process_group()


def test_two_rank_column_shards_and_aggregation(oracle):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q), daemon=True) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, isum, total, agg_dp, agg_tp, err = q.get(timeout=240)
        res[r] = (isum, total, agg_dp, agg_tp, err)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert res[r][4] is None, res[r][4]

    W, x = _inputs()
    xq = oracle.quantize_q8_0(x)
    full_isum = oracle.block_sums(W, xq)
    per = (COLS // 32) // 2
    for r in range(2):
        np.testing.assert_array_equal(res[r][0], full_isum[:, r * per:(r + 1) * per])
    full_y = oracle.matvec(W, xq).astype(np.float64)
    # bound of the re-association: a few ulp of the sum of |terms|
    wd = W["d"].astype(np.float32).astype(np.float64)
    xd = xq["d"].astype(np.float64)
    scale = np.sum(np.abs(wd * xd[None, :] * full_isum), axis=1)
    for r in range(2):
        assert np.all(np.abs(res[r][1] - full_y) <= 2e-6 * scale + 1e-30)
    np.testing.assert_array_equal(res[0][1], res[1][1])   # every rank holds the same sums
    for r in range(2):
        assert res[r][2] == (11.0, 201.0)                  # data parallel: slowest time, all tokens
        assert res[r][3] == (11.0, float(100 + r))         # tensor parallel: one stream's tokens
