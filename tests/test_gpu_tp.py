"""Tensor parallelism (Wq/Wk/Wv/W1/W3 by rows, Wo/W2 by columns, an all-reduce after o-proj and
down-proj -- by NCCL, or inside the norm kernels over peer memory) against the single-GPU context on the
MINI model: both ranks agree bit for bit, logits stay
within the 1e-2 relative bar (only the fp32 partial-sum order differs), and greedy tokens match up to a
near-tie of the single-GPU logits.  Needs two GPUs; each rank is its own process, as in deployment.
"""
import os
import socket

import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a CUDA GPU")]

LOGIT_RTOL = 1e-2


def _n_gpus():
    import torch
    return torch.cuda.device_count()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _tokens():
    rng = np.random.default_rng(11)
    return rng.integers(3, 2048, 12).tolist()


def _tokens12():
    rng = np.random.default_rng(12)
    return rng.integers(3, 2048, 12).tolist()


def _worker(rank, world, path, port, q, mode):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(rank)
        from anetransformers_b200.engine import Context, NcclComm, nccl_unique_id
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, 0)
        comm = NcclComm(obj[0], world, rank, rank)
        ctx = Context(path, device=rank, max_seq=256, tp_rank=rank, tp_size=world, nccl_comm=comm.handle)
        if mode == "peer":
            # all-reduce inside the norm kernels over NVLink instead of NCCL
            handles = [None] * world
            dist.all_gather_object(handles, ctx.tp_handle())
            ctx.tp_connect(handles)
        toks = _tokens()
        ctx.prefill(toks[:7], 0)
        lg, _ = ctx.forward(toks[7:], 7)
        # a 12-token verify (two consecutive forwards under tensor parallelism)
        ctx.prefill(toks[:3], 0)
        lg12, _ = ctx.forward(_tokens12(), 3)
        out, _ = ctx.generate(toks, mode="greedy", max_tokens=12, temp=0.0, rep_penalty=1.0, ignore_eos=True)
        q.put((rank, (lg, lg12), out, None))
        ctx.close()
        comm.close()
    except Exception as e:  # reported to the parent
        q.put((rank, None, None, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def mini(tmp_path_factory):
    from anetransformers_b200 import gguf as G
    path = str(tmp_path_factory.mktemp("tp") / "mini.gguf")
    G.write_synthetic_gguf(path, G.MINI, seed=5)
    return path


@pytest.mark.skipif(gpu_available() and _n_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["nccl", "peer"])
def test_tp2_matches_single_gpu(mini, mode):
    import multiprocessing as mp
    from anetransformers_b200.engine import Context

    ref = Context(mini, device=0, max_seq=256)
    toks = _tokens()
    ref.prefill(toks[:3], 0)
    lg12_ref, _ = ref.forward(_tokens12(), 3)
    ref.prefill(toks[:7], 0)
    lg_ref, _ = ref.forward(toks[7:], 7)
    out_ref, _ = ref.generate(toks, mode="greedy", max_tokens=12, temp=0.0, rep_penalty=1.0, ignore_eos=True)

    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    port = _free_port()
    procs = [ctxm.Process(target=_worker, args=(r, 2, mini, port, q, mode), daemon=True) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, lg, out, err = q.get(timeout=300)
        res[rank] = (lg, out, err)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert res[r][2] is None, res[r][2]
    ((lg0, lg12_0), out0, _), ((lg1, lg12_1), out1, _) = res[0], res[1]
    # ranks agree bit for bit (the all-reduce hands every rank the same sums)
    np.testing.assert_array_equal(lg0.view(np.uint32), lg1.view(np.uint32))
    np.testing.assert_array_equal(lg12_0.view(np.uint32), lg12_1.view(np.uint32))
    assert out0 == out1
    # vs one GPU: only the partial-sum order differs
    for a, b in ((lg0, lg_ref), (lg12_0, lg12_ref)):
        err = np.max(np.abs(a.astype(np.float64) - b)) / np.max(np.abs(b))
        assert err < LOGIT_RTOL, err
    if out0 != out_ref:
        i = next(j for j in range(min(len(out0), len(out_ref))) if out0[j] != out_ref[j])
        # the single-GPU logits that chose token i
        hist = toks + out_ref[:i]
        ref.prefill(hist[:-1], 0)
        lg, _ = ref.forward([hist[-1]], len(hist) - 1)
        s = np.sort(lg[0])
        assert s[-1] - s[-2] <= 1e-3 * np.max(np.abs(lg[0])), (i, out0, out_ref)
    ref.close()


def _worker_both(rank, world, path, port, q):
    """Per rank: the persistent-kernel forward and the per-op forward, both tensor parallel over peer
    memory, on the same inputs."""
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(rank)
        from anetransformers_b200.engine import Context, NcclComm, nccl_unique_id
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, 0)
        comm = NcclComm(obj[0], world, rank, rank)
        res = []
        for fk in (1, 0):
            ctx = Context(path, device=rank, max_seq=256, tp_rank=rank, tp_size=world, nccl_comm=comm.handle,
                          forward_kernel=fk)
            handles = [None] * world
            dist.all_gather_object(handles, ctx.tp_handle())
            ctx.tp_connect(handles)
            toks = _tokens()
            ctx.prefill(toks[:7], 0)
            lg, _ = ctx.forward(toks[7:], 7)
            res.append((ctx.info.forward_kernel, lg))
            ctx.close()
        q.put((rank, res, None))
        comm.close()
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(gpu_available() and _n_gpus() < 2, reason="needs 2 GPUs")
def test_tp2_persistent_forward_equals_per_op(mini):
    import multiprocessing as mp
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    port = _free_port()
    procs = [ctxm.Process(target=_worker_both, args=(r, 2, mini, port, q), daemon=True) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        rank, res, err = q.get(timeout=300)
        assert err is None, err
        out[rank] = res
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        (fk1, lg1), (fk0, lg0) = out[r]
        assert fk1 == 1 and fk0 == 0
        np.testing.assert_array_equal(lg1.view(np.uint32), lg0.view(np.uint32))
    np.testing.assert_array_equal(out[0][0][1].view(np.uint32), out[1][0][1].view(np.uint32))
