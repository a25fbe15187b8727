#!/usr/bin/env python3
"""Benchmark: Mistral-7B Q4_0 speculative decode on B200.

Workload: Mistral-7B-v0.2 architecture with seeded random-init Q4_0 weights
(all 2-D tensors Q4_0, norms = 1); a 1024-token prompt of 16 segments drawn with replacement from a
pool of 6 random 64-token segments; n-gram (prompt-lookup) drafting with n=3, K=4; temp 0; 512 tokens.
A step = one 512-token speculative decode from the prefilled prompt (the prompt's KV stays resident in
HBM; every step re-decodes the same 512 positions).  value = generated tokens / device time.

Every forward streams the 4.0 GB of Q4_0 weights (> 126 MB L2), so no L2 flush is needed between steps.

N > 1 (torchrun): configs 3 and 4 run tensor-parallel (BASELINE's layout): Wq/Wk/Wv/W1/W3 split by rows,
Wo/W2 by columns, the sum all-reduce after o-proj and down-proj over NVLink peer memory (or NCCL with
--tp-allreduce nccl); value = the one stream's tokens / max-over-ranks time (strong scaling).  --parallel dp
runs one independent stream per GPU instead; config 5 (serving) is always data-parallel replicas (weak
scaling, value = all ranks' tokens / max-over-ranks time).

--impl reference: the reference's CPU decode path, restated in C (oracle/, the reference itself needs
arm_neon.h / GCD / Accelerate and does not compile on x86), timed on the host cores on a bounded sample.

Other workloads (--workload): greedy = config 2 (greedy decode without speculation, 128-token prompt, 256
tokens), selfspec = config 4 (self-speculation, 32K context), gemv = config 1 (single
W4A8 matvec), serving = config 5 (64 streams per GPU through the batched path, 4096-token contexts, K=4 n-gram,
one batch per rank under torchrun), forward / serving-forward = single forwards for profiling.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Mistral-7B Q4_0 spec-decode tok/s @1/2/4/8 B200; W4A8 GEMV HBM GB/s"
UNIT = "tok/s"
PROMPT_LEN, GEN_TOKENS, NGRAM_N, SPEC_K = 1024, 512, 3, 4
# self-speculative decode, K = 8 drafts from the first 8 layers, 32768-position KV
SELF_CTX, SELF_TOKENS, SELF_K, SELF_LAYERS = 32768, 256, 8, 8
GREEDY_PROMPT, GREEDY_TOKENS = 128, 256
GREEDY_PUBLISHED = 17.8  # tok/s: the reference's published non-speculative decode of 256 tokens (its README.md:137)
def kernels_per_iter(persistent: bool, tp_peer: bool = False, tp_nccl: bool = False, layers: int = 32) -> int:
    """Our kernel launches per n-gram decode iteration: prepare + commit around one verify forward, which
    is k_forward + argmax on the persistent path, or embed-norm, 8 per layer, LM head + argmax per op.
    Tensor parallel adds the sequence-advance kernel (peer path) or the NCCL all-reduces."""
    n = 2 + (2 if persistent else 1 + 8 * layers + 2)
    if tp_peer:
        n += 1
    if tp_nccl:
        n += 2 * layers
    return n
BYTES_PER_FORWARD = 32 * 122_683_392 + 73_728_000   # Q4_0 weights streamed per forward (3.9996 GB)
KV_BYTES_PER_POS = 32 * 2 * 1024 * 2                # fp16 K+V of one position, all layers


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def aggregate_ranks(dist, ms: float, tokens: float, tp: bool, device="cuda"):
    """Whole-job time and tokens over the ranks: the slowest rank's time (max), and the tokens of one
    stream under tensor parallelism (every rank emits the same tokens) or of all streams (data parallel:
    the sum).  Every rank takes part (two all-reduces in the same order)."""
    if dist is None:
        return ms, float(tokens)
    import torch
    t = torch.tensor([ms, float(tokens)], device=device, dtype=torch.float64)
    mx = t.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    sm = t.clone()
    dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    return float(mx[0]), (float(tokens) if tp else float(sm[1]))


def config3_prompt(seed: int = 1234, vocab: int = 32000):
    rng = np.random.default_rng(seed)
    pool = [rng.integers(3, vocab, 64).tolist() for _ in range(6)]
    picks = rng.integers(0, 6, 16)
    return sum((pool[i] for i in picks), [])


def model_path(rank: int, world: int, dist) -> str:
    from anetransformers_b200 import gguf as G
    path = os.environ.get("SPECDEC_BENCH_MODEL") or os.path.join(tempfile.gettempdir(), "specdec_mistral7b_q4_0_seed0.gguf")
    if rank == 0 and not os.path.exists(path):
        t = time.time()
        G.write_synthetic_gguf_parallel(path, G.MISTRAL_7B, seed=0)
        log(f"[bench] wrote synthetic model {path} in {time.time() - t:.1f}s")
    if world > 1:
        dist.barrier()
    return path


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [l.strip().split(",") for l in self.f.read().splitlines() if l.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except Exception:
                pass
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {}


def matvec_timing(rows, cols, S, n=64, copies=None, seed=7):
    """Average device time (us) of the W4A8 matvec for a rows x cols Q4_0 matrix and S activation rows,
    from CUDA events around a captured loop of n launches over rotating weight copies (> L2 in total),
    plus the algorithmic bytes of one launch (Q4_0 weights + Q8_0 activations + fp32 outputs)."""
    import torch
    from anetransformers_b200 import dequant as dq
    from anetransformers_b200.gguf import random_q4_0
    W = random_q4_0(np.random.default_rng(seed), rows, cols)
    copies = copies or max(2, int(np.ceil(400e6 / W.nbytes)))
    mats = [dq.QMat(W, device=torch.cuda.current_device()) for _ in range(copies)]
    x = torch.randn(S, cols, device="cuda")
    act = dq.quantize_dev(x)
    y = torch.empty(S, rows, device="cuda")
    for i in range(4):
        dq.matvec_dev(mats[i % copies], act, y)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(n):
            dq.matvec_dev(mats[i % copies], act, y)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / n
    alg = W.nbytes + S * (cols + cols // 32 * 8) + S * rows * 4
    del g, mats
    return us, alg


def gemv_roofline(peaks, rows=28672, cols=4096, S=SPEC_K + 1):
    """The stand-alone W4A8 matvec k_gemv (default: the fused gate|up shape, 28672 x 4096 Q4_0, 66 MB, at the
    verify width S = K+1 = 5), timed live with CUDA events (matvec_timing).  The default decode path runs the
    same tile math inside k_forward and never launches k_gemv; this entry is config 1's kernel."""
    us, alg = matvec_timing(rows, cols, S)
    achieved = alg / (us * 1e-6) / 1e9
    peak = peaks.get("hbm_gbs", 6650.0)
    return {"bound": "hbm", "kernel": f"k_gemv<EPI_STORE> {rows}x{cols} Q4_0, S={S}", "achieved": round(achieved, 1),
            "peak": peak, "peak_source": "measured" if "hbm_gbs" in peaks else "fallback", "unit": "GB/s",
            "frac": round(achieved / peak, 4), "us_per_launch": round(us, 2), "algorithmic_bytes": alg}


def config1_numbers(peaks):
    """the 4096 x 4096 W4A8 matvec at S = 1 and S = 5 (GB/s of algorithmic bytes and the
    fraction of the measured HBM copy peak), on rotating weight copies (> L2)."""
    peak = peaks.get("hbm_gbs", 6650.0)
    out = {}
    for S in (1, 5):
        us, alg = matvec_timing(4096, 4096, S)
        gbs = alg / (us * 1e-6) / 1e9
        out[f"S{S}"] = {"us_per_launch": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                        "algorithmic_bytes": alg}
    return out


def profile_traffic(name: str):
    """traffic_bytes_per_full_forward from a committed ncu summary (the capture itself is too large to take
    on the full workload; the summary states how its figure was scaled)."""
    try:
        for line in open(os.path.join(ROOT, "profiles", name)):
            if line.startswith("traffic_bytes_per_full_forward:"):
                return int(line.split(":")[1])
    except Exception:
        pass
    return None


def forward_roofline(ctx, peaks, world: int, tp: bool, S: int = SPEC_K + 1, pos: int = PROMPT_LEN + GEN_TOKENS // 2,
                     n: int = 20):
    """The dominant kernel of the timed path, k_forward (one persistent kernel per verify forward; 99.5 % of the
    decode step's launch time): n stream-ordered verify forwards of S tokens at the decode step's middle context,
    timed with CUDA events on the context's stream.  Each forward also runs the control-block upload, the
    sync-word memset and the 32-thread argmax-key decode (< 1 % of its time).  Algorithmic bytes per forward:
    this rank's Q4_0 weights (32 layers / tp ranks + the replicated LM head) + the fp16 K/V it attends."""
    import torch
    pos = min(pos, ctx.info.max_seq - S - 1)  # a shorter run (--tokens) has a shorter ring
    toks = torch.tensor(np.random.default_rng(9).integers(3, 32000, S), dtype=torch.int32, device="cuda")
    am = torch.empty(S, dtype=torch.int32, device="cuda")
    for _ in range(3):
        ctx.forward_dev(toks, pos, argmax_dev=am)
    stream = torch.cuda.ExternalStream(ctx.stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        ctx.forward_dev(toks, pos, argmax_dev=am)
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / n
    ranks = world if tp else 1
    wbytes = (BYTES_PER_FORWARD - 73_728_000) // ranks + 73_728_000
    kvbytes = KV_BYTES_PER_POS * (pos + S) // ranks
    alg = wbytes + kvbytes
    achieved = alg / (us * 1e-6) / 1e9
    peak = peaks.get("hbm_gbs", 6650.0)
    traffic = profile_traffic("forward_4layer_s5.md") if ranks == 1 else None
    return {"bound": "hbm", "kernel": f"k_forward (persistent verify forward, S={S}, context {pos + S})",
            "achieved": round(achieved, 1), "peak": peak,
            "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if "hbm_gbs" in peaks else "fallback",
            "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
            "traffic_source": "profiles/forward_4layer_s5.md: ncu dram bytes of a 4-layer capture, scaled to 32 "
                              "layers by the layer count" if traffic else None,
            "us_per_launch": round(us, 2), "algorithmic_bytes": alg}


def cpu_decode_sample(path: str, n_tokens: int, threads: int):
    """Time single-token forwards of the oracle (the reference's CPU W4A8 SDOT decode, restated in C)
    on the host cores.  The reference's CPU speculative loop verifies with sequential single-token
    forwards (speculative.h:92-101), so its speculative tok/s is bounded by this decode rate."""
    from anetransformers_b200 import gguf as G
    from oracle import oracle as O
    O.build()
    O.set_threads(threads)
    g = G.GGUFFile(path)
    om = O.OracleModel(g, max_seq=64)
    kv = om.new_kv()
    toks = config3_prompt()[:n_tokens + 2]
    om.forward(kv, toks[0], 0)                      # warm the page cache / thread pool
    t = time.perf_counter()
    for i in range(1, n_tokens + 1):
        om.forward(kv, toks[i], i)
    dt = time.perf_counter() - t
    om.free_kv(kv)
    return n_tokens / dt, dt


def run_reference(args, rank, world, dist):
    if rank != 0:
        return
    path = model_path(rank, 1, None)
    threads = os.cpu_count() or 1
    per_step = 2
    vals = []
    for i in range(args.warmup + args.steps):
        tps, dt = cpu_decode_sample(path, per_step, threads)
        if i >= args.warmup:
            vals.append(dt)
    tok = per_step * len(vals)
    value = tok / sum(vals)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * sum(vals) / len(vals), 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int4 -> int32, fp32",
            "data": "synthetic (seeded random-init Q4_0 Mistral-7B, config 3 prompt tokens)",
            "config": {"workload": "config 3 (n-gram spec decode, K=4, n=3, temp 0) on the CPU: greedy W4A8 "
                                   "decode rate, the upper bound of the reference's sequential-verify loop",
                       "model": "Mistral-7B-v0.2 arch, random Q4_0", "parallelism": "cpu threads"},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{per_step} single-token forwards per step, 7B model, all host threads"},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_gemv(args):
    """single-op W4A8 matvec (Q4_0 4096 x 4096 by default, Q8_0 activations), S = 1 and
    S = 5, in HBM GB/s of algorithmic bytes.  --shape / --S select other shapes (profiling runs)."""
    import torch
    rows, cols = (int(v) for v in args.shape.split("x"))
    peaks = measured_peaks()
    out = {}
    for S in ([args.S] if args.S else [1, 5]):
        us, alg = matvec_timing(rows, cols, S, n=args.steps * 8)
        out[f"S{S}"] = {"us_per_launch": round(us, 3), "gbs": round(alg / (us * 1e-6) / 1e9, 1)}
    best = max(v["gbs"] for v in out.values())
    print(json.dumps({"metric": "W4A8 GEMV HBM GB/s", "value": best, "unit": "GB/s", "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                      "config": {"workload": f"BASELINE config 1: Q4_0 {rows}x{cols} x Q8_0, rotating weight copies > L2"},
                      "per_S": out, "peak": peaks.get("hbm_gbs"),
                      "frac": round(best / peaks.get("hbm_gbs", 6650.0), 4)}), flush=True)


def run_greedy(args, ctx, rank, world, local, dist, tp, peaks):
    """plain greedy decode, no speculation: a 128-token prompt of uniform-random token ids
    (prefilled once, outside the timed region), then 256 greedy tokens per step through sd_decode, one S = 1
    forward per token.  A step = one 256-token decode from the prefilled prompt."""
    import torch
    rng = np.random.default_rng(128)
    prompt = rng.integers(3, 32000, GREEDY_PROMPT).tolist()
    first, _ = ctx.generate(prompt, mode="greedy", max_tokens=1, temp=0.0, rep_penalty=1.0, ignore_eos=True)
    hist = prompt + [first[0]]
    kw = dict(mode="greedy", max_tokens=args.tokens, temp=0.0, rep_penalty=1.0, ignore_eos=True)
    for _ in range(args.warmup):
        ctx.decode(hist, first[0], **kw)
    stream = torch.cuda.ExternalStream(ctx.stream)
    clocks = ClockSampler(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    tokens = 0
    for _ in range(args.steps):
        out, _ = ctx.decode(hist, first[0], **kw)
        tokens += len(out)
    e1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms_max, tokens_all = aggregate_ranks(dist, ms, tokens, tp)
    value = tokens_all / (ms_max * 1e-3)
    # one S = 1 forward per token: this rank's weights + the K/V it attends (middle of the decode)
    ranks = world if tp else 1
    fwd_b = ((BYTES_PER_FORWARD - 73_728_000) // ranks + 73_728_000 +
             KV_BYTES_PER_POS // ranks * (GREEDY_PROMPT + args.tokens // 2))
    fwd_per_s = (tokens / args.steps) / (ms / args.steps * 1e-3)
    step_roof = {"bytes_per_forward": fwd_b, "forwards_per_s": round(fwd_per_s, 2),
                 "achieved_gbs": round(fwd_b * fwd_per_s / 1e9, 1)}
    step_roof["frac_of_hbm"] = round(step_roof["achieved_gbs"] / peaks.get("hbm_gbs", 6650.0), 4)
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True,
                "scaling": "strong" if tp else "weak", "vs_baseline": round(value / GREEDY_PUBLISHED, 2),
                "vs_baseline_ref": f"{GREEDY_PUBLISHED} tok/s: the reference's published non-speculative decode of 256 "
                                   "tokens on an M5 (CPU NEON SDOT)",
                "dtype": "int8 x int4 -> int32 MMA, fp32 accumulate",
                "data": "synthetic: seeded random-init Q4_0 weights of the Mistral-7B-v0.2 architecture, "
                        "uniform-random token ids",
                "config": {"workload": "BASELINE config 2: greedy decode without speculation, 128-token random "
                                       "prompt, 256 generated tokens per step",
                           "model": "Mistral-7B-v0.2 (32 x 4096, FFN 14336, 32/8 heads, vocab 32000) Q4_0",
                           "global_batch": 1 if tp else world, "seq_len": GREEDY_PROMPT + args.tokens,
                           "parallelism": ((f"tp{world} ({args.tp_allreduce} all-reduce)" if tp else f"dp{world}")
                                           if world > 1 else "single GPU"),
                           "l2": "no flush: each forward streams 4.0 GB of weights (> 126 MB L2)"},
                "step_roofline": step_roof, "clocks": clk,
                # one iteration per token: prepare + commit around the S = 1 forward
                "gpu_launches": int(tokens * kernels_per_iter(bool(ctx.info.forward_kernel),
                                                              tp and args.tp_allreduce == "peer",
                                                              tp and args.tp_allreduce == "nccl"))}
        print(json.dumps(line), flush=True)


def run_selfspec(args, ctx, rank, world, local, dist, tp, peaks):
    """self-speculative decode (K = 8 drafts through the first 8 layers and the LM head,
    a 9-token verify), KV ring pre-filled to 32768 positions of uniform-random tokens by the device
    prefill, temp 0.7 / top-k 40 / top-p 0.9 / repetition penalty 1.1, fixed seed, 256 tokens per step.
    A step = one 256-token decode from the filled ring (the prefix K/V of target and drafter stay resident)."""
    import torch
    rng = np.random.default_rng(4321)
    prompt = rng.integers(3, 32000, SELF_CTX).tolist()
    t = time.perf_counter()
    ctx.prefill(prompt[:-1], 0)
    lg, am = ctx.forward([prompt[-1]], SELF_CTX - 1, want_logits=False)
    t_prefill = time.perf_counter() - t
    first = int(am[0])
    hist = prompt + [first]
    kw = dict(mode="self", max_tokens=args.tokens, temp=0.7, top_k=40, top_p=0.9, rep_penalty=1.1,
              ignore_eos=True, spec_k=SELF_K, draft_layers=SELF_LAYERS, seed=99)
    t = time.perf_counter()
    ctx.decode(hist, first, **kw)             # warm-up 1 also fills the drafter's K/V for the prefix
    t_draft_prefill = time.perf_counter() - t
    kw["reuse_draft_kv"] = True
    for _ in range(args.warmup - 1):
        ctx.decode(hist, first, **kw)
    stream = torch.cuda.ExternalStream(ctx.stream)
    clocks = ClockSampler(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    tokens = iters = drafted = accepted = 0
    for _ in range(args.steps):
        out, st = ctx.decode(hist, first, **kw)
        tokens += len(out)
        iters += st["total_iterations"]
        drafted += st["total_draft"]
        accepted += st["total_accepted"]
    e1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms_max, tokens_all = aggregate_ranks(dist, ms, tokens, tp)
    value = tokens_all / (ms_max * 1e-3)
    # weight + KV bytes per iteration: K drafter passes (8 layers + LM head) and a 9-token verify that runs
    # as an 8-token and a 1-token forward
    layer_b = (BYTES_PER_FORWARD - 73_728_000) // 32
    draft_b = SELF_LAYERS * layer_b + 73_728_000 + SELF_LAYERS * 2 * 1024 * 2 * SELF_CTX
    verify_b = 2 * (BYTES_PER_FORWARD + KV_BYTES_PER_POS * SELF_CTX)
    it_per_s = (iters / args.steps) / (ms / args.steps * 1e-3)
    step_roof = {"bytes_per_iteration": SELF_K * draft_b + verify_b, "iterations_per_s": round(it_per_s, 2)}
    step_roof["achieved_gbs"] = round(step_roof["bytes_per_iteration"] * it_per_s / 1e9, 1)
    step_roof["frac_of_hbm"] = round(step_roof["achieved_gbs"] / peaks.get("hbm_gbs", 6650.0), 4)
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True,
                "scaling": "strong" if tp else "weak", "vs_baseline": None,
                "dtype": "int8 x int4 -> int32 MMA, fp32 accumulate",
                "data": "synthetic: seeded random-init Q4_0 weights of the Mistral-7B-v0.2 architecture, "
                        "uniform-random token ids",
                "config": {"workload": "BASELINE config 4: self-speculative decode K=8 (drafter = first 8 layers "
                                       "+ LM head), KV pre-filled to 32768 positions, temp 0.7 top-k 40 top-p 0.9 "
                                       "rep 1.1, seed 99, 256 generated tokens per step",
                           "model": "Mistral-7B-v0.2 (32 x 4096, FFN 14336, 32/8 heads, vocab 32000) Q4_0",
                           "global_batch": 1 if tp else world, "seq_len": SELF_CTX + args.tokens,
                           "parallelism": ((f"tp{world} ({args.tp_allreduce} all-reduce)" if tp else f"dp{world}")
                                           if world > 1 else "single GPU"),
                           "l2": "no flush: each forward streams >= 1 GB of weights and K/V (> 126 MB L2)"},
                "acceptance_rate": round((accepted - iters) / drafted, 4) if drafted else None,
                "tokens_per_iteration": round(tokens / max(iters, 1), 3),
                "step_roofline": step_roof, "clocks": clk,
                "setup_s": {"prefill_32k": round(t_prefill, 2), "first_decode_with_drafter_prefill": round(t_draft_prefill, 2)},
                "gpu_launches": int(iters * (SELF_K * 3 + 2 * 2 + 1 + 1 + 2))}
        print(json.dumps(line), flush=True)


# batched speculative serving, 64 streams per GPU, 4096-token random contexts, K = 4 n-gram drafts
SERVE_STREAMS, SERVE_CTX, SERVE_TOKENS = 64, 4096, 256
GEMM_MODES = {"auto": 0, "mma": 1, "tc": 2}  # sd_batch_set_gemm modes


def run_serving(args, ctx_path, rank, world, local, dist, peaks):
    """per GPU, 64 concurrent streams, each with a 4096-token uniform-random context (K/V
    prefilled by the device), n-gram drafting n=3 K=4, temp 0, 256 generated tokens per stream; every verify
    forward carries 64 x 5 = 320 tokens (M = 320 wide-token W4A8 GEMMs).  A step = one batched 256-token decode
    of all streams from the prefilled contexts.  N GPUs = N data-parallel replicas (weak scaling)."""
    import torch
    from anetransformers_b200.engine import BatchContext, Context
    B, n_ctx = args.streams, args.ctx_serve
    ctx = Context(ctx_path, device=local, max_seq=64)
    # batch width = the verify width: the GEMMs' K splits are planned for it (prefill runs in chunks of it)
    bc = BatchContext(ctx, B, max_seq=n_ctx + args.tokens + 64, width=SPEC_K + 1)
    bc.set_gemm(GEMM_MODES[args.gemm])
    rng = np.random.default_rng(2024 + rank)
    prompts = rng.integers(3, 32000, (B, n_ctx)).astype(np.int32)
    t = time.perf_counter()
    bc.prefill(prompts[:, :-1])
    lg = bc.forward(prompts[:, -1:], np.full(B, n_ctx - 1, np.int32))
    t_prefill = time.perf_counter() - t
    first = lg[:, 0].argmax(axis=1).astype(np.int32)
    hist = np.concatenate([prompts, first[:, None]], axis=1)
    kw = dict(mode="ngram", max_tokens=args.tokens, temp=0.0, rep_penalty=1.0, ignore_eos=True, spec_k=SPEC_K,
              ngram_n=NGRAM_N)
    for _ in range(args.warmup):
        bc.decode(hist, first, **kw)
    stream = torch.cuda.ExternalStream(bc.stream)
    clocks = ClockSampler(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    tokens = iters = drafted = accepted = fwds = 0
    for _ in range(args.steps):
        outs, st = bc.decode(hist, first, **kw)
        tokens += sum(len(o) for o in outs)
        iters += st["total_iterations"]
        drafted += st["total_draft"]
        accepted += st["total_accepted"]
        fwds += st["verify_forwards"]
    e1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms_max, tokens_all = aggregate_ranks(dist, ms, tokens, False)
    value = tokens_all / (ms_max * 1e-3)
    # e2e: the same decode through the public API, history from pinned host memory, tokens back to the host
    hist_pinned = torch.from_numpy(hist).pin_memory()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    e2e_tok = 0
    for _ in range(max(1, args.steps // 2)):
        outs, _ = bc.decode(hist_pinned.numpy(), first, **kw)
        e2e_tok += sum(len(o) for o in outs)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    e2e_s, e2e_tok = aggregate_ranks(dist, e2e_s, e2e_tok, False)
    e2e = {"value": round(e2e_tok / e2e_s, 2), "unit": UNIT, "h2d_bytes_per_step": int(hist.nbytes + first.nbytes),
           "d2h_bytes_per_step": int(4 * tokens / max(args.steps, 1)),
           "what": f"sd_batch_decode per step: {B} histories ({n_ctx}-token context + first token) from pinned "
                   f"host memory, {args.tokens}-token n-gram spec decode of every stream, tokens back to host; "
                   "wall clock"}
    fwd_ms = ms / max(fwds, 1)
    ctx_mid = n_ctx + args.tokens / 2
    wbytes = BYTES_PER_FORWARD
    kvbytes = B * KV_BYTES_PER_POS * ctx_mid
    M = B * (SPEC_K + 1)
    flops = 2 * M * (BYTES_PER_FORWARD / 18 * 32)  # 2 x tokens x weights (Q4_0: 32 weights per 18 bytes)
    step_roof = {"verify_forward_ms": round(fwd_ms, 3), "M": M,
                 "weight_plus_kv_bytes_per_forward": int(wbytes + kvbytes),
                 "achieved_gbs": round((wbytes + kvbytes) / (fwd_ms * 1e-3) / 1e9, 1),
                 "int8_tops": round(flops / (fwd_ms * 1e-3) / 1e12, 1),
                 "hbm_time_floor_ms": round((wbytes + kvbytes) / (peaks.get("hbm_gbs", 6650.0) * 1e6), 3)}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        tps, dt = cpu_decode_sample(ctx_path, 4, threads)
        cpu = {"value": round(tps, 4), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": "4 single-token W4A8 forwards of the 7B model (oracle restatement of the reference's CPU "
                         "SDOT decode, all host threads); the reference serves one stream per process"}
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int4 -> int32 MMA, fp32 accumulate",
                "data": "synthetic: seeded random-init Q4_0 weights of the Mistral-7B-v0.2 architecture, "
                        "uniform-random token ids",
                "config": {"workload": f"BASELINE config 5: batched serving, {B} streams per GPU, {n_ctx}-token "
                                       f"random contexts, n-gram n=3 K=4 drafts (verify M = {M}), temp 0, "
                                       f"{args.tokens} generated tokens per stream per step",
                           "model": "Mistral-7B-v0.2 (32 x 4096, FFN 14336, 32/8 heads, vocab 32000) Q4_0",
                           "global_batch": B * world, "seq_len": n_ctx + args.tokens,
                           "parallelism": f"dp{world}" if world > 1 else "single GPU",
                           "l2": "no flush: each forward streams 4.0 GB of weights and ~1 GB of K/V (> 126 MB L2)"},
                "acceptance_rate": round((accepted - iters) / drafted, 4) if drafted else None,
                "tokens_per_stream_iteration": round(tokens / max(iters, 1), 3),
                "step_roofline": step_roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
                "setup_s": {"prefill": round(t_prefill, 2)},
                # per verify iteration: prepare, embed-norm, 9 per layer, LM GEMM, argmax, commit, done count
                "gpu_launches": int(fwds * (32 * 9 + 6))}
        print(json.dumps(line), flush=True)
    bc.close()
    ctx.close()


def run_serving_forward(args):
    """One batched verify forward (T = K+1 tokens of each of --streams streams at position --ctx-serve) on a
    Mistral-7B-shaped model with --layers layers; the rings hold zeros (attention reads every position of
    the window all the same).  For per-kernel timing and ncu captures of the batched path; CUDA events around
    --steps forwards."""
    import dataclasses
    import torch
    from anetransformers_b200 import gguf as G
    from anetransformers_b200.engine import BatchContext, Context
    cfg = dataclasses.replace(G.MISTRAL_7B, n_layers=args.layers)
    path = os.path.join(tempfile.gettempdir(), f"specdec_mistral7b_{args.layers}l_q4_0_seed0.gguf")
    if args.layers == 32:
        path = os.path.join(tempfile.gettempdir(), "specdec_mistral7b_q4_0_seed0.gguf")
    if not os.path.exists(path):
        G.write_synthetic_gguf_parallel(path, cfg, seed=0)
    T = args.S or SPEC_K + 1
    ctx = Context(path, max_seq=64)
    bc = BatchContext(ctx, args.streams, max_seq=args.ctx_serve + T + 64, width=T)
    bc.set_gemm(GEMM_MODES[args.gemm])
    rng = np.random.default_rng(5)
    toks = rng.integers(3, 32000, (args.streams, T)).astype(np.int32)
    pos = np.full(args.streams, args.ctx_serve, np.int32)
    for _ in range(args.warmup):
        bc.forward(toks, pos, want_logits=False)
    stream = torch.cuda.ExternalStream(bc.stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        bc.forward(toks, pos, want_logits=False)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    wbytes = args.layers * 122_683_392
    kv = args.layers * 2 * 1024 * 2 * (args.ctx_serve + T) * args.streams
    print(json.dumps({"workload": "serving-forward", "layers": args.layers, "streams": args.streams, "T": T,
                      "ctx": args.ctx_serve, "ms_per_forward": round(ms, 3),
                      "weight_plus_kv_gbs": round((wbytes + kv) / (ms * 1e-3) / 1e9, 1)}), flush=True)
    bc.close()
    ctx.close()


def run_forward(args):
    """Single verify forwards of S tokens (default K+1 = 5) after a ctx-token prefill, on a Mistral-7B-shaped
    synthetic model with --layers layers (a few layers keep ncu captures small while every matrix keeps its
    7B shape and the weights still exceed L2).  CUDA events around --steps forwards."""
    import dataclasses
    import torch
    from anetransformers_b200 import gguf as G
    from anetransformers_b200.engine import Context
    cfg = dataclasses.replace(G.MISTRAL_7B, n_layers=args.layers)
    path = os.path.join(tempfile.gettempdir(), f"specdec_mistral7b_{args.layers}l_q4_0_seed0.gguf")
    if not os.path.exists(path):
        G.write_synthetic_gguf_parallel(path, cfg, seed=0)
    S = args.S or SPEC_K + 1
    # matvec prefill: the workload times verify forwards, and the ncu commands of profiles/ count its launches
    ctx = Context(path, max_seq=args.ctx + S * (args.steps + args.warmup) + 64, forward_kernel=args.forward_kernel,
                  prefill_gemm=False)
    rng = np.random.default_rng(5)
    ctx.prefill(rng.integers(3, 32000, args.ctx).tolist(), 0)
    pos = args.ctx
    toks = torch.tensor(rng.integers(3, 32000, S), dtype=torch.int32, device="cuda")
    for _ in range(args.warmup):
        ctx.forward_dev(toks, pos)
        pos += S
    stream = torch.cuda.ExternalStream(ctx.stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        ctx.forward_dev(toks, pos)   # stream-ordered, no host synchronisation between forwards
        pos += S
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    wbytes = args.layers * 122_683_392 + 73_728_000
    kv = args.layers * 2 * 1024 * 2 * (args.ctx + S)
    print(json.dumps({"workload": "forward", "layers": args.layers, "S": S, "ctx": args.ctx,
                      "forward_kernel": ctx.info.forward_kernel, "us_per_forward": round(us, 2),
                      "weight_plus_kv_gbs": round((wbytes + kv) / (us * 1e-6) / 1e9, 1)}), flush=True)
    ctx.close()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--tokens", type=int, default=None, help="generated tokens per step (default: the config's)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="specdec",
                    choices=["specdec", "greedy", "selfspec", "gemv", "forward", "serving", "serving-forward"],
                    help="specdec = BASELINE config 3 (the default line), greedy = config 2, selfspec = config 4, "
                         "gemv = config 1, "
                         "serving = config 5 (batched streams), forward = single verify forwards (profiling: "
                         "--layers, --S, --ctx)")
    ap.add_argument("--streams", type=int, default=SERVE_STREAMS, help="serving: streams per GPU")
    ap.add_argument("--gemm", default="auto", choices=sorted(GEMM_MODES),
                    help="serving: batched GEMM (auto = tcgen05 from 64 tokens per forward, mma = mma.sync, tc = tcgen05)")
    ap.add_argument("--ctx-serve", type=int, default=SERVE_CTX, help="serving: context tokens per stream")
    ap.add_argument("--layers", type=int, default=32, help="forward workload: layers of the 7B-shaped model")
    ap.add_argument("--ctx", type=int, default=1024, help="forward workload: context positions before the forward")
    ap.add_argument("--forward-kernel", type=int, default=None, choices=[0, 1],
                    help="1 = one persistent kernel per forward, 0 = one kernel per op (default: library default)")
    ap.add_argument("--parallel", default=None, choices=["tp", "dp"],
                    help="with --gpus > 1: tp = one stream tensor-parallel over the GPUs (BASELINE configs 3 and 4, "
                         "the default for specdec / selfspec, strong scaling), dp = one independent stream per GPU "
                         "(aggregate tok/s, weak scaling; serving is always dp: config 5's 8 replicas)")
    ap.add_argument("--tp-allreduce", default="peer", choices=["peer", "nccl"],
                    help="tp: all-reduce inside the norm kernels over peer memory, or by NCCL")
    ap.add_argument("--shape", default="4096x4096")
    ap.add_argument("--S", type=int, default=0)
    args = ap.parse_args()
    if args.parallel is None:
        args.parallel = "dp" if args.workload == "serving" else "tp"
    if args.tokens is None:
        args.tokens = {"selfspec": SELF_TOKENS, "serving": SERVE_TOKENS, "greedy": GREEDY_TOKENS}.get(args.workload,
                                                                                                    GEN_TOKENS)
    if args.workload == "gemv":
        run_gemv(args)
        return
    if args.workload == "forward":
        run_forward(args)
        return
    if args.workload == "serving-forward":
        run_serving_forward(args)
        return
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    import torch
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    if args.impl == "reference":
        run_reference(args, rank, world, dist)
        if dist:
            dist.destroy_process_group()
        return

    from anetransformers_b200.engine import Context, NcclComm, nccl_unique_id, NCCL_ID_BYTES
    torch.cuda.set_device(local)
    path = model_path(rank, world, dist)
    peaks = measured_peaks()
    if args.workload == "serving":
        run_serving(args, path, rank, world, local, dist, peaks)
        if dist:
            dist.destroy_process_group()
        return
    tp = world > 1 and args.parallel == "tp"
    comm = None
    if tp:
        # one NCCL communicator for the model's all-reduces, from an id rank 0 creates
        uid = torch.zeros(NCCL_ID_BYTES, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        comm = NcclComm(bytes(uid.cpu().numpy().tobytes()), world, rank, local)
    n_ctx = SELF_CTX if args.workload == "selfspec" else GREEDY_PROMPT if args.workload == "greedy" else PROMPT_LEN
    ctx = Context(path, device=local, max_seq=n_ctx + args.tokens + 64, forward_kernel=args.forward_kernel,
                  tp_rank=rank if tp else 0, tp_size=world if tp else 1, nccl_comm=comm.handle if comm else 0)
    if tp and args.tp_allreduce == "peer":
        # all-reduces inside the norm kernels over NVLink (peer memory) instead of NCCL
        handles = [None] * world
        dist.all_gather_object(handles, ctx.tp_handle())
        ctx.tp_connect(handles)
    if args.workload in ("selfspec", "greedy"):
        (run_selfspec if args.workload == "selfspec" else run_greedy)(args, ctx, rank, world, local, dist, tp, peaks)
        ctx.close()
        if comm:
            comm.close()
        if dist:
            dist.destroy_process_group()
        return
    prompt = config3_prompt()
    first, _ = ctx.generate(prompt, mode="greedy", max_tokens=1, temp=0.0, rep_penalty=1.0, ignore_eos=True)
    hist = prompt + [first[0]]
    kw = dict(mode="ngram", max_tokens=args.tokens, temp=0.0, rep_penalty=1.0, ignore_eos=True, spec_k=SPEC_K,
              ngram_n=NGRAM_N)
    for _ in range(args.warmup):
        ctx.decode(hist, first[0], **kw)
    stream = torch.cuda.ExternalStream(ctx.stream)
    clocks = ClockSampler(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    tokens = 0
    iters = 0
    stats = None
    for _ in range(args.steps):
        out, stats = ctx.decode(hist, first[0], **kw)
        tokens += len(out)
        iters += stats["total_iterations"]
    e1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    # tp: every rank emits the same single stream; dp: the streams add up
    ms_max, tokens_all = aggregate_ranks(dist, ms, tokens, tp)
    value = tokens_all / (ms_max * 1e-3)
    per_rank_tps = tokens / (ms * 1e-3)
    fwd_per_s = (iters / args.steps) / (ms / args.steps * 1e-3)
    ctx_len = PROMPT_LEN + args.tokens / 2
    step_roof = {"bytes_per_forward": BYTES_PER_FORWARD + int(KV_BYTES_PER_POS * ctx_len),
                 "forwards_per_s": round(fwd_per_s, 2)}
    step_roof["achieved_gbs"] = round(step_roof["bytes_per_forward"] * fwd_per_s / 1e9, 1)
    step_roof["frac_of_hbm"] = round(step_roof["achieved_gbs"] / peaks.get("hbm_gbs", 6650.0), 4)

    # e2e: the same step through the public API with host buffers -- the history (prompt + first token) is
    # copied from pinned host memory to the device and the generated tokens come back to the host, every
    # step, inside the timed region (wall clock)
    hist_pinned = torch.tensor(hist, dtype=torch.int32).pin_memory()
    e2e_steps = max(2, args.steps // 2)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    e2e_tok = 0
    for _ in range(e2e_steps):
        out, _ = ctx.decode(hist_pinned.numpy(), first[0], **kw)
        e2e_tok += len(out)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    e2e_s, e2e_tok = aggregate_ranks(dist, e2e_s, e2e_tok, tp)
    e2e = {"value": round(e2e_tok / e2e_s, 2), "unit": UNIT, "h2d_bytes_per_step": 4 * len(hist),
           "d2h_bytes_per_step": 4 * len(out),
           "what": "sd_decode per step: history (1024-token prompt + first token) from pinned host memory, "
                   "512-token n-gram spec decode, tokens back to host; wall clock"}
    # a whole request (host prompt in, prefill + first token + decode, tokens out) for reference
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out, _ = ctx.generate(prompt, **kw)
    torch.cuda.synchronize()
    req_s = time.perf_counter() - t0
    e2e_request = {"value": round(len(out) / req_s, 2), "unit": UNIT, "ms_per_request": round(1e3 * req_s, 2),
                   "what": "sd_generate: 1024-token prompt from host, prefill " +
                           ("in 8-token W4A8 forwards (tensor parallel)" if tp and world > 1 else
                            "of the first 1016 tokens through the batched tensor-core GEMMs (64 slices of 8 tokens per "
                            "forward) and of the last 8 in one W4A8 forward") +
                           ", first token, 512-token decode, tokens to host"}
    roof = forward_roofline(ctx, peaks, world, tp)
    roof_gemv = gemv_roofline(peaks) if rank == 0 else None
    cfg1 = config1_numbers(peaks) if rank == 0 else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        tps, dt = cpu_decode_sample(path, 6, threads)
        cpu = {"value": round(tps, 4), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": "6 single-token W4A8 forwards of the 7B model (oracle restatement of the reference's "
                         "CPU SDOT decode, all host threads); the reference's CPU speculative loop verifies with "
                         "sequential single-token forwards, so this rate bounds its spec-decode tok/s"}
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True,
                "scaling": "strong" if tp else "weak", "vs_baseline": None,
                "dtype": "int8 x int4 -> int32 MMA, fp32 accumulate",
                "data": "synthetic: seeded random-init Q4_0 weights of the Mistral-7B-v0.2 architecture, "
                        "seeded random token ids",
                "config": {"workload": "BASELINE config 3: n-gram spec decode n=3 K=4, temp 0, 1024-token prompt "
                                       "(16 of 6 random 64-token segments), 512 generated tokens per step",
                           "model": "Mistral-7B-v0.2 (32 x 4096, FFN 14336, 32/8 heads, vocab 32000) Q4_0",
                           "global_batch": 1 if tp else world, "seq_len": PROMPT_LEN + args.tokens,
                           "parallelism": ((f"tp{world} ({args.tp_allreduce} all-reduce)" if tp else f"dp{world}")
                                           if world > 1 else "single GPU"),
                           "l2": "no flush: each forward streams 4.0 GB of weights (> 126 MB L2)"},
                "per_rank_tok_s": round(per_rank_tps, 2),
                "acceptance_rate": round(stats["acceptance_rate"], 4) if stats else None,
                "tokens_per_iteration": round(tokens / max(iters, 1), 3),
                "step_roofline": step_roof,
                "roofline": roof, "roofline_gemv": roof_gemv, "config1_gemv": cfg1, "cpu_baseline": cpu, "e2e": e2e, "e2e_request": e2e_request, "clocks": clk,
                "gpu_launches": int(iters * kernels_per_iter(bool(ctx.info.forward_kernel), tp and args.tp_allreduce == "peer",
                                                             tp and args.tp_allreduce == "nccl"))}
        print(json.dumps(line), flush=True)
    ctx.close()  # releases the forward graphs (they hold NCCL calls) before the communicator
    if comm:
        comm.close()
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
