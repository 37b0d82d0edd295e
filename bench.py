#!/usr/bin/env python3
"""Benchmark of the B200 token-sampling engine.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (benchmark configuration 4, the north star's target): a
batched-serving decode step over 256 rows x 151,936 bf16 logits with
heterogeneous per-row parameters (temperature, top_k 0 or 1..100, top_p,
min_p, repetition penalty) and per-row histories of 1..32,768 tokens.  A
step is one q38s_batch_sample_commit call: prepare (penalties, temperature,
top-k, min-p, top-p, seeded draw) plus commit of the decision and of the
sampled token, for all 256 rows.  Inputs rotate over distinct batches
(more than 320 MB per GPU > the 126 MB L2), so every step reads its logits
from HBM.

N > 1 (torchrun, one process per GPU): the 256 rows are split into
contiguous blocks of 256 / N rows, one per GPU, with no collective on the
data path (strong scaling: the headline value).  The line adds weak scaling
(every GPU its own 256 rows) and configuration 5 (vocab-parallel sampling:
1,024 fp32 rows split column-wise over the N GPUs, local top-64, all-gather
of the candidates, merge and draw, with each phase's time).

N = 1 adds configuration 2 (batch-1 latency), configuration 3 (speculative
verification), configuration 4 over eight parameter draws, greedy argmax and
MoE router top-k device times, and the CPU baseline.

--impl reference times the reference's own CPU implementation
(src/sampling.cc compiled unmodified into oracle/_ref/libq38ref.so, one
TransactionalSampler per row, rows spread over all host threads) on the same
workload and metric; with a GPU present its line adds the device times of
the reference's own argmax and router kernels at the same shapes.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "qwen3.8-flash-next-dual-gpu_b200")
sys.path.insert(0, PKG)

from q38s import synth  # noqa: E402

ROWS = 256
VOCAB = synth.VOCAB
ROW_BYTES_BF16 = VOCAB * 2
ROW_BYTES_F32 = VOCAB * 4
N_INPUT_BATCHES = 4
METRIC = "sampled rows/sec & HBM GB/s at 151,936 vocab; batch-1 sample latency (µs)"


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic(name: str):
    """dram bytes per launch from a committed ncu summary (profiles/*.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(name)
    except Exception:
        return None


# ------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"],
                    "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- workload
def cfg4_configs(q38s, spec):
    return [q38s.config_v2(top_k=int(spec.top_k[r]), top_p=float(spec.top_p[r]),
                           min_p=float(spec.min_p[r]), temperature=float(spec.temperature[r]),
                           repetition_penalty=float(spec.repetition_penalty[r]),
                           seed=int(spec.seed[r])) for r in range(spec.rows)]


def bf16_tensor(arr, dev):
    import torch
    return torch.from_numpy(arr.view(np.int16)).to(dev).view(torch.bfloat16)


def device_cfg4_logits(rows: int, seed: int, dev):
    """A batch with the configuration-4 row distribution generated on the
    GPU (seeded): bf16 N(0, 2.5^2) with 32 spikes per row at distinct random
    columns, the spike of Zipf rank k at 15 - 1.1 ln k."""
    import torch
    g = torch.Generator(dev).manual_seed(seed)
    x = torch.randn((rows, VOCAB), device=dev, generator=g) * 2.5
    cols = torch.rand((rows, VOCAB), device=dev, generator=g).topk(32, dim=1).indices
    ranks = torch.arange(1, 33, device=dev, dtype=torch.float32)
    x.scatter_(1, cols, (15.0 - 1.1 * torch.log(ranks)).expand(rows, 32).contiguous())
    return x.to(torch.bfloat16)


def input_batches(rows: int, seed: int, dev, min_bytes: float = 320e6):
    """Distinct input batches whose rotation exceeds the 126 MB L2 (and at
    least four)."""
    n = max(N_INPUT_BATCHES, int(np.ceil(min_bytes / (rows * ROW_BYTES_BF16))))
    return [device_cfg4_logits(rows, seed * 1000 + b, dev) for b in range(n)]


def time_steps(step_fns, steps, stream, graph_len=32):
    """Runs `steps` steps (step i calls step_fns[i % len]) as CUDA graphs of
    graph_len steps plus one graph of the remainder; returns elapsed ms
    measured with CUDA events on the launch stream.  Each graph is replayed
    once before the timed region (its first replay uploads it), so those
    replays are untimed warm-up steps."""
    import torch
    n = len(step_fns)
    g_len = max(n, (graph_len // n) * n)
    full, rest = divmod(steps, g_len)

    def capture(count):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                for i in range(count):
                    step_fns[i % n](stream)
        return g

    g = capture(g_len) if full else None
    g_rest = capture(rest) if rest else None
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for x in (g, g_rest):
            if x is not None:
                x.replay()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(full):
            g.replay()
        if g_rest is not None:
            g_rest.replay()
        t1.record(stream)
    t1.synchronize()
    ms = t0.elapsed_time(t1)
    del g, g_rest
    return ms


def run_ours(args, rank, world, dist):
    import torch
    import q38s

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    peak, peak_kind = load_peaks()

    # ---- configuration 4, strong scaling (the headline): the 256 rows of the
    # seed-4 draw split into contiguous blocks, rank r samples rows
    # [r * 256 / N, (r + 1) * 256 / N) on its own GPU; no collective.
    spec = synth.cfg4_spec(seed=4)
    configs = cfg4_configs(q38s, spec)
    lo, hi = rank * ROWS // world, (rank + 1) * ROWS // world
    rows_local = hi - lo
    inputs = input_batches(rows_local, 4 + 1000 * rank, dev)
    clocks = ClockSampler(dev.index)
    clocks.start()
    batch, decisions, ms_max, ms = cfg4_measure(q38s, configs[lo:hi], spec.histories[lo:hi],
                                                inputs, args, dev, stream, dist)
    soak_t0 = time.time()  # keep the GPU under load until a few clock samples exist
    while time.time() - soak_t0 < 1.2:
        cfg4_replay(batch, decisions, inputs, stream, 2048)
    clk = clocks.stop()
    st = batch.decode_decisions(decisions[0])
    assert (st["status"] == 0).all(), "sampler reported a row error"
    ms_per_step = ms_max / args.steps
    rows_total = ROWS
    value = rows_total / (ms_per_step / 1e3)
    algo_bytes = rows_local * ROW_BYTES_BF16
    achieved = algo_bytes / (ms / args.steps / 1e3) / 1e9

    # weak scaling, an extra key at N > 1: every rank its own 256 rows
    weak = None
    if world > 1:
        winputs = input_batches(ROWS, 7 + 1000 * rank, dev)
        wb, wd, wms_max, _ = cfg4_measure(q38s, configs, spec.histories, winputs, args, dev,
                                          stream, dist)
        weak = {"value": ROWS * world / (wms_max / args.steps / 1e3), "unit": "rows/s",
                "ms_per_step": wms_max / args.steps, "rows_per_gpu": ROWS,
                "scaling": "weak"}
        del wb, wd, winputs

    # ---- end to end: pinned host logits -> device -> sample -> host decisions
    e2e_steps = max(3, min(40, args.steps))
    pinned = [inputs[i].view(torch.int16).cpu().pin_memory() for i in range(2)]
    dev_in = torch.empty((rows_local, VOCAB), dtype=torch.int16, device=dev)
    host_dec = torch.empty(rows_local * 3, dtype=torch.int64).pin_memory()
    with torch.cuda.stream(stream):
        for _ in range(2):
            dev_in.copy_(pinned[0], non_blocking=True)
            batch.sample_commit(dev_in.view(torch.bfloat16), decisions[0], stream=stream)
            host_dec.copy_(decisions[0], non_blocking=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(e2e_steps):
            dev_in.copy_(pinned[i % 2], non_blocking=True)
            batch.sample_commit(dev_in.view(torch.bfloat16), decisions[0], stream=stream)
            host_dec.copy_(decisions[0], non_blocking=True)
            stream.synchronize()  # the step's result is read on the host
        e1.record(stream)
    e1.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if dist:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    line = {
        "metric": METRIC,
        "value": value,
        "unit": "rows/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded on the GPU: N(0,2.5^2) bf16 + Zipf(1.1)-ranked spikes, the "
                "cfg4 distribution; row parameters and histories from q38s.synth.cfg4_spec(4))",
        "config": {"workload": "cfg4 batched serving: 256 rows x 151,936 bf16 in total, "
                               "heterogeneous T/top_k/top_p/min_p/repetition, histories "
                               "U{1..32768}; step = prepare + commit + commit_token",
                   "rows_per_gpu": rows_local, "vocab": VOCAB, "global_batch": rows_total,
                   "parallelism": f"row-sharded x{world}: contiguous blocks of "
                                  f"{rows_local} rows, no collective",
                   "l2": f"inputs rotate over {len(inputs)} batches "
                         f"({len(inputs) * rows_local * ROW_BYTES_BF16 / 1e6:.0f} MB per GPU "
                         "> 126 MB L2)",
                   "timing": "CUDA graphs of 32 steps, CUDA events on the launch stream, "
                             "max over ranks"},
        "hbm_gbs": achieved,
        "e2e": {"value": rows_total / (e2e_ms / 1e3), "unit": "rows/s",
                "h2d_bytes_per_step": rows_total * ROW_BYTES_BF16,
                "d2h_bytes_per_step": rows_total * 24,
                "path": "pinned host logits -> cudaMemcpyAsync -> q38s_batch_sample_commit "
                        "-> decisions to pinned host, stream sync each step (bytes summed "
                        "over ranks)"},
        "gpu_launches": 2 * args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "frac_of_8tbs_nominal": achieved / 8000.0,
                     "traffic": load_traffic("cfg4_stream_kernel_bf16"),
                     "kernel": "stream_kernel<bf16> (one launch per step, plus the general "
                               "kernel behind it, which returns at once when no row is "
                               "deferred)",
                     "algorithmic_bytes_per_launch": algo_bytes},
        "clocks": clk,
    }
    if weak is not None:
        line["weak_scaling"] = weak

    if world == 1:
        line.update(extra_single_gpu(args, dev, stream))
        if "draws" in args.workloads:
            line["cfg4_draws"] = cfg4_draws(q38s, dev, stream)
        if "cpu" in args.workloads:
            host0 = inputs[0].view(torch.int16).cpu().numpy().view(np.uint16)
            line["cpu_baseline"] = cpu_baseline(spec, host0)
    elif "cfg5" in args.workloads:
        line["vocab_parallel"] = vocab_parallel(args, rank, world, dev, stream, dist)
    return line


def cfg4_replay(batch, decisions, inputs, stream, steps):
    fns = [lambda s, i=i: batch.sample_commit(inputs[i], decisions[i % len(decisions)], stream=s)
           for i in range(len(inputs))]
    return time_steps(fns, steps, stream)


def cfg4_measure(q38s, configs, histories, inputs, args, dev, stream, dist):
    """args.warmup + args.steps sample-commit steps of a batch over the
    rotating inputs; returns (batch, decisions, max-over-ranks ms, own ms)."""
    import torch
    batch = q38s.Batch(VOCAB, configs, device=dev.index)
    batch.commit_tokens(histories)
    decisions = [batch.decisions_buffer() for _ in range(N_INPUT_BATCHES)]
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            batch.sample_commit(inputs[i % len(inputs)], decisions[i % N_INPUT_BATCHES],
                                stream=stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ms = cfg4_replay(batch, decisions, inputs, stream, args.steps)
    torch.cuda.synchronize()
    ms_max = ms
    if dist:
        dist.barrier()
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    return batch, decisions, ms_max, ms


def cfg4_draws(q38s, dev, stream, draws=range(4, 12), steps=1024):
    """Configuration 4 over eight parameter draws (row parameters and
    histories of q38s.synth.cfg4_spec(seed)), 1,024 consecutive sample-commit
    steps each: the mean step time per draw and the slowest 32-step stretch."""
    import torch
    inputs = input_batches(ROWS, 11, dev)
    per_draw, worst = [], []
    for seed in draws:
        spec = synth.cfg4_spec(seed=seed)
        batch = q38s.Batch(VOCAB, cfg4_configs(q38s, spec), device=dev.index)
        batch.commit_tokens(spec.histories)
        decisions = [batch.decisions_buffer() for _ in range(N_INPUT_BATCHES)]
        cfg4_replay(batch, decisions, inputs, stream, 32)
        chunks = [cfg4_replay(batch, decisions, inputs, stream, 32) * 1e3 / 32
                  for _ in range(steps // 32)]
        per_draw.append(float(np.mean(chunks)))
        worst.append(float(np.max(chunks)))
        st = batch.decode_decisions(decisions[0])
        assert (st["status"] == 0).all(), f"draw {seed}: a row error"
        del batch, decisions
        torch.cuda.synchronize()
    return {"draws": list(draws), "steps_per_draw": steps,
            "us_per_step_by_draw": per_draw,
            "min_us": min(per_draw), "median_us": float(np.median(per_draw)),
            "max_us": max(per_draw), "slowest_32_step_stretch_us": max(worst)}


def extra_single_gpu(args, dev, stream):
    """Configuration 2 (batch-1 latency) and 3 (speculative verification)."""
    import torch
    import q38s

    out = {}
    if "cfg2" in args.workloads:
        out.update(batch1_latency(dev, stream))
    if "cfg3" in args.workloads:
        out.update(mtp_bench(dev, stream))
    if "kernels" in args.workloads:
        out["greedy_and_router"] = device_kernel_times("ours", dev, stream)
    return out


def device_kernel_times(impl, dev, stream, launches=500):
    """Greedy argmax (one row of 151,936 and of 248,320 bf16 logits) and the
    MoE router top-k (512 experts, top 10, normalised: 1 token, the decode
    shape, and 64 tokens), mean device time per launch in µs from CUDA events
    on the launch stream over `launches` back-to-back launches.  impl "ours"
    calls q38s_argmax_bf16 / q38s_topk_router_bf16; "reference" the
    reference's own cuda_argmax_bf16 / cuda_topk_router_bf16 (its
    cuda/q38_kernels.cu compiled unmodified into oracle/_ref)."""
    import torch
    if impl == "ours":
        import q38s
        argmax = lambda x, o: q38s.argmax_bf16(x, o, stream=stream)  # noqa: E731
        router = lambda w, i, p: q38s.topk_router_bf16(w, i, p, 10, True,  # noqa: E731
                                                       stream=stream)
    else:
        import oracle as O
        if not O.ref_kernels_available():
            return {"unavailable": "oracle/_ref/libq38ref_kernels.so not built"}
        argmax = lambda x, o: O.ref_argmax_bf16(x.data_ptr(), x.numel(),  # noqa: E731
                                                o.data_ptr(), stream.cuda_stream, dev.index)
        router = lambda w, i, p: O.ref_topk_router_bf16(  # noqa: E731
            w.data_ptr(), i.data_ptr(), p.data_ptr(), w.shape[0], w.shape[1], 10, True,
            stream.cuda_stream, dev.index)
    rng = np.random.default_rng(77)

    def timed(fn):
        with torch.cuda.stream(stream):
            for _ in range(20):
                fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(launches):
                fn()
            e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) * 1e3 / launches

    out = {"unit": "us per launch", "launches": launches}
    res = torch.zeros(1, dtype=torch.int32, device=dev)
    for n in (151_936, 248_320):
        x = bf16_tensor(synth.f32_to_bf16_rne(rng.normal(0, 2.5, n).astype(np.float32)), dev)
        out[f"argmax_{n}"] = timed(lambda: argmax(x, res))
    for tokens in (1, 64):
        w = bf16_tensor(synth.f32_to_bf16_rne(
            rng.normal(0, 1.5, (tokens, 512)).astype(np.float32)), dev)
        ids = torch.zeros((tokens, 10), dtype=torch.int32, device=dev)
        wts = torch.zeros((tokens, 10), dtype=torch.float32, device=dev)
        out[f"router_{tokens}x512_top10"] = timed(lambda: router(w, ids, wts))
    return out


def batch1_latency(dev, stream):
    """Configuration 2: batch-1 decode latency per call through the session API."""
    import torch
    import q38s

    out = {}
    c2 = synth.CFG2
    cfg = q38s.config_v2(top_k=c2["top_k"], top_p=c2["top_p"], min_p=c2["min_p"],
                         temperature=c2["temperature"], presence_penalty=c2["presence_penalty"],
                         seed=c2["seed"])
    s = q38s.Sampler(VOCAB, cfg, device=dev.index)
    s.commit_tokens(synth.cfg2_history())
    pool_n = 600  # 182 MB of distinct rows > L2
    rng = np.random.default_rng(2)
    pool = torch.empty((pool_n, VOCAB), dtype=torch.bfloat16, device=dev)
    for i in range(0, pool_n, 100):
        x = (torch.randn((100, VOCAB), device=dev, generator=torch.Generator(dev).manual_seed(i))
             * 2.5)
        idx = torch.from_numpy(rng.integers(0, VOCAB, (100, 32))).to(dev)
        x.scatter_(1, idx, torch.from_numpy(rng.uniform(8, 15, (100, 32)).astype(np.float32)).to(dev))
        pool[i:i + 100] = x.to(torch.bfloat16)
    torch.cuda.synchronize()
    n_steps = 10_000
    lat = np.empty(n_steps)
    for i in range(50):
        s.prepare_device(pool[i % pool_n])
    for i in range(n_steps):
        row = pool[i % pool_n]
        t0 = time.perf_counter_ns()
        d = s.prepare_device(row)
        lat[i] = (time.perf_counter_ns() - t0) / 1e3
        s.commit(d)
        s.commit_token(d[0])
    lat.sort()
    rank = lambda q: lat[max(0, int(np.ceil(n_steps * q / 100.0)) - 1)]  # executor.cc:126-131
    # the same loop driven from C++ through q38::TransactionalSampler (the
    # reference executor's caller), lib/libq38s_latency.so
    import ctypes as C
    native = C.CDLL(os.path.join(os.path.dirname(q38s.LIB_PATH), "libq38s_latency.so"))
    native.q38s_latency_batch1.argtypes = [C.c_uint32, C.c_void_p, C.c_void_p, C.c_size_t,
                                           C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32,
                                           C.c_void_p]
    cfg1 = q38s.config_v1(top_k=c2["top_k"], top_p=c2["top_p"], temperature=c2["temperature"],
                          presence_penalty=c2["presence_penalty"], seed=c2["seed"])
    hist = np.ascontiguousarray(synth.cfg2_history(), dtype=np.int32)
    nlat = np.empty(n_steps)
    rc = native.q38s_latency_batch1(VOCAB, C.byref(cfg1), hist.ctypes.data, hist.size,
                                    pool.data_ptr(), pool_n, 50, n_steps, nlat.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"native batch-1 latency harness failed ({rc})")
    nlat.sort()
    nrank = lambda q: nlat[max(0, int(np.ceil(n_steps * q / 100.0)) - 1)]
    # device time of the same kernels, batch of 1 row, events over 2,400
    # calls rotating through the 600 pool rows (182 MB > L2)
    b1 = q38s.Batch(VOCAB, [cfg], device=dev.index)
    b1.commit_tokens([synth.cfg2_history()])
    dec = b1.decisions_buffer()
    fns = [lambda st, i=i: b1.sample_commit(pool[i:i + 1], dec, stream=st)
           for i in range(pool_n)]
    with torch.cuda.stream(stream):
        for f in fns[:8]:
            f(stream)
    dev_ms = time_steps(fns, 4 * pool_n, stream) / (4 * pool_n)
    out["batch1"] = {"config": "cfg2: 1 row bf16, T 0.6, top_k 20, top_p 0.95, min_p 0, "
                               "presence 0.5, history 8,192 -> 18,192, 10,000 calls",
                     "p50_us": float(nrank(50)), "p99_us": float(nrank(99)),
                     "mean_us": float(nlat.mean()),
                     "call": "q38::TransactionalSampler::prepare_device from C++ (host wall "
                             "time per call, incl. launch and the wait for the 24-byte "
                             "decision, which the kernel writes into mapped host memory); "
                             "commit + commit_token between calls",
                     "python": {"p50_us": float(rank(50)), "p99_us": float(rank(99)),
                                "mean_us": float(lat.mean()),
                                "call": "q38s.Sampler.prepare_device (ctypes), same loop"},
                     "device_us": dev_ms * 1e3,
                     "device_timing": "q38s_batch_sample_commit on one row, CUDA graphs, "
                                      "rows rotating through 182 MB (> L2)",
                     "target_us": 20.0}
    return out


def mtp_bench(dev, stream):
    """Configuration 3: speculative verification, 64 drafts + bonus row, fp32."""
    import torch
    import q38s

    out = {}
    c3 = synth.CFG3
    cfg3 = q38s.config_v2(top_k=c3["top_k"], top_p=c3["top_p"], temperature=c3["temperature"],
                          seed=c3["seed"])
    b3 = q38s.Batch(VOCAB, [cfg3], device=dev.index)
    # two input sets (158 MB > L2), each with draft tokens sampled from its
    # draft distributions by the engine itself
    bq = q38s.Batch(VOCAB, [q38s.config_v2(top_k=20, top_p=0.95, temperature=0.7,
                                           seed=1000 + i) for i in range(64)], device=dev.index)
    sets = []
    for seed in (3, 4):
        tgt, drf = synth.cfg3_rows(seed=seed)
        t_t = torch.from_numpy(tgt).to(dev)
        d_t = torch.from_numpy(drf).to(dev)
        dq = bq.decode_decisions(bq.prepare(d_t[:64]))
        sets.append((t_t, d_t, torch.from_numpy(dq["token"].astype(np.int32)).to(dev)))
    res = torch.zeros(q38s.C.sizeof(q38s.MtpResult), dtype=torch.uint8, device=dev)
    fns = [lambda st, x=x: b3.mtp_verify(0, x[0], x[1][:64], x[2], result=res, stream=st)
           for x in sets]
    with torch.cuda.stream(stream):
        for _ in range(4):
            for f in fns:
                f(stream)
    torch.cuda.synchronize()
    mtp_ms = time_steps(fns, 200, stream, graph_len=8) / 200
    accepted = []
    for f in fns:
        with torch.cuda.stream(stream):
            f(stream)
        stream.synchronize()
        accepted.append(int(b3.decode_mtp(res).n_accepted))
    r = b3.decode_mtp(res)
    mtp_bytes = 129 * ROW_BYTES_F32
    out["mtp_verify"] = {"config": "cfg3: 65 target + 64 draft rows x 151,936 fp32, top_k 20, "
                                   "top_p 0.95, T 0.7",
                         "us": mtp_ms * 1e3, "accepted_by_set": accepted,
                         "published": int(r.n_tokens), "status": int(r.status),
                         "hbm_gbs": mtp_bytes / (mtp_ms / 1e3) / 1e9,
                         "algorithmic_bytes": mtp_bytes,
                         "l2": "two input sets alternate (158 MB > 126 MB L2)"}
    return out


def vocab_parallel(args, rank, world, dev, stream, dist):
    """Configuration 5: 1,024 fp32 rows of the cfg4 distribution, columns
    split over the ranks: local top-64 (q38s_shard_topk), NCCL all-gather of
    the (value, token) lists, merge and draw (q38s_shard_merge_sample) on
    every rank.  Step time (max over ranks) and each phase's CUDA-event time;
    every rank must draw the same tokens."""
    import torch
    import q38s

    rows, k = 1024, 64
    w = VOCAB // world
    col0 = rank * w
    spec = synth.cfg5_spec(rows=rows)
    configs = [q38s.config_v2(top_k=64, top_p=0.9, temperature=0.8, repetition_penalty=1.1,
                              seed=int(spec.seed[r])) for r in range(rows)]
    sb = q38s.Batch(VOCAB, configs, device=dev.index, shard=(col0, w))
    sb.commit_tokens([h[(h >= col0) & (h < col0 + w)] for h in spec.histories])
    host = np.empty((rows, w), np.float32)
    for r in range(rows):
        host[r] = synth.cfg5_row(r)[col0:col0 + w]
    shard = torch.from_numpy(host).to(dev)
    local = torch.zeros(rows * k * 2, dtype=torch.int32, device=dev)
    gathered = torch.zeros(world * rows * k * 2, dtype=torch.int32, device=dev)
    dec = sb.decisions_buffer()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    def step(timed=False):
        if timed:
            ev[0].record(stream)
        sb.shard_topk(shard, k, out=local, stream=stream)
        if timed:
            ev[1].record(stream)
        with torch.cuda.stream(stream):
            dist.all_gather_into_tensor(gathered, local)
        if timed:
            ev[2].record(stream)
        sb.shard_merge_sample(gathered, world, k, decisions=dec, stream=stream)
        if timed:
            ev[3].record(stream)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    steps = max(3, min(args.steps, 200))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    # per phase, over 20 separately timed steps
    phases = [[], [], []]
    for _ in range(20):
        step(timed=True)
        ev[3].synchronize()
        for i in range(3):
            phases[i].append(ev[i].elapsed_time(ev[i + 1]) * 1e3)
    t = torch.tensor([ms] + [float(np.median(p)) for p in phases], device=dev,
                     dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, topk_us, gather_us, merge_us = [float(x) for x in t.tolist()]
    st = sb.decode_decisions(dec)
    # the same tokens on every rank (same candidates, same seeds)
    tok = torch.from_numpy(st["token"].astype(np.int64)).to(dev)
    lo_t, hi_t = tok.clone(), tok.clone()
    dist.all_reduce(lo_t, op=dist.ReduceOp.MIN)
    dist.all_reduce(hi_t, op=dist.ReduceOp.MAX)
    identical = bool(torch.equal(lo_t, hi_t))
    return {"config": f"cfg5: 1,024 rows x 151,936 fp32 (cfg4 distribution, q38s.synth.cfg5_row), "
                      f"{world} column shards of {w}, local top-64, NCCL all-gather of "
                      "(value, token), merge, top_p 0.9",
            "rows_per_s": rows / (ms / 1e3), "ms_per_step": ms,
            "phase_us": {"shard_topk": topk_us, "all_gather": gather_us,
                         "shard_merge_sample": merge_us},
            "hbm_gbs_per_gpu": rows * w * 4 / (ms / 1e3) / 1e9,
            "row_errors": int((st["status"] != 0).sum()),
            "tokens_identical_across_ranks": identical,
            "collective": "torch.distributed all_gather_into_tensor (NCCL), launches issued "
                          "eagerly"}


PROFILE_CASES = {
    # case: (kernel the capture selects, what one launch covers)
    "general": ("general_kernel", "4 rows x 151,936 bf16 (cfg4 distribution), top_k 0, "
                "top_p 0.9, T 1.0, repetition 1.1, 2,000-token histories: every row "
                "deferred to the general kernel"),
    "cfg2": ("stream_kernel", "batch-1: 1 row x 151,936 bf16, cfg2 parameters, history "
             "8,192, split over a cluster"),
    "cfg3": ("stream_kernel", "MTP verification: 65 target + 64 draft rows x 151,936 fp32"),
    "shard_topk": ("stream_kernel", "1,024 rows x 18,992 fp32 (one of 8 column shards of "
                   "cfg5), local top-64"),
    "shard_merge": ("shard_merge_kernel", "1,024 rows, 8 shards x 64 candidates, merge, "
                    "top_p 0.9 draw"),
    "argmax": ("argmax_bf16_kernel", "greedy argmax over 248,320 bf16 logits"),
    "router": ("topk_router_kernel", "MoE router top-10 over 64 tokens x 512 experts"),
}


def profile_case(name, dev, stream, launches=4):
    """A small run of one kernel for an ncu capture (`--profile CASE`): the
    case's setup, then `launches` launches of the kernel on one GPU."""
    import torch
    import q38s
    rng = np.random.default_rng(11)

    def spiked(rows, cols):
        x = rng.normal(0, 2.5, (rows, cols)).astype(np.float32)
        for r in range(rows):
            synth.zipf_spikes(rng, x[r])
        return x

    with torch.cuda.stream(stream):
        if name == "general":
            cfgs = [q38s.config_v2(top_k=0, top_p=0.9, repetition_penalty=1.1, seed=r + 1)
                    for r in range(4)]
            b = q38s.Batch(VOCAB, cfgs, device=dev.index)
            b.commit_tokens([rng.integers(0, VOCAB, 2000).astype(np.int32) for _ in range(4)])
            x = bf16_tensor(synth.f32_to_bf16_rne(spiked(4, VOCAB)), dev)
            fn = lambda: b.prepare(x, stream=stream)  # noqa: E731
        elif name == "cfg2":
            c2 = synth.CFG2
            cfg = q38s.config_v2(top_k=c2["top_k"], top_p=c2["top_p"], min_p=c2["min_p"],
                                 temperature=c2["temperature"],
                                 presence_penalty=c2["presence_penalty"], seed=c2["seed"])
            b = q38s.Batch(VOCAB, [cfg], device=dev.index)
            b.commit_tokens([synth.cfg2_history()])
            x = bf16_tensor(synth.f32_to_bf16_rne(spiked(8, VOCAB)), dev)
            dec = b.decisions_buffer()
            it = iter(range(10 ** 9))
            fn = lambda: b.sample_commit(x[next(it) % 8:][:1], dec, stream=stream)  # noqa
        elif name == "cfg3":
            c3 = synth.CFG3
            b = q38s.Batch(VOCAB, [q38s.config_v2(top_k=c3["top_k"], top_p=c3["top_p"],
                                                  temperature=c3["temperature"],
                                                  seed=c3["seed"])], device=dev.index)
            tgt, drf = synth.cfg3_rows(seed=3)
            t_t, d_t = torch.from_numpy(tgt).to(dev), torch.from_numpy(drf).to(dev)
            toks = torch.from_numpy(rng.integers(0, VOCAB, 64).astype(np.int32)).to(dev)
            res = torch.zeros(q38s.C.sizeof(q38s.MtpResult), dtype=torch.uint8, device=dev)
            fn = lambda: b.mtp_verify(0, t_t, d_t[:64], toks, result=res, stream=stream)  # noqa
        elif name in ("shard_topk", "shard_merge"):
            rows, k, world = 1024, 64, 8
            w = VOCAB // world
            spec = synth.cfg5_spec(rows=rows)
            cfgs = [q38s.config_v2(top_k=64, top_p=0.9, temperature=0.8, repetition_penalty=1.1,
                                   seed=int(spec.seed[r])) for r in range(rows)]
            sb = q38s.Batch(VOCAB, cfgs, device=dev.index, shard=(0, w))
            sb.commit_tokens([h[h < w] for h in spec.histories])
            shard = torch.from_numpy(np.stack([synth.cfg5_row(r)[:w]
                                               for r in range(rows)])).to(dev)
            local = sb.shard_topk(shard, k, stream=stream)
            if name == "shard_topk":
                fn = lambda: sb.shard_topk(shard, k, out=local, stream=stream)  # noqa: E731
            else:
                gathered = local.repeat(world)
                dec = sb.decisions_buffer()
                fn = lambda: sb.shard_merge_sample(gathered, world, k, decisions=dec,  # noqa
                                                   stream=stream)
        elif name == "argmax":
            x = bf16_tensor(synth.f32_to_bf16_rne(spiked(1, 248_320)[0]), dev)
            out = torch.zeros(1, dtype=torch.int32, device=dev)
            fn = lambda: q38s.argmax_bf16(x, out, stream=stream)  # noqa: E731
        elif name == "router":
            w = bf16_tensor(synth.f32_to_bf16_rne(
                rng.normal(0, 1.5, (64, 512)).astype(np.float32)), dev)
            ids = torch.zeros((64, 10), dtype=torch.int32, device=dev)
            wts = torch.zeros((64, 10), dtype=torch.float32, device=dev)
            fn = lambda: q38s.topk_router_bf16(w, ids, wts, 10, True, stream=stream)  # noqa
        else:
            raise SystemExit(f"unknown profile case {name}")
        for _ in range(launches):
            fn()
    torch.cuda.synchronize()
    kernel, what = PROFILE_CASES[name]
    print(json.dumps({"profile_case": name, "kernel": kernel, "launches": launches,
                      "workload": what}), flush=True)


def cpu_baseline(spec, logits_bf16, budget_s: float = 12.0):
    """The reference's own sampler on the host cores over a bounded sample of
    the configuration-4 rows (one TransactionalSampler per row)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = os.cpu_count() or 1
    if not O.ref_available():
        return {"value": None, "unit": "rows/s", "cores": threads, "kind": "reference",
                "sample": "oracle/_ref missing"}
    samplers = []
    for r in range(spec.rows):
        c = O.make_config(top_k=int(spec.top_k[r]), top_p=float(spec.top_p[r]),
                          temperature=float(spec.temperature[r]),
                          repetition_penalty=float(spec.repetition_penalty[r]),
                          seed=int(spec.seed[r]))
        s = O.RefSampler(VOCAB, c)
        s.commit_tokens(spec.histories[r])
        samplers.append(s)
    done = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        O.ref_prepare_rows(samplers, logits_bf16, threads)
        done += spec.rows
    dt = time.perf_counter() - t0
    return {"value": done / dt, "unit": "rows/s", "cores": threads, "kind": "reference",
            "sample": f"{done} row-prepares ({done // spec.rows} passes over the 256 cfg4 rows, "
                      f"min_p ignored: sampling.cc has none) in {dt:.1f} s"}


def run_reference(args, rank, world):
    """--impl reference: src/sampling.cc (unmodified) on the host cores."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    if not O.ref_available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libq38ref.so not built"}
    spec = synth.cfg4_spec()
    logits = synth.cfg4_logits()
    samplers = []
    for r in range(spec.rows):
        c = O.make_config(top_k=int(spec.top_k[r]), top_p=float(spec.top_p[r]),
                          temperature=float(spec.temperature[r]),
                          repetition_penalty=float(spec.repetition_penalty[r]),
                          seed=int(spec.seed[r]))
        s = O.RefSampler(VOCAB, c)
        s.commit_tokens(spec.histories[r])
        samplers.append(s)
    # size each step's row sample so warmup + steps stay within ~90 s
    t0 = time.perf_counter()
    O.ref_prepare_rows(samplers, logits, threads)
    per_row = (time.perf_counter() - t0) / spec.rows
    per_step_rows = int(np.clip(90.0 / max(1, args.steps + args.warmup) / per_row, threads,
                                spec.rows))
    sub = list(range(0, spec.rows, max(1, spec.rows // per_step_rows)))[:per_step_rows]
    sub_samplers = [samplers[i] for i in sub]
    sub_logits = np.ascontiguousarray(logits[sub])
    for _ in range(args.warmup):
        O.ref_prepare_rows(sub_samplers, sub_logits, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.ref_prepare_rows(sub_samplers, sub_logits, threads)
    dt = time.perf_counter() - t0
    value = len(sub) * args.steps / dt
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg4 batched serving rows (256 x 151,936 bf16, "
                                   "heterogeneous); reference prepare() per row",
                       "rows_per_step": len(sub)},
            "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads,
                             "kind": "reference",
                             "sample": f"{len(sub)} of the 256 cfg4 rows per step, "
                                       "sampling.cc prepare() on std::threads"},
            "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    if "kernels" in args.workloads:
        import torch
        if torch.cuda.is_available():
            dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
            torch.cuda.set_device(dev)
            line["greedy_and_router"] = device_kernel_times("reference", dev,
                                                            torch.cuda.Stream(dev))
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workloads", default="cfg4,cfg2,cfg3,cfg5,draws,kernels,cpu",
                    help="comma list of the measurements to run (cfg4 always runs)")
    ap.add_argument("--profile", choices=sorted(PROFILE_CASES),
                    help="run a small case of one kernel for an ncu capture and exit")
    args = ap.parse_args()
    if args.profile:
        import torch
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        profile_case(args.profile, dev, torch.cuda.Stream(dev))
        return
    args.warmup = max(args.warmup, 3)
    args.workloads = set(args.workloads.split(","))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        dist = tdist
    try:
        line = run_ours(args, rank, world, dist)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
