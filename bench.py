#!/usr/bin/env python
"""Benchmark of the B200 hot path.

Default workload (the headline line): GPT-2 Small decode tokens/s.  A GPT-2
Small-shaped model (12 layers x 768, 12 heads, vocab 50257, context 1024;
attention/MLP weights Q4_K, ffn_down and output Q6_K, fp32 norms and biases)
with seeded synthetic N(0, 0.02) weights, an 8-token random prompt, batch 1,
fp32 head-major KV cache.  One step = one greedy decode token (embedding, 12
blocks, final norm, lm_head GEMV, device argmax) replayed as one CUDA graph;
on one GPU the step is one persistent kernel.  The weights (86.7 MB) fit in the
126 MB L2, so L2 is flushed (256 MB write) before every timed step, in the
device-timed loop and in the end-to-end loop alike: every step streams its
weights from HBM.  The line also carries the Q4_K 3072x768 GEMV (the other
half of the metric) with LMc's matmul_vec time on the same weights beside it.

GPT-2 Small does not shard: with --gpus N each rank decodes its own replica
(weak scaling, no collective on the data path); value = all ranks' tokens /
the slowest rank's time.  With N > 1 the line also carries "tp": the 8B
shape decoded tensor parallel over the same N ranks (batch 1 and 32; heads,
FFN rows and vocabulary sharded, two NCCL all-reduces per layer); --no-tp
skips it.

Other workloads (--workload), one JSON line each (sweep: one per case):
  gemv       one GEMV (--type/--rows/--cols/--batch; default Q4_K 3072x768 B=1)
  sweep      the format sweep: Q4_0 Q5_1 Q8_0 Q3_K Q5_K Q6_K IQ4_XS at 6400x1600
             and 1600x6400, batch 1 / 8 / 64 / 512
  tinyllama  TinyLlama-1.1B shape, --batch sequences, --prompt / --gen tokens
  llama8b    Llama-8B shape; under torchrun with --tp, tensor parallel over the ranks
Model weights for tinyllama / llama8b are random blocks of the named formats
(the same bytes per weight as quantized weights, written in seconds).

--impl reference times LMc's own C sources (oracle/_ref, built from source
with its `make omp` flags) on this host's cores: rank 0 only.
"""
import argparse
import json
import os
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_K GEMV HBM GB/s vs ~8 TB/s; GPT-2/TinyLlama decode tok/s at 1/2/4/8 GPU"
UNIT = "tokens/s"
N_PROMPT = 8
GPT2 = dict(L=12, D=768, H=12, S=1024, V=50257, F=3072)
WORKLOAD = ("gpt2-small decode: 12L x 768 (12 heads), vocab 50257, ctx 1024; Q4_K attn/MLP, Q6_K ffn_down+output, "
            "fp32 norms/biases; 8-token prompt, batch 1 per GPU, greedy, fp32 KV")
L2_NOTE = "L2 flushed (256 MB write) before every timed step (device-timed and end-to-end loops)"
CPU_REPS = 5  # repetitions of the LMc baseline; the median is reported


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def step_traffic(kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu capture of it
    (profiles/traffic.json: {kernel: {"bytes": ..., "source": ...}}), or None."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f).get(kernel)
    except (OSError, ValueError):
        return None


def model_path(rank, barrier):
    from lmc_b200 import synth
    d = os.environ.get("LMC_BENCH_CACHE", "/tmp/lmc_bench_models")
    if rank == 0:
        p = synth.cached_model("gpt2", d, seed=0)
    barrier()
    if rank != 0:
        p = synth.cached_model("gpt2", d, seed=0)
    return p


def prompt_ids():
    return np.random.default_rng(0).integers(0, 50257, N_PROMPT).astype(np.int32)


def gpt2_step_bytes(ctx_positions):
    """Algorithmic bytes of one GPT-2 Small decode step: every weight once
    (Q4_K 0.5625 B/weight, Q6_K 0.8203, fp32 norms and biases), the embedding
    row, and the fp32 K and V rows of the `ctx_positions` cached positions."""
    from lmc_b200 import synth
    g = GPT2
    D, F, L, V, S = g["D"], g["F"], g["L"], g["V"], g["S"]
    q4 = lambda r, c: synth.tensor_bytes(synth.Q4_K, r * c)
    q6 = lambda r, c: synth.tensor_bytes(synth.Q6_K, r * c)
    layer = q4(3 * D, D) + q4(D, D) + q4(F, D) + q6(D, F) + 4 * (4 * D + 3 * D + D + F + D)
    head = q6(V, D) + 4 * 2 * D
    embed = synth.tensor_bytes(synth.Q6_K, 256) * ((D + 255) // 256) + 4 * D
    kv = 2 * L * D * 4 * ctx_positions
    return L * layer + head + embed + kv


class Clocks:
    """SM clock and clock-event (throttle) reasons sampled through NVML every
    millisecond while the timed region runs (the region can be a few tens of
    milliseconds, far shorter than nvidia-smi's sampling period)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index, period_s=0.001):
        self.cuda_index, self.period = cuda_index, period_s
        self.sm, self.reasons, self.max_mhz, self.h, self.nv = [], set(), None, None, None
        self.stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            try:
                import torch
                idx = torch.cuda._get_nvml_device_index(self.cuda_index)
            except Exception:
                idx = self.cuda_index
            self.nv, self.h = nv, nv.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
        except Exception:
            self.h = None
        return self

    def _sample(self):
        nv = self.nv
        self.sm.append(float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)))
        getr = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        bits = int(getr(self.h))
        self.reasons.update(name for b, name in self.REASONS.items() if bits & b)

    def _poll(self):
        while not self.stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(self.period)

    def __exit__(self, *a):
        if self.h is not None:
            self.stop.set()
            self.t.join(timeout=2)
            if not self.sm:
                try:
                    self._sample()
                except Exception:
                    pass

    def summary(self):
        return {"sm_mhz": float(np.median(self.sm)) if self.sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.sm)}


# ---------------------------------------------------------------------------
# CPU side: LMc's own sources (oracle/_ref), timed on this host's cores
# ---------------------------------------------------------------------------
def cpu_reference(path, n_decode, reps=CPU_REPS, prompt=None):
    """Greedy decode with LMc's model_forward on all host threads: one
    untimed warm-up run, then `reps` runs of the prompt (default: the
    8-token GPT-2 prompt) and n_decode decode tokens; returns the median
    decode and prompt-feed tokens/s."""
    from oracle import Ref
    ref = Ref()
    threads = os.cpu_count() or 1
    ref.set_threads(threads)
    ref.load(path)
    p = prompt_ids() if prompt is None else np.ascontiguousarray(prompt, np.int32)
    ref.generate(p, 2)
    dec, feed = [], []
    for _ in range(reps):
        _, tp, td = ref.generate(p, n_decode + 1)  # n_decode forwards after the prompt
        dec.append(n_decode / td)
        feed.append(len(p) / tp)
    sample = (f"LMc model_forward (oracle/_ref, make-omp flags, {os.path.basename(ref.path)}), "
              f"{len(p)}-token prompt then {n_decode} greedy decode tokens, median of {reps} runs after a warm-up, "
              f"wall clock; prompt fed token by token (timed apart)")
    return float(np.median(dec)), float(np.median(feed)), threads, sample


def cpu_matmul(t, M, K, reps=20, seed=0):
    """LMc's matmul_vec on the dequantized weights of a `t` matrix M x K (the
    same seeded blocks as the GPU measurement; LMc dequantizes at load, so
    its per-token work is the fp32 product), all host threads: seconds per
    call (median of 5 timings of `reps` calls)."""
    from lmc_b200 import synth
    from oracle import Ref
    ref = Ref()
    ref.set_threads(os.cpu_count() or 1)
    blk = synth.random_blocks(t, M * K, seed=seed)
    w = ref.dequant(t, blk, M * K).reshape(M, K)
    x = np.random.default_rng(0).normal(0, 1, K).astype(np.float32)
    ref.time_matmul(w, x, max(reps // 10, 2))
    return float(np.median([ref.time_matmul(w, x, reps) / reps for _ in range(5)]))


def cpu_matmul_c1(reps=200):
    """cpu_matmul on the C1 weights (Q4_K 3072x768, seed 0)."""
    from lmc_b200 import synth
    return cpu_matmul(synth.Q4_K, 3072, 768, reps)


def run_reference(args, rank, world):
    if rank != 0:
        return
    path = model_path(0, lambda: None)
    n_dec = max(args.steps, 8)
    rate, feed, threads, sample = cpu_reference(path, n_dec)
    line = {"metric": METRIC, "value": round(rate, 3), "unit": UNIT, "n_gpus": world, "steps": n_dec,
            "warmup": args.warmup, "ms_per_step": round(1000.0 / rate, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "parallelism": "replicas", "global_batch": 1,
                       "seq_len": 1024, "l2": "n/a (CPU)"},
            "cpu_baseline": {"value": round(rate, 3), "unit": UNIT, "cores": threads, "kind": "reference",
                             "sample": sample, "prompt_feed_tok_s": round(feed, 3)},
            "e2e": {"value": round(rate, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU side: GPT-2 Small decode (the headline)
# ---------------------------------------------------------------------------
def run_gpt2(args, rank, world, local_rank, dist):
    import torch
    from lmc_b200 import microbench
    from lmc_b200 import runtime as rt
    from lmc_b200 import synth

    torch.cuda.set_device(local_rank)
    rt.init(local_rank)
    barrier = (lambda: dist.barrier()) if dist else (lambda: None)
    path = model_path(rank, barrier)
    m = rt.Model(path, max_batch=1)
    p = prompt_ids()
    K, W = args.steps, args.warmup
    if N_PROMPT + W + 2 * K + 2 > m.cfg.seq_len:
        raise SystemExit(f"steps + warmup exceed the context of {m.cfg.seq_len}")
    # prompt + W warm-up decode steps; captures the step graph
    m.generate(p[None], max(W, 1), use_graph=True)
    pos_start = N_PROMPT + max(W, 1) - 1  # position of the first timed step
    sh = m.replay(0)
    s = torch.cuda.ExternalStream(sh)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    barrier()
    torch.cuda.synchronize()
    with Clocks(local_rank) as clk:
        with torch.cuda.stream(s):
            for i in range(K):
                flush.zero_()
                evs[i][0].record(s)
                m.replay(1)
                evs[i][1].record(s)
        torch.cuda.synchronize()
    barrier()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    total_ms = float(np.sum(step_ms))
    if dist:
        t = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    value = world * K / (total_ms * 1e-3)
    kernels_per_step = m.graph_kernels()
    launches = kernels_per_step * K

    # end to end: the per-token public call (model_forward drop-in) with the
    # token/position copied from host memory and the greedy id read back;
    # L2 flushed before each call (outside the timed interval), like the
    # device-timed loop
    pos0 = pos_start + K + 1
    n_e2e = min(K, m.cfg.seq_len - pos0 - 1)
    tok = np.array([int(p[0])], np.int32)
    e2e_s = 0.0
    barrier()
    for i in range(n_e2e):
        flush.zero_()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _, nxt = m.forward(tok, np.array([pos0 + i], np.int32), want_logits=False)
        e2e_s += time.perf_counter() - t0
        tok = nxt
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * n_e2e / e2e_s

    # C1: the single Q4_K 3072x768 GEMV (rotated copies > 2x L2)
    c1 = microbench.run(torch, synth.Q4_K, 3072, 768, 1, iters=200, seed=0)
    peak, peak_kind = measured_peaks()
    cpu = None
    ref_c1 = None
    if rank == 0:
        rate, feed, threads, sample = cpu_reference(path, 32)
        cpu = {"value": round(rate, 3), "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample,
               "prompt_feed_tok_s": round(feed, 3)}
        ref_c1 = cpu_matmul_c1()
    if rank == 0:
        # the dominant kernel: the persistent step kernel (one launch per
        # token) when the step is one kernel, else the step as a whole
        ctx_mean = pos_start + (K + 1) / 2.0
        alg = gpt2_step_bytes(ctx_mean)
        step_ms_avg = total_ms / K
        gbs = alg / (step_ms_avg * 1e-3) / 1e9
        kname = "k_step" if kernels_per_step == 1 else None
        tr = step_traffic(kname) if kname else None
        traffic = traffic_src = None
        if tr:
            # the capture's context differs from this run's: only the K/V
            # reads depend on it, by the bytes one cached position adds
            per_pos = gpt2_step_bytes(1) - gpt2_step_bytes(0)
            c0 = tr.get("ctx", ctx_mean)
            traffic = int(round(tr["bytes"] + per_pos * (ctx_mean - c0)))
            traffic_src = (f"{tr['source']}; carried from {c0} to this run's {ctx_mean:.1f} cached rows by "
                           f"{per_pos} B of K/V rows per row")
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K,
                "warmup": W, "ms_per_step": round(step_ms_avg, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": WORKLOAD, "l2": L2_NOTE, "parallelism": f"replicas x{world}",
                           "global_batch": world, "seq_len": 1024, "prompt": N_PROMPT},
                "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4},
                "gpu_launches": launches,
                "roofline": {"bound": "hbm",
                             "kernel": ("persistent decode step k_step (one launch per token)" if kname else
                                        f"decode step ({kernels_per_step} launches)"),
                             "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
                             "peak_kind": peak_kind + " (hbm_gbs, burst)",
                             "traffic": traffic,
                             "traffic_source": traffic_src,
                             "algorithmic_bytes": int(alg), "avg_launch_ms": round(step_ms_avg, 5)},
                "gemv_c1": {"kernel": f"{c1['kernel']}: Q4_K 3072x768, batch 1, rotated copies > 2x L2",
                            "us": round(c1["ms"] * 1e3, 3), "gbs": round(c1["gbs"], 1),
                            "frac": round(c1["gbs"] / peak, 4), "algorithmic_bytes": c1["bytes"],
                            "reference_matmul_vec_us": round(ref_c1 * 1e6, 2) if ref_c1 else None},
                "cpu_baseline": cpu,
                "clocks": clk.summary()}
    m.close()
    if world > 1 and dist and not args.no_tp:
        # GPT-2 Small does not shard (replicas above); the 8B shape decodes
        # tensor parallel over the same ranks: batch 1 and batch 32
        tp = {"model": "llama-8b shape (32 x 4096, FFN 14336, 32/8 heads, vocab 128256), random Q4_K/Q6_K blocks",
              "tensor_parallel": world, "kv": "f16", "prompt": 16, "gen": 16}
        for B in (1, 32):
            a = argparse.Namespace(workload="llama8b", kv="f16", batch=B, prompt=16, gen=16, prefill_rows=0)
            r = model_decode(a, rank, world, local_rank, dist)
            if rank == 0:
                tp[f"batch{B}_tok_s"] = r["value"]
                tp[f"batch{B}_ms_per_step"] = r["ms_per_step_decode"]
        if rank == 0:
            line["tp"] = tp
    if rank == 0:
        print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# other workloads
# ---------------------------------------------------------------------------
SWEEP_TYPES = ["Q4_0", "Q5_1", "Q8_0", "Q3_K", "Q5_K", "Q6_K", "IQ4_XS"]
SWEEP_SHAPES = ["6400x1600", "1600x6400"]
SWEEP_BATCHES = [1, 8, 64, 512]
MODELS = {
    # TinyLlama-1.1B architecture: 22 x 2048, FFN 5632, 32 / 4 heads, vocab 32000
    "tinyllama": dict(kind="llama", L=22, D=2048, H=32, Hkv=4, F=5632, S=2048, V=32000),
    # Llama-style 8B shape: 32 x 4096, FFN 14336, 32 / 8 heads, vocab 128256, ctx 4096
    "llama8b": dict(kind="llama", L=32, D=4096, H=32, Hkv=8, F=14336, S=4096, V=128256),
}


def run_gemv(args):
    import torch
    from lmc_b200 import microbench as mb
    from lmc_b200 import runtime as rt
    from lmc_b200 import synth
    torch.cuda.set_device(0)
    rt.init(0)
    names = {v: k for k, v in synth.NAMES.items()}
    peak, kind = measured_peaks()
    cases = []
    if args.workload == "sweep":
        for tn in SWEEP_TYPES:
            for shp in SWEEP_SHAPES:
                for b in SWEEP_BATCHES:
                    cases.append((tn, shp, b))
    else:
        cases.append((args.type, f"{args.rows}x{args.cols}", args.batch))
    from oracle import ref_library_path
    have_ref = os.path.exists(ref_library_path())
    ref_s = {}  # LMc's seconds per matmul_vec call, per (type, shape)
    for tn, shp, b in cases:
        t = names[tn]
        rows, cols = (int(v) for v in shp.split("x"))
        r = mb.run(torch, t, rows, cols, b, iters=max(args.steps, 20), seed=0)
        fl = 2.0 * rows * cols * b / (r["ms"] * 1e-3) / 1e12
        line = {"metric": "GEMV/GEMM throughput", "workload": "gemv", "type": tn, "rows": rows,
                "cols": cols, "batch": b, "kernel": r["kernel"],
                "us": round(r["ms"] * 1e3, 3), "gbs": round(r["gbs"], 1),
                "hbm_frac": round(r["gbs"] / peak, 4), "tflops": round(fl, 2),
                "algorithmic_bytes": r["bytes"], "peak_kind": kind,
                "l2": "rotated weight copies > 2x L2, graph of back-to-back launches"}
        if have_ref:  # LMc has no batched product: batch b is b matmul_vec calls
            if (t, shp) not in ref_s:
                ref_s[(t, shp)] = cpu_matmul(t, rows, cols)
            line["reference_matmul_vec_us"] = round(ref_s[(t, shp)] * b * 1e6, 2)
            line["reference"] = f"LMc matmul_vec (oracle/_ref), {os.cpu_count() or 1} host threads, b calls"
        print(json.dumps(line), flush=True)


def run_model(args, rank, world, local_rank, dist):
    res = model_decode(args, rank, world, local_rank, dist)
    if rank == 0:
        print(json.dumps(res), flush=True)


def model_decode(args, rank, world, local_rank, dist):
    """Prompt feed + greedy decode through lmc_model_generate (one graph
    launch per step for the whole batch); with a process group every rank
    holds its tensor-parallel shard and the times are the maximum over the
    ranks.  Returns the result line on rank 0 (None elsewhere)."""
    import torch
    from lmc_b200 import runtime as rt
    from lmc_b200 import synth
    kw = dict(MODELS[args.workload])
    kind = kw.pop("kind")
    kw["blocks"] = "random"
    d = os.environ.get("LMC_BENCH_CACHE", "/tmp/lmc_bench_models")
    torch.cuda.set_device(local_rank)
    rt.init(local_rank)
    path = synth.cached_model(kind, d, **kw) if rank == 0 else None
    if dist:
        obj = [path]
        dist.broadcast_object_list(obj, src=0)
        path = obj[0]
    kvd = {"f16": rt.KV_F16, "f32": rt.KV_F32, "q8": rt.KV_Q8}[args.kv]
    B = args.batch
    rows = args.prefill_rows or None
    # paged cache: just the pages prompt + gen positions of every sequence take
    P = args.kv_page
    paged = dict(page_size=P, n_pages=B * -(-(args.prompt + args.gen) // P)) if P else {}
    res = None
    t_load = time.perf_counter()  # GGUF parse + weight upload (the file is in the page cache: just written)
    if dist and world > 1:
        from lmc_b200 import tp as tpm
        nid = tpm.exchange_id(dist, rt.nccl_unique_id)
        m = rt.Model(path, max_batch=B, kv_dtype=kvd, tp=(rank, world, nid), max_rows=rows, **paged)
    else:
        m = rt.Model(path, max_batch=B, kv_dtype=kvd, max_rows=rows, **paged)
    torch.cuda.synchronize()
    t_load = time.perf_counter() - t_load
    prompts = np.random.default_rng(0).integers(0, m.cfg.vocab_size, (B, args.prompt)).astype(np.int32)

    def slowest(dt):
        if dist:
            t = torch.tensor([dt], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
        return dt

    def timed(n_new):
        m.generate(prompts, n_new)  # captures this shape's step graph
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        m.generate(prompts, n_new)
        torch.cuda.synchronize()
        return slowest(time.perf_counter() - t0)

    t_prefill = None
    if rows:
        for _ in range(2):  # the first pass warms up
            torch.cuda.synchronize()
            if dist:
                dist.barrier()
            t0 = time.perf_counter()
            for b in range(B):
                m.prefill(b, prompts[b], 0, want_logits=False)
            torch.cuda.synchronize()
            t_prefill = slowest(time.perf_counter() - t0)
    t_feed = timed(1)
    t_all = timed(args.gen)
    t_dec = max(t_all - t_feed, 1e-9)
    if rank == 0:
        wbytes = os.path.getsize(path)
        dec = B * (args.gen - 1) / t_dec
        step_s = t_dec / max(args.gen - 1, 1)
        peak, kind_p = measured_peaks()
        res = {"metric": METRIC, "workload": args.workload, "value": round(dec, 2), "unit": UNIT,
               "n_gpus": world, "batch": B, "prompt": args.prompt, "gen": args.gen, "kv": args.kv,
               "prompt_feed_tok_s": round(B * args.prompt / t_feed, 2),
               "ms_per_step_decode": round(1e3 * step_s, 4),
               "graph_kernels_per_step": m.graph_kernels(), "weights_bytes": wbytes,
               "weights_hbm_frac_per_rank": round(wbytes / world / step_s / 1e9 / peak, 4),
               "tensor_parallel": world, "data": "synthetic (random blocks of the named formats)",
               "load_s": round(t_load, 3), "load_gbs": round(wbytes / max(t_load, 1e-9) / 1e9, 2),
               "timing": "host clock around synchronised generate runs (second of two)", "peak_kind": kind_p}
        if t_prefill:
            res.update({"prefill_rows": rows, "prefill_tok_s": round(B * args.prompt / t_prefill, 2)})
        if P:
            ps, npg, _ = m.kv_pages()
            res.update({"kv_page": ps, "kv_pages": npg})
    m.close()
    if res is not None and world == 1 and (args.workload == "tinyllama" or os.environ.get("LMC_BENCH_CPU_8B") == "1"):
        # LMc's model_forward on the same file, one sequence (it cannot
        # batch), a bounded sample: the first 8 prompt ids of sequence 0,
        # then 8 greedy tokens.  Its fp32 arena takes 4 bytes a weight of
        # host memory (32 GB for the 8B shape: opt in with LMC_BENCH_CPU_8B=1).
        rate, feed, threads, sample = cpu_reference(path, 8, reps=3, prompt=prompts[0][:N_PROMPT])
        res["cpu_baseline"] = {"value": round(rate, 3), "unit": UNIT, "cores": threads, "kind": "reference",
                               "sample": sample, "prompt_feed_tok_s": round(feed, 3)}
    return res if rank == 0 else None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["lmc", "reference"], default="lmc")
    ap.add_argument("--workload", choices=["gpt2", "gemv", "sweep", "tinyllama", "llama8b"], default="gpt2")
    ap.add_argument("--type", default="Q4_K")
    ap.add_argument("--rows", type=int, default=3072)
    ap.add_argument("--cols", type=int, default=768)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--gen", type=int, default=64)
    ap.add_argument("--kv", choices=["f16", "f32", "q8"], default="f16")
    ap.add_argument("--prefill-rows", type=int, default=0)
    ap.add_argument("--kv-page", type=int, default=0,
                    help="paged KV cache of this many positions per page, the pool sized to prompt + gen")
    ap.add_argument("--tp", action="store_true", help="tensor parallel over the torchrun ranks (llama8b)")
    ap.add_argument("--no-tp", action="store_true",
                    help="gpt2 on several GPUs: skip the tensor-parallel 8B line (tp sub-object)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        if args.workload == "gpt2":
            run_reference(args, rank, world)
        elif rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the gpt2 workload only"}))
        return
    if args.workload in ("gemv", "sweep") or (args.workload != "gpt2" and world > 1 and not args.tp):
        if rank == 0:  # single-GPU workloads: rank 0 alone
            if args.workload in ("gemv", "sweep"):
                run_gemv(args)
            else:
                run_model(args, 0, 1, local_rank, None)
        return
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "gpt2":
            run_gpt2(args, rank, world, local_rank, dist)
        else:
            run_model(args, rank, world, local_rank, dist if args.tp else None)
    finally:
        if dist:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
