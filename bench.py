#!/usr/bin/env python
"""Benchmark of the B200 hot path: GPT-2 Small decode tokens/s.

Workload (the decode configuration the headline metric is quoted on): a
GPT-2 Small-shaped model (12 layers x 768, 12 heads, vocab 50257, context
1024; attention/MLP weights Q4_K, ffn_down and output Q6_K, fp32 norms and
biases) with seeded synthetic N(0, 0.02) weights, an 8-token random prompt,
batch 1, fp32 head-major KV cache.  One step = one greedy decode token
(embedding, 12 blocks, final norm, lm_head GEMV, device argmax), replayed as
one CUDA graph.  The weights (86.7 MB) fit in the 126 MB L2, so L2 is flushed
(256 MB write) before every timed step: every step streams its weights from
HBM.

GPT-2 Small does not shard: with --gpus N each rank decodes its own replica
(weak scaling, no collective on the data path); value = all ranks' tokens /
the slowest rank's time.

--impl reference times LMc's own C sources (oracle/_ref, built from source
with its `make omp` flags) on this host's cores: rank 0 only.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_K GEMV HBM GB/s vs ~8 TB/s; GPT-2/TinyLlama decode tok/s at 1/2/4/8 GPU"
UNIT = "tokens/s"
N_PROMPT = 8
WORKLOAD = ("gpt2-small decode: 12L x 768 (12 heads), vocab 50257, ctx 1024; Q4_K attn/MLP, Q6_K ffn_down+output, "
            "fp32 norms/biases; 8-token prompt, batch 1 per GPU, greedy, fp32 KV")
L2_NOTE = "L2 flushed (256 MB write) before every timed step"


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


# DRAM bytes (read + write) of one lm_head-shape GEMV launch, from the ncu
# capture summarised in profiles/gemv_q6k_50257x768.md (same kernel and shape
# as the roofline line below).
LM_HEAD_DRAM_BYTES = 31747584


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
def cpu_reference(path, n_decode, warmup=1):
    """Greedy decode with LMc's model_forward on all host threads; returns
    (tokens/s of the decode part, threads, sample description)."""
    from oracle import Ref
    ref = Ref()
    threads = os.cpu_count() or 1
    ref.set_threads(threads)
    ref.load(path)
    p = prompt_ids()
    if warmup:
        ref.generate(p, 2)
    ids, tp, td = ref.generate(p, n_decode + 1)  # n_decode forwards after the prompt
    rate = n_decode / td
    return rate, threads, (f"LMc model_forward (oracle/_ref, make-omp flags, {os.path.basename(ref.path)}), "
                           f"{N_PROMPT}-token prompt then {n_decode} greedy decode tokens, wall clock")


def run_reference(args, rank, world):
    if rank != 0:
        return
    path = model_path(0, lambda: None)
    n_dec = max(args.steps, 8)
    from oracle import Ref  # noqa: F401  (fails loudly if the reference build is missing)
    rate, threads, sample = cpu_reference(path, n_dec, warmup=args.warmup)
    line = {"metric": METRIC, "value": round(rate, 3), "unit": UNIT, "n_gpus": world, "steps": n_dec,
            "warmup": args.warmup, "ms_per_step": round(1000.0 / rate, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "parallelism": "replicas", "global_batch": 1,
                       "seq_len": 1024, "l2": "n/a (CPU)"},
            "cpu_baseline": {"value": round(rate, 3), "unit": UNIT, "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": round(rate, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------
def run_lmc(args, rank, world, local_rank, dist):
    import torch
    from lmc_b200 import runtime as rt
    from lmc_b200 import synth

    torch.cuda.set_device(local_rank)
    rt.init(local_rank)
    barrier = (lambda: dist.barrier()) if dist else (lambda: None)
    path = model_path(rank, barrier)
    m = rt.Model(path, max_batch=1)
    p = prompt_ids()
    K, W = args.steps, args.warmup
    if N_PROMPT + W + K + 2 > m.cfg.seq_len:
        raise SystemExit(f"steps + warmup exceed the context of {m.cfg.seq_len}")
    # prefill + W warm-up decode steps; captures the step graph
    m.generate(p[None], max(W, 1), use_graph=True)
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
    launches = m.graph_kernels() * K

    # end to end: the per-token public call (model_forward drop-in) with the
    # token/position copied from host memory and the greedy id read back
    pos0 = N_PROMPT + W + K + 1
    n_e2e = min(K, m.cfg.seq_len - pos0 - 1)
    tok = np.array([int(p[0])], np.int32)
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for i in range(n_e2e):
        _, nxt = m.forward(tok, np.array([pos0 + i], np.int32), want_logits=False)
        tok = nxt
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * n_e2e / e2e_s

    from lmc_b200 import microbench
    # the dominant kernel of the step: the largest GEMV (lm_head shape)
    r = microbench.run(torch, synth.Q6_K, 50257, 768, 1, iters=60)
    gbs, gemv_ms, alg, tiled = r["gbs"], r["ms"], r["bytes"], r["tiled"]
    peak, peak_kind = measured_peaks()
    cpu = None
    if rank == 0:
        rate, threads, sample = cpu_reference(path, 16, warmup=1)
        cpu = {"value": round(rate, 3), "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample}
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K,
                "warmup": W, "ms_per_step": round(total_ms / K, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": WORKLOAD, "l2": L2_NOTE, "parallelism": f"replicas x{world}",
                           "global_batch": world, "seq_len": 1024, "prompt": N_PROMPT},
                "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4},
                "gpu_launches": launches,
                "roofline": {"bound": "hbm", "kernel": "gemv " + ("tiled tensor-core" if tiled else "generic") +
                             " Q6_K 50257x768 (lm_head shape), rotated copies > 2x L2",
                             "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(gbs / peak, 4), "peak_kind": peak_kind + " (hbm_gbs, burst)",
                             "traffic": LM_HEAD_DRAM_BYTES, "traffic_source": "profiles/gemv_q6k_50257x768.md",
                             "algorithmic_bytes": alg, "avg_launch_ms": round(gemv_ms, 5)},
                "cpu_baseline": cpu,
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    m.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["lmc", "reference"], default="lmc")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        run_reference(args, rank, world)
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
        run_lmc(args, rank, world, local_rank, dist)
    finally:
        if dist:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
