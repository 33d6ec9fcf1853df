"""Whole-model throughput on one GPU: batched prompt feed + greedy decode
through lmc_model_generate (one CUDA-graph launch per step for the whole
batch), for the model shapes of the workloads:

    python -m lmc_b200.modelbench --model tinyllama --batch 64 --prompt 512 --gen 256
    python -m lmc_b200.modelbench --model llama8b --batch 1 --prompt 1024 --gen 64
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m lmc_b200.modelbench --model llama8b --tp

With --tp (under torchrun, one process per GPU) every rank loads its
tensor-parallel shard (lmc_model_load_tp) and the times are the maximum
over the ranks.

Weights: seeded random blocks of the named formats (Q4_K matrices, Q6_K
output and token embedding), written as GGUF into --dir once.  Prompts are
uniform random ids.  The prompt is fed one position per step for all
sequences (LMc's token-by-token prefill), so a step is one forward of
`batch` tokens; batches above 8 rows run their projections on the
tcgen05 GEMM.  Prints one JSON line: prompt-feed and decode tokens/s (host
clock around synchronised runs, second of two identical runs).
"""
import argparse
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from lmc_b200 import runtime as rt  # noqa: E402
from lmc_b200 import synth  # noqa: E402

SHAPES = {
    # TinyLlama-1.1B architecture: 22 x 2048, FFN 5632, 32 / 4 heads, vocab 32000
    "tinyllama": dict(kind="llama", L=22, D=2048, H=32, Hkv=4, F=5632, S=2048, V=32000),
    # Llama-style 8B shape: 32 x 4096, FFN 14336, 32 / 8 heads, vocab 128256, ctx 4096
    "llama8b": dict(kind="llama", L=32, D=4096, H=32, Hkv=8, F=14336, S=4096, V=128256),
    # GPT-2 Small: 12 x 768, 12 heads, vocab 50257, ctx 1024
    "gpt2": dict(kind="gpt2", L=12, D=768, H=12, S=1024, V=50257),
}


def model_file(name, directory):
    kw = dict(SHAPES[name])
    kind = kw.pop("kind")
    if kind == "llama":
        kw["blocks"] = "random"
    return synth.cached_model(kind, directory, **kw)


def run(name, batch, n_prompt, n_gen, kv, directory, tp=False, prefill_rows=0):
    import torch
    dist, rank, world, dev = None, 0, 1, 0
    if tp:
        import datetime

        import torch.distributed as dist
        rank, world, dev = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
        torch.cuda.set_device(dev)
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    path = model_file(name, directory) if rank == 0 else None
    if dist:
        obj = [path]
        dist.broadcast_object_list(obj, src=0)
        path = obj[0]
    torch.cuda.set_device(dev)
    rt.init(dev)
    kvd = rt.KV_F16 if kv == "f16" else rt.KV_F32
    if dist:
        from lmc_b200 import tp as tpm
        nid = tpm.exchange_id(dist, rt.nccl_unique_id)
        m = rt.Model(path, max_batch=batch, kv_dtype=kvd, tp=(rank, world, nid), max_rows=prefill_rows or None)
    else:
        m = rt.Model(path, max_batch=batch, kv_dtype=kvd, max_rows=prefill_rows or None)
    rng = np.random.default_rng(0)
    prompts = rng.integers(0, m.cfg.vocab_size, (batch, n_prompt)).astype(np.int32)

    def timed(n_new):
        m.generate(prompts, n_new)  # captures this shape's step graph
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        m.generate(prompts, n_new)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        if dist:  # the slowest rank
            t = torch.tensor([dt])
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
        return dt

    def timed_prefill():  # every sequence's prompt, chunks of prefill_rows positions
        for rep in range(2):  # the first pass warms up (GEMM workspace, lazy module loads)
            torch.cuda.synchronize()
            if dist:
                dist.barrier()
            t0 = time.perf_counter()
            for b in range(batch):
                m.prefill(b, prompts[b], 0, want_logits=False)
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
        if dist:
            t = torch.tensor([dt])
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
        return dt

    t_prefill = timed_prefill() if prefill_rows else None
    t_feed = timed(1)        # n_prompt steps
    t_all = timed(n_gen)     # n_prompt + n_gen - 1 steps
    t_dec = max(t_all - t_feed, 1e-9)
    res = {"model": name, "batch": batch, "prompt": n_prompt, "gen": n_gen, "kv": kv,
           "prompt_tok_s": batch * n_prompt / t_feed, "decode_tok_s": batch * (n_gen - 1) / t_dec,
           "ms_per_step_prompt": 1e3 * t_feed / n_prompt, "ms_per_step_decode": 1e3 * t_dec / max(n_gen - 1, 1),
           "graph_kernels_per_step": m.graph_kernels(), "weights_bytes": os.path.getsize(path),
           "tensor_parallel": world}
    if t_prefill:
        res.update({"prefill_rows": prefill_rows, "prefill_tok_s": batch * n_prompt / t_prefill,
                    "prefill_ms": 1e3 * t_prefill})
    m.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return res if rank == 0 else None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", choices=sorted(SHAPES), default="tinyllama")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--gen", type=int, default=256)
    ap.add_argument("--kv", choices=["f16", "f32"], default="f16")
    ap.add_argument("--dir", default=os.environ.get("LMC_BENCH_DIR", "/tmp/lmc_models"))
    ap.add_argument("--tp", action="store_true", help="tensor parallel over the torchrun ranks")
    ap.add_argument("--prefill-rows", type=int, default=0,
                    help="also time batched prefill (lmc_model_prefill) in chunks of this many positions")
    a = ap.parse_args()
    r = run(a.model, a.batch, a.prompt, a.gen, a.kv, a.dir, tp=a.tp, prefill_rows=a.prefill_rows)
    if r is not None:
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
