"""GEMV microbenchmark: one quantized matrix-vector product, timed on the
device with CUDA events around a CUDA graph of back-to-back launches over
rotated weight copies whose total exceeds twice the 126 MB L2 (so every
launch streams its weights from HBM and host launch cost is excluded).

    python -m lmc_b200.microbench --type Q4_K --rows 3072 --cols 768 --batch 1
    python -m lmc_b200.microbench --attention --batch 64 --heads 32 --kv-heads 4 \
        --head-dim 64 --ctx 2048 --pos 640 --kv f16

The second form times one decode-step attention (lmc_attention_decode: split
context, separate merge kernel) over a random fp16/fp32 cache, every
sequence at position --pos; bytes are the K and V rows read (positions
0..pos of every sequence and kv head).

Prints one JSON line: average launch time, algorithmic bytes per launch
(weights + fp32 x + fp32 y, as counted in the roofline), GB/s and the
fraction of the measured HBM peak.  Weights are seeded random blocks (fp16
scales |N(0,1e-3)|, uniform codes), x ~ N(0,1).
"""
import argparse
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from lmc_b200 import runtime as rt  # noqa: E402
from lmc_b200 import synth  # noqa: E402

L2_BYTES = 126e6


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def algorithmic_bytes(qtype, rows, cols, batch):
    return synth.tensor_bytes(qtype, rows * cols) + 4 * cols * batch + 4 * rows * batch


def run(torch, qtype, rows, cols, batch=1, iters=50, stream=None, generic=False, seed=100):
    """Returns dict(ms, gbs, bytes, tiled).  The `iters` launches (round robin
    over the weight copies) are captured once as a CUDA graph and the graph
    replay is timed, so host launch overhead is not in the number."""
    wbytes = synth.tensor_bytes(qtype, rows * cols)
    copies = max(2, int(np.ceil(2.2 * L2_BYTES / wbytes)) + 1)
    qs = [rt.QTensor(qtype, rows, cols, synth.random_blocks(qtype, rows * cols, seed=seed + i)) for i in range(copies)]
    x = torch.randn(batch, cols, device="cuda")
    y = torch.empty(batch, rows, device="cuda")

    def launch(q, st):
        if generic:
            rt.call("lmc_matmul_blocks", qtype, rt.lib().lmc_qtensor_blocks(q.h), rows, cols, x.data_ptr(), cols,
                    None, y.data_ptr(), rows, batch, 0, st)
        else:
            q.matmul(x, y, batch=batch, stream=st)

    s = stream or torch.cuda.Stream()
    with torch.cuda.stream(s):
        for q in qs:
            launch(q, s.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        cs = torch.cuda.current_stream().cuda_stream
        for i in range(iters):
            launch(qs[i % copies], cs)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (reps * iters)
    alg = algorithmic_bytes(qtype, rows, cols, batch)
    tiled = qs[0].tiled and not generic
    kernel = ("generic GEMV (bit-exact decoders, CUDA cores)" if generic
              else rt.lib().lmc_matmul_kernel(qs[0].h, batch, 0).decode())
    del g
    for q in qs:
        q.close()
    return {"ms": ms, "gbs": alg / (ms * 1e-3) / 1e9, "bytes": alg, "tiled": tiled, "kernel": kernel}


def run_attention(torch, B, H, Hkv, Dh, S, pos, kv, iters=20):
    kvd = rt.KV_F16 if kv == "f16" else rt.KV_F32
    cdt = torch.float16 if kv == "f16" else torch.float32
    g = torch.Generator(device="cuda").manual_seed(0)
    kc = torch.randn(B, Hkv, S, Dh, device="cuda", generator=g).to(cdt)
    vc = torch.randn(B, Hkv, S, Dh, device="cuda", generator=g).to(cdt)
    q = torch.randn(B, H * Dh, device="cuda", generator=g)
    kn = torch.randn(B, Hkv * Dh, device="cuda", generator=g)
    vn = torch.randn(B, Hkv * Dh, device="cuda", generator=g)
    poss = torch.full((B,), pos, dtype=torch.int32, device="cuda")
    out = torch.empty(B, H * Dh, device="cuda")
    wsb = rt.lib().lmc_attention_workspace_bytes(B, H, Dh, S)
    ws = torch.empty(max(wsb, 4), dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()

    def go():
        rt.call("lmc_attention_decode", out.data_ptr(), q.data_ptr(), kn.data_ptr(), vn.data_ptr(), kc.data_ptr(),
                vc.data_ptr(), kvd, poss.data_ptr(), B, H, Hkv, Dh, S, ws.data_ptr(), wsb, s.cuda_stream)

    for _ in range(3):
        go()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(iters):
        go()
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    nbytes = B * Hkv * (pos + 1) * Dh * 2 * (2 if kv == "f16" else 4)
    return {"ms": ms, "bytes": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--attention", action="store_true", help="time the decode attention instead of a GEMV")
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=4)
    ap.add_argument("--head-dim", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--pos", type=int, default=640)
    ap.add_argument("--kv", choices=["f16", "f32"], default="f16")
    ap.add_argument("--type", default="Q4_K")
    ap.add_argument("--rows", type=int, default=3072)
    ap.add_argument("--cols", type=int, default=768)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--generic", action="store_true", help="time the generic CUDA-core kernel")
    a = ap.parse_args()
    import torch
    qtype = {v: k for k, v in synth.NAMES.items()}[a.type]
    torch.cuda.set_device(0)
    rt.init(0)
    if a.attention:
        r = run_attention(torch, a.batch, a.heads, a.kv_heads, a.head_dim, a.ctx, a.pos, a.kv, a.iters)
        peak, kind = hbm_peak()
        r.update({"kernel": "attention", "batch": a.batch, "heads": a.heads, "kv_heads": a.kv_heads,
                  "head_dim": a.head_dim, "ctx": a.ctx, "pos": a.pos, "kv": a.kv, "peak_gbs": peak,
                  "frac": r["gbs"] / peak, "peak_kind": kind})
        print(json.dumps(r), flush=True)
        return
    r = run(torch, qtype, a.rows, a.cols, a.batch, a.iters, generic=a.generic)
    peak, kind = hbm_peak()
    r.update({"type": a.type, "rows": a.rows, "cols": a.cols, "batch": a.batch, "peak_gbs": peak,
              "frac": r["gbs"] / peak, "peak_kind": kind,
              "tflops": 2.0 * a.rows * a.cols * a.batch / (r["ms"] * 1e-3) / 1e12})
    print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
