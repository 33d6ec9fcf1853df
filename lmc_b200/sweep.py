"""GEMV / GEMM sweep over formats, shapes and batch widths:

    python -m lmc_b200.sweep                # the format sweep workload
    python -m lmc_b200.sweep --types Q4_K Q6_K --shapes 3072x768 --batches 1 64

Each case is timed like lmc_b200.microbench (random blocks, rotated weight
copies > 2x L2, a graph of back-to-back launches) and printed as one JSON
line with the kernel family that ran: the tensor-core GEMV on the tiled copy
(Q4_K/Q6_K/Q8_0 with cols % 256 == 0, batch <= 8), the generic CUDA-core GEMV
(other formats or shapes, batch <= 8), or the tcgen05 GEMM (batch > 8;
the fast path for the tiled formats, the generic decoders otherwise).
"""
import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from lmc_b200 import microbench as mb  # noqa: E402
from lmc_b200 import runtime as rt  # noqa: E402
from lmc_b200 import synth  # noqa: E402

TYPES = ["Q4_0", "Q5_1", "Q8_0", "Q3_K", "Q5_K", "Q6_K", "IQ4_XS"]
SHAPES = ["6400x1600", "1600x6400"]
BATCHES = [1, 8, 64, 512]


def family(qtype, cols, batch):
    tiled = qtype in (synth.Q4_K, synth.Q6_K, synth.Q8_0) and cols % 256 == 0
    if batch > 8:
        return "tcgen05 gemm (tiled fast path)" if tiled else "tcgen05 gemm (generic decoders)"
    return "tensor-core gemv (tiled)" if tiled else "generic gemv"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--types", nargs="+", default=TYPES)
    ap.add_argument("--shapes", nargs="+", default=SHAPES)
    ap.add_argument("--batches", nargs="+", type=int, default=BATCHES)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    import torch
    torch.cuda.set_device(0)
    rt.init(0)
    peak, kind = mb.hbm_peak()
    names = {v: k for k, v in synth.NAMES.items()}
    for tname in a.types:
        t = names[tname]
        for shp in a.shapes:
            rows, cols = (int(v) for v in shp.split("x"))
            for b in a.batches:
                r = mb.run(torch, t, rows, cols, b, iters=a.iters)
                print(json.dumps({"type": tname, "rows": rows, "cols": cols, "batch": b,
                                  "kernel": family(t, cols, b), "us": round(r["ms"] * 1e3, 2),
                                  "gbs": round(r["gbs"], 1), "hbm_frac": round(r["gbs"] / peak, 4),
                                  "tflops": round(2.0 * rows * cols * b / (r["ms"] * 1e-3) / 1e12, 2),
                                  "peak_kind": kind}), flush=True)


if __name__ == "__main__":
    main()
