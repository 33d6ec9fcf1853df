"""Regenerate the golden fixtures in tests/golden/ from LMc's own compiled
sources (oracle/_ref, built from source by oracle/Makefile).

LMc ships no test vectors, so these fixtures are LMc's outputs on seeded
synthetic inputs: every block format's dequant, one matmul_vec, the small
ops, and the logits / greedy ids of two tiny models.  The tests compare the
oracle (and through it the CUDA path) against them.

    python tests/golden/make_golden.py
"""
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from lmc_b200 import synth  # noqa: E402
from oracle import Ref  # noqa: E402


def main():
    ref = Ref()
    out = {}
    for t in synth.ALL_TYPES:
        be = max(synth.GEOMETRY[t][0], 8)
        n = be * (4 if be == 256 else 16)
        blk = synth.random_blocks(t, n, seed=1000 + t)
        out[f"dq_{synth.NAMES[t]}_blocks"] = blk
        out[f"dq_{synth.NAMES[t]}_out"] = ref.dequant(t, blk, n)
    rng = np.random.default_rng(7)
    M, K = 48, 512
    blk = synth.random_blocks(synth.Q4_K, M * K, seed=77)
    x = rng.normal(0, 1, K).astype(np.float32)
    b = rng.normal(0, 1, M).astype(np.float32)
    w = ref.dequant(synth.Q4_K, blk, M * K).reshape(M, K)
    out.update(gemv_blocks=blk, gemv_x=x, gemv_bias=b, gemv_y=ref.matmul_vec(w, x, b))
    v = rng.normal(0, 2, 768).astype(np.float32)
    lw = rng.normal(1, 0.1, 768).astype(np.float32)
    lb = rng.normal(0, 0.1, 768).astype(np.float32)
    out.update(ops_x=v, ops_w=lw, ops_b=lb, ops_layer_norm=ref.layer_norm(v, lw, lb),
               ops_rms_norm=ref.rms_norm(v, lw, 1e-5), ops_softmax=ref.softmax(v))
    out["ops_gelu"] = np.array([ref.lib.gelu(float(a)) for a in v[:64]], np.float32)
    out["ops_silu"] = np.array([ref.lib.silu(float(a)) for a in v[:64]], np.float32)
    np.savez_compressed(os.path.join(HERE, "kernels.npz"), **out)

    # tiny models: GGUF bytes + teacher-forced logits + greedy ids
    for kind, kw in (("gpt2", dict(L=1, D=64, H=2, S=32, V=96, seed=11)),
                     ("llama", dict(L=1, D=64, H=4, Hkv=2, F=128, S=32, V=96, seed=11))):
        with tempfile.TemporaryDirectory() as d:
            p = os.path.join(d, "m.gguf")
            (synth.make_gpt2 if kind == "gpt2" else synth.make_llama)(p, **kw)
            raw = np.frombuffer(open(p, "rb").read(), np.uint8)
            r = Ref()  # LMc keeps one model per process in globals; reload
            r.load(p)
            toks = [3, 90, 17, 44]
            logits = np.stack([r.forward(t, i) for i, t in enumerate(toks)])
            r.load(p)
            ids, _, _ = r.generate(np.array([5, 6, 7], np.int32), 8)
        np.savez_compressed(os.path.join(HERE, f"model_{kind}.npz"), gguf=raw, tokens=np.array(toks, np.int32),
                            logits=logits, prompt=np.array([5, 6, 7], np.int32), ids=ids)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
