"""Parity at the workloads' own shapes.

- Format sweep (GPT-2 XL MLP shapes 6400x1600 and 1600x6400, the seven sweep
  formats) at batch 64 and 512, where the batched tcgen05 GEMM runs: within
  rel-err 1e-3 of the dequantized weights (the oracle's bit-exact decoders)
  times x in float64.
- TinyLlama-1.1B shape (22 layers x 2048, 32 / 4 heads, SwiGLU 5632, vocab
  32000), fp32 KV: 32 greedy ids identical to LMc compiled from source
  (oracle/_ref), and with an fp16 KV cache, teacher-forced logits against
  LMc's within the fp16-cache tolerance.
- Llama-8B width (4096, 32 / 8 heads, FFN 14336, vocab 128256) with two
  layers: teacher-forced logits within 1e-3 of LMc's.
The models are random blocks of the named formats (Q4_K matrices, Q6_K
output and embedding): the same bytes per weight, written in seconds."""
import numpy as np
import pytest

from lmc_b200 import runtime as rt
from lmc_b200 import synth
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu

SWEEP = [synth.Q4_0, synth.Q5_1, synth.Q8_0, synth.Q3_K, synth.Q5_K, synth.Q6_K, synth.IQ4_XS]
TINYLLAMA = dict(L=22, D=2048, H=32, Hkv=4, F=5632, S=2048, V=32000, blocks="random", seed=7)
LLAMA8B_2L = dict(L=2, D=4096, H=32, Hkv=8, F=14336, S=256, V=128256, blocks="random", seed=8)


@pytest.mark.parametrize("t", SWEEP, ids=lambda t: synth.NAMES[t])
@pytest.mark.parametrize("shape", [(6400, 1600), (1600, 6400)], ids=lambda s: f"{s[0]}x{s[1]}")
@pytest.mark.parametrize("B", [64, 512])
def test_sweep_gemm(cuda, orc, t, shape, B):
    M, K = shape
    blk = synth.random_blocks(t, M * K, seed=M + K + t)
    w = orc.dequant(t, blk, M * K).reshape(M, K).astype(np.float64)
    x = np.random.default_rng(B + t).normal(0, 1, (B, K)).astype(np.float32)
    want = x.astype(np.float64) @ w.T
    q = rt.QTensor(t, M, K, blk)
    y = cuda.empty((B, M), dtype=cuda.float32, device="cuda")
    q.matmul(cuda.from_numpy(x).cuda(), y, batch=B)
    assert rel_err(y.cpu().numpy(), want) < 1e-3
    assert rt.lib().lmc_device_status() == 0


def _ref_model(path):
    from oracle import Ref
    ref = Ref()
    ref.set_threads(0)
    ref.load(path)
    return ref


def test_tinyllama_greedy_32_vs_lmc(cuda, model_dir):
    path = synth.cached_model("llama", model_dir, **TINYLLAMA)
    prompt = np.random.default_rng(0).integers(0, TINYLLAMA["V"], 8).astype(np.int32)
    ref = _ref_model(path)
    want, _, _ = ref.generate(prompt, 32)
    m = rt.Model(path, max_batch=1)
    got = m.generate(prompt[None], 32)
    assert got[0].tolist() == want.tolist()
    m.close()


def test_tinyllama_fp16_kv_logits_vs_lmc(cuda, model_dir):
    path = synth.cached_model("llama", model_dir, **TINYLLAMA)
    toks = np.random.default_rng(1).integers(0, TINYLLAMA["V"], 6)
    ref = _ref_model(path)
    m = rt.Model(path, max_batch=1, kv_dtype=rt.KV_F16)
    for pos, t in enumerate(toks):
        want = ref.forward(int(t), pos)
        got, _ = m.forward([int(t)], [pos])
        assert rel_err(got[0], want) < 5e-3
    m.close()


def test_llama8b_width_logits_vs_lmc(cuda, model_dir):
    path = synth.cached_model("llama", model_dir, **LLAMA8B_2L)
    toks = np.random.default_rng(2).integers(0, LLAMA8B_2L["V"], 4)
    ref = _ref_model(path)
    m = rt.Model(path, max_batch=1)
    for pos, t in enumerate(toks):
        want = ref.forward(int(t), pos)
        got, nxt = m.forward([int(t)], [pos])
        assert rel_err(got[0], want) < 1e-3
        assert nxt[0] == int(np.argmax(got[0]))
    m.close()
