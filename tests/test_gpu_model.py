"""Whole-model decode on the device against LMc's own compiled sources
(oracle/_ref) and the C restatement: teacher-forced logits within rel-err
1e-3 and identical greedy ids."""
import os

import numpy as np
import pytest

from lmc_b200 import runtime as rt
from lmc_b200 import synth
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def tiny(kind, model_dir, **kw):
    return synth.cached_model(kind, model_dir, **kw)


@pytest.mark.parametrize("kind,kw", [
    ("gpt2", dict(L=2, D=256, H=4, S=128, V=1000, seed=1)),
    ("llama", dict(L=2, D=256, H=8, Hkv=2, F=512, S=128, V=1000, seed=1)),
])
@pytest.mark.parametrize("kvd", [rt.KV_F32, rt.KV_F16])
def test_tiny_model_logits(cuda, orc, model_dir, kind, kw, kvd):
    path = tiny(kind, model_dir, **kw)
    om = orc.model(path)
    m = rt.Model(path, max_batch=1, kv_dtype=kvd)
    toks = [5, 17, 900, 3, 999, 0, 42, 7]
    for pos, t in enumerate(toks):
        want = om.forward(t, pos)
        got, nxt = m.forward([t], [pos])
        assert rel_err(got[0], want) < (1e-3 if kvd == rt.KV_F32 else 5e-3)
        assert nxt[0] == int(np.argmax(got[0]))


@pytest.mark.parametrize("kind,kw", [
    ("gpt2", dict(L=2, D=256, H=4, S=128, V=1000, seed=2)),
    ("llama", dict(L=2, D=256, H=8, Hkv=2, F=512, S=128, V=1000, seed=2)),
])
def test_tiny_generate_matches_oracle(cuda, orc, model_dir, kind, kw):
    path = tiny(kind, model_dir, **kw)
    prompt = np.random.default_rng(0).integers(0, kw["V"], 8).astype(np.int32)
    om = orc.model(path)
    ids, lg = [], None
    for pos, t in enumerate(prompt):
        lg = om.forward(int(t), pos)
    pos = len(prompt)
    for _ in range(32):
        nxt = orc.argmax(lg)
        ids.append(nxt)
        lg = om.forward(nxt, pos)
        pos += 1
    m = rt.Model(path, max_batch=2)
    got = m.generate(np.stack([prompt, prompt]), 32, use_graph=True)
    assert got[0].tolist() == ids and got[1].tolist() == ids
    got2 = m.generate(prompt[None], 32, use_graph=False)
    assert got2[0].tolist() == ids


def test_llama_long_rows_logits(cuda, orc, model_dir):
    """A one-layer LLaMA whose Q6_K head (K = 4352, RMS prologue fused) takes
    the GEMV's register-held activation variant, and whose Q4_K down
    projection (K = 4608) takes the SwiGLU prologue with the short silu."""
    path = tiny("llama", model_dir, L=1, D=4352, H=34, Hkv=17, F=4608, S=64, V=512, seed=4)
    om = orc.model(path)
    m = rt.Model(path, max_batch=1)
    for pos, t in enumerate([3, 500, 77, 1]):
        want = om.forward(t, pos)
        got, nxt = m.forward([t], [pos])
        assert rel_err(got[0], want) < 1e-3
        assert nxt[0] == int(np.argmax(got[0]))


def test_gpt2_small_greedy_32(cuda, model_dir):
    """GPT-2 Small shape (12 x 768, V 50257, Q4_K + Q6_K): 8-token prompt,
    32 greedy ids identical to LMc's compiled model_forward."""
    from oracle import Ref
    path = tiny("gpt2", model_dir, seed=0)
    prompt = np.random.default_rng(0).integers(0, 50257, 8).astype(np.int32)
    ref = Ref()
    ref.load(path)
    want, _, _ = ref.generate(prompt, 32)
    m = rt.Model(path, max_batch=1)
    got = m.generate(prompt[None], 32)
    assert got[0].tolist() == want.tolist()


@pytest.mark.parametrize("kind,kw", [
    ("gpt2", dict(L=2, D=256, H=4, S=128, V=1000, seed=3)),
    ("llama", dict(L=2, D=256, H=8, Hkv=2, F=512, S=128, V=1000, seed=3)),
])
def test_batched_gemm_path_matches_oracle(cuda, orc, model_dir, kind, kw):
    """12 sequences per step: every projection runs on the batched tensor-core
    GEMM (fp16 weights, fp16 hi+lo activations).  Teacher-forced logits of each
    sequence within 1e-3 of the oracle, then 16 greedy ids per sequence equal
    to the oracle's."""
    B, n_new = 12, 16
    path = tiny(kind, model_dir, **kw)
    rng = np.random.default_rng(7)
    prompts = rng.integers(0, kw["V"], (B, 6)).astype(np.int32)
    m = rt.Model(path, max_batch=B)
    oms = [orc.model(path) for _ in range(B)]
    for pos in range(prompts.shape[1]):
        got, _ = m.forward(prompts[:, pos], [pos] * B)
        for b in range(B):
            want = oms[b].forward(int(prompts[b, pos]), pos)
            assert rel_err(got[b], want) < 1e-3
    want_ids = []
    for b in range(B):
        om = orc.model(path)
        lg = None
        for pos, t in enumerate(prompts[b]):
            lg = om.forward(int(t), pos)
        ids, pos = [], prompts.shape[1]
        for _ in range(n_new):
            nxt = orc.argmax(lg)
            ids.append(nxt)
            lg = om.forward(nxt, pos)
            pos += 1
        want_ids.append(ids)
    m2 = rt.Model(path, max_batch=B)
    got = m2.generate(prompts, n_new, use_graph=True)
    for b in range(B):
        assert got[b].tolist() == want_ids[b]


@pytest.mark.parametrize("kind,kw", [
    ("gpt2", dict(L=2, D=256, H=4, S=128, V=1000, seed=5)),
    ("llama", dict(L=2, D=256, H=8, Hkv=2, F=512, S=128, V=1000, seed=5)),
])
@pytest.mark.parametrize("kvd", [rt.KV_F32, rt.KV_F16, rt.KV_Q8])
def test_prefill_matches_oracle(cuda, orc, model_dir, kind, kw, kvd):
    """Batched prefill (lmc_model_prefill): a 21-token prompt of sequence 1 in
    chunks of 16 and 5 rows (the first through the tensor-core GEMM) gives
    the oracle's last-position logits and next id, and greedy decoding then
    continues with the oracle's ids from the cache the prefill wrote.  The
    oracle stores its K/V rows as the cache does (fp32, fp16, int8 rows)."""
    path = tiny(kind, model_dir, **kw)
    prompt = np.random.default_rng(3).integers(0, kw["V"], 21).astype(np.int32)
    om = orc.model(path).set_kv(kvd)
    lg = None
    for pos, t in enumerate(prompt):
        lg = om.forward(int(t), pos)
    tol = 1e-3
    m = rt.Model(path, max_batch=2, kv_dtype=kvd, max_rows=16)
    got, nxt = m.prefill(1, prompt)
    assert rel_err(got, lg) < tol
    assert nxt == orc.argmax(lg) == int(np.argmax(got))
    pos, ids, want = len(prompt), [], []
    for _ in range(8):
        want.append(orc.argmax(lg))
        lg = om.forward(want[-1], pos)
        _, n2 = m.forward([0, nxt], [0, pos])  # sequence 0 is idle (any token at position 0)
        ids.append(nxt)
        nxt = int(n2[1])
        pos += 1
    assert ids == want


@pytest.mark.parametrize("kind,kw", [
    ("gpt2", dict(L=2, D=256, H=4, S=128, V=1000, seed=6)),
    ("llama", dict(L=2, D=256, H=8, Hkv=2, F=512, S=128, V=1000, seed=6)),
])
def test_generate_with_prefill_matches_oracle(cuda, orc, model_dir, kind, kw):
    """lmc_model_generate on a model with more rows per step than sequences
    prefills the prompts in chunks and then runs the step graph from the last
    prompt position: the oracle's greedy ids for both sequences."""
    path = tiny(kind, model_dir, **kw)
    rng = np.random.default_rng(7)
    prompts = rng.integers(0, kw["V"], (2, 21)).astype(np.int32)
    want = []
    for p in prompts:
        om = orc.model(path)
        lg = None
        for pos, t in enumerate(p):
            lg = om.forward(int(t), pos)
        ids, pos = [], len(p)
        for _ in range(16):
            ids.append(orc.argmax(lg))
            lg = om.forward(ids[-1], pos)
            pos += 1
        want.append(ids)
    m = rt.Model(path, max_batch=2, max_rows=16)
    got = m.generate(prompts, 16, use_graph=True)
    assert got.tolist() == want
    got2 = m.generate(prompts, 16, use_graph=False)
    assert got2.tolist() == want


@pytest.mark.parametrize("kind,kw", [
    ("gpt2", dict(L=2, D=256, H=4, S=128, V=1000, seed=9)),
    ("llama", dict(L=2, D=512, H=8, Hkv=2, F=768, S=128, V=1000, seed=9)),
])
@pytest.mark.parametrize("persistent", ["1", "0"])
def test_int8_kv_generate_matches_oracle(cuda, orc, model_dir, monkeypatch, kind, kw, persistent):
    """int8 K/V rows (LMC_KV_Q8) through the whole model, in the persistent
    step and kernel by kernel: teacher-forced logits within 1e-3 of the
    oracle storing its rows the same way, its greedy ids for 24 tokens, and
    within the int8 rounding (3e-2) of LMc's fp32 cache."""
    monkeypatch.setenv("LMC_PERSISTENT", persistent)
    path = tiny(kind, model_dir, **kw)
    prompt = np.random.default_rng(4).integers(0, kw["V"], 6).astype(np.int32)
    om, of = orc.model(path).set_kv(rt.KV_Q8), orc.model(path)
    m = rt.Model(path, max_batch=1, kv_dtype=rt.KV_Q8)
    for pos, t in enumerate(prompt):
        got, _ = m.forward([int(t)], [pos])
        want = om.forward(int(t), pos)
        assert rel_err(got[0], want) < 1e-3
        assert rel_err(got[0], of.forward(int(t), pos)) < 3e-2
    om2 = orc.model(path).set_kv(rt.KV_Q8)
    lg = None
    for pos, t in enumerate(prompt):
        lg = om2.forward(int(t), pos)
    ids, pos = [], len(prompt)
    for _ in range(24):
        ids.append(orc.argmax(lg))
        lg = om2.forward(ids[-1], pos)
        pos += 1
    m2 = rt.Model(path, max_batch=1, kv_dtype=rt.KV_Q8)
    assert m2.generate(prompt[None], 24, use_graph=True)[0].tolist() == ids
    assert rt.lib().lmc_device_status() == 0
