"""The persistent decode step (one cooperative launch per token, grid-wide
barriers between ops) against the oracle and against the kernel-by-kernel
step: teacher-forced logits within rel-err 1e-3, identical greedy ids, and a
captured generate step that is one kernel."""
import os

import numpy as np
import pytest

from lmc_b200 import runtime as rt
from lmc_b200 import synth
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu

MODELS = [
    ("gpt2", dict(L=2, D=256, H=4, S=128, V=1000, seed=11)),
    # head size 64 (the persistent attention takes 64 and 128)
    ("llama", dict(L=2, D=512, H=8, Hkv=2, F=768, S=128, V=1000, seed=11)),
    ("llama", dict(L=1, D=1024, H=8, Hkv=4, F=1536, S=96, V=700, seed=12)),
]


def oracle_ids(orc, path, prompt, n):
    om = orc.model(path)
    lg = None
    for pos, t in enumerate(prompt):
        lg = om.forward(int(t), pos)
    ids, pos = [], len(prompt)
    for _ in range(n):
        ids.append(orc.argmax(lg))
        lg = om.forward(ids[-1], pos)
        pos += 1
    return ids


@pytest.mark.parametrize("kind,kw", MODELS)
@pytest.mark.parametrize("kvd", [rt.KV_F32, rt.KV_F16, rt.KV_Q8])
@pytest.mark.parametrize("B", [1, 2])
def test_persistent_forward_logits(cuda, orc, model_dir, kind, kw, kvd, B):
    path = synth.cached_model(kind, model_dir, **kw)
    om = [orc.model(path).set_kv(kvd) for _ in range(B)]  # the oracle stores K/V rows as the cache does
    m = rt.Model(path, max_batch=B, kv_dtype=kvd)
    toks = np.random.default_rng(5).integers(0, kw["V"], (B, 9))
    tol = 1e-3
    for pos in range(toks.shape[1]):
        got, nxt = m.forward(toks[:, pos], [pos] * B)
        for b in range(B):
            want = om[b].forward(int(toks[b, pos]), pos)
            assert rel_err(got[b], want) < tol
            assert nxt[b] == int(np.argmax(got[b]))


@pytest.mark.parametrize("kind,kw", MODELS)
def test_persistent_generate_one_kernel(cuda, orc, model_dir, kind, kw):
    path = synth.cached_model(kind, model_dir, **kw)
    prompt = np.random.default_rng(1).integers(0, kw["V"], 6).astype(np.int32)
    want = oracle_ids(orc, path, prompt, 24)
    m = rt.Model(path, max_batch=2)
    got = m.generate(np.stack([prompt, prompt]), 24, use_graph=True)
    assert m.graph_kernels() == 1, "the captured step is one persistent kernel"
    assert got[0].tolist() == want and got[1].tolist() == want
    got1 = m.generate(prompt[None], 24, use_graph=False)
    assert got1[0].tolist() == want
    assert rt.call("lmc_device_status") == 0


def test_persistent_matches_kernel_by_kernel(cuda, model_dir, monkeypatch):
    """LMC_PERSISTENT=0 launches the same step op by op: same ids, logits
    equal to rounding (the two differ only in where the GEMV splits its rows)."""
    kind, kw = MODELS[0]
    path = synth.cached_model(kind, model_dir, **kw)
    prompt = np.random.default_rng(2).integers(0, kw["V"], 5).astype(np.int32)
    m1 = rt.Model(path, max_batch=1)
    a = m1.generate(prompt[None], 20, use_graph=True)
    lg1, _ = m1.forward([3], [30])
    monkeypatch.setenv("LMC_PERSISTENT", "0")
    m2 = rt.Model(path, max_batch=1)
    b = m2.generate(prompt[None], 20, use_graph=True)
    assert m2.graph_kernels() > 1
    lg2, _ = m2.forward([3], [30])
    assert a.tolist() == b.tolist()
    assert rel_err(lg1, lg2) < 1e-5


def test_persistent_forced_on_wide_model(cuda, model_dir, monkeypatch):
    """Models above the size where the kernel-by-kernel path is the default
    still run the persistent step when it is asked for (LMC_PERSISTENT=1):
    the TinyLlama width (2048, 32 / 4 heads, FFN 5632, vocab 32000), two
    layers, tensor-core GEMVs on the long rows: the same logits and ids as
    the kernel-by-kernel step."""
    kw = dict(L=2, D=2048, H=32, Hkv=4, F=5632, S=256, V=32000, blocks="random", seed=13)
    path = synth.cached_model("llama", model_dir, **kw)
    toks = np.random.default_rng(6).integers(0, kw["V"], 5)
    monkeypatch.setenv("LMC_PERSISTENT", "0")
    m0 = rt.Model(path, max_batch=1)
    want = [m0.forward([int(t)], [pos])[0][0] for pos, t in enumerate(toks)]
    m0.close()
    monkeypatch.setenv("LMC_PERSISTENT", "1")
    m1 = rt.Model(path, max_batch=1)
    for pos, t in enumerate(toks):
        got, nxt = m1.forward([int(t)], [pos])
        assert rel_err(got[0], want[pos]) < 1e-3
        assert nxt[0] == int(np.argmax(want[pos]))
    prompt = toks[:4].astype(np.int32)
    a = m1.generate(prompt[None], 12, use_graph=True)
    assert m1.graph_kernels() == 1
    monkeypatch.setenv("LMC_PERSISTENT", "0")
    m2 = rt.Model(path, max_batch=1)
    assert m2.generate(prompt[None], 12, use_graph=True).tolist() == a.tolist()
