"""Tensor-parallel decode on two GPUs (one process each; residual sums over
peer memory or NCCL, both over NVLink):
a LLaMA model sharded by heads / ffn rows / vocabulary must give each rank's
vocabulary slice of the oracle's logits within 1e-3 and the oracle's greedy
ids.  Skipped on a single-GPU machine."""
import multiprocessing as mp

import numpy as np
import pytest

from lmc_b200 import runtime as rt
from lmc_b200 import synth
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu

KW = dict(L=2, D=512, H=8, Hkv=2, F=1024, S=128, V=1000, seed=4)


def _rank(rank, world, path, nid, prompts, n_new, q):
    try:
        import torch
        torch.cuda.set_device(rank)
        rt.init(rank)
        m = rt.Model(path, max_batch=prompts.shape[0], tp=(rank, world, nid))
        logits = []
        for pos in range(prompts.shape[1]):
            lg, _ = m.forward(prompts[:, pos], [pos] * prompts.shape[0])
            logits.append(lg)
        ids = m.generate(prompts, n_new)  # (one communicator per group id: same model, restarts at position 0)
        q.put((rank, m.vocab_begin, m.vocab_rows, np.stack(logits), ids, None))
        m.close()
    except Exception as e:  # reported to the parent
        q.put((rank, 0, 0, None, None, repr(e)))


@pytest.mark.parametrize("peer", ["1", "0"], ids=["peer-sums", "nccl-sums"])
def test_tp2_matches_oracle(cuda, orc, model_dir, monkeypatch, peer):
    """The residual sums over peer memory (the default) and through NCCL."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    monkeypatch.setenv("LMC_TP_PEER", peer)  # inherited by the spawned ranks
    world, n_new = 2, 12
    path = synth.cached_model("llama", model_dir, **KW)
    rng = np.random.default_rng(11)
    prompts = rng.integers(0, KW["V"], (2, 5)).astype(np.int32)
    # oracle: teacher-forced logits and greedy continuation per sequence
    want_lg, want_ids = [], []
    for b in range(prompts.shape[0]):
        om = orc.model(path)
        lgs = [om.forward(int(t), pos) for pos, t in enumerate(prompts[b])]
        want_lg.append(np.stack(lgs))
        lg, pos, ids = lgs[-1], prompts.shape[1], []
        for _ in range(n_new):
            nxt = orc.argmax(lg)
            ids.append(nxt)
            lg = om.forward(nxt, pos)
            pos += 1
        want_ids.append(ids)
    nid = rt.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, path, nid, prompts, n_new, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=300) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    for rank, v0, vl, lg, ids, err in res:
        assert err is None, err
        for b in range(prompts.shape[0]):
            for pos in range(prompts.shape[1]):
                assert rel_err(lg[pos, b], want_lg[b][pos, v0:v0 + vl]) < 1e-3
            assert ids[b].tolist() == want_ids[b]
    assert res[0][1] == 0 and res[0][2] + res[1][2] == KW["V"]


# The Llama-8B width (4096, 32 / 8 heads, FFN 14336, vocab 128256) with two
# layers, sharded over 2, 4 and 8 GPUs: each rank's vocabulary slice of the
# teacher-forced logits within 1e-3 of LMc's own (oracle/_ref), and the
# group's greedy pick equal to the argmax of LMc's logits.
W8B = dict(L=2, D=4096, H=32, Hkv=8, F=14336, S=256, V=128256, blocks="random", seed=8)


def _rank_logits(rank, world, path, nid, toks, q):
    try:
        import torch
        torch.cuda.set_device(rank)
        rt.init(rank)
        m = rt.Model(path, max_batch=1, tp=(rank, world, nid))
        out = []
        for pos, t in enumerate(toks):
            lg, nxt = m.forward([int(t)], [pos])
            out.append((lg[0], int(nxt[0])))
        q.put((rank, m.vocab_begin, m.vocab_rows, out, None))
        m.close()
    except Exception as e:
        q.put((rank, 0, 0, None, repr(e)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_8b_width_vs_lmc(cuda, model_dir, world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle import Ref
    path = synth.cached_model("llama", model_dir, **W8B)
    toks = np.random.default_rng(3).integers(0, W8B["V"], 3)
    ref = Ref()
    ref.load(path)
    want = [ref.forward(int(t), pos) for pos, t in enumerate(toks)]
    nid = rt.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_logits, args=(r, world, path, nid, toks, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=600) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    covered = 0
    for rank, v0, vl, out, err in res:
        assert err is None, err
        covered += vl
        for pos, (lg, nxt) in enumerate(out):
            assert rel_err(lg, want[pos][v0:v0 + vl]) < 1e-3
            assert nxt == int(np.argmax(want[pos]))
    assert covered == W8B["V"]
