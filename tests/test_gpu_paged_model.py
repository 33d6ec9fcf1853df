"""The model's own KV cache paged (lmc_model_load_paged) against LMc's
forward restated by the oracle (storing its K/V rows the way the cache does):
teacher-forced logits within rel-err 1e-3 and identical greedy ids while
sequences take pages from one pool, give them back and take them again in
another order; a call that finds too few free pages fails with
LMC_ERR_OOM and changes nothing."""
import numpy as np
import pytest

from lmc_b200 import runtime as rt
from lmc_b200 import synth
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu

ERR_INVALID, ERR_OOM = -1, -4
GPT2 = ("gpt2", dict(L=2, D=256, H=4, S=128, V=1000, seed=5))
# head size 64 with 4 query heads per kv head: the tensor-core attention body
LLAMA = ("llama", dict(L=2, D=512, H=8, Hkv=2, F=768, S=128, V=1000, seed=5))


def _model(kind, model_dir, kw):
    return synth.cached_model(kind, model_dir, **kw)


def _check(m, oms, toks, pos):
    """One forward of rows 0..len(toks)-1 (row b = sequence b) against the
    oracles of those sequences."""
    got, nxt = m.forward(toks, pos)
    for b, (t, p) in enumerate(zip(toks, pos)):
        want = oms[b].forward(int(t), int(p))
        assert rel_err(got[b], want) < 1e-3, (b, p)
        assert nxt[b] == int(np.argmax(got[b]))


@pytest.mark.parametrize("kind,kw", [GPT2, LLAMA])
@pytest.mark.parametrize("kvd", [rt.KV_F32, rt.KV_F16, rt.KV_Q8])
def test_paged_cache_pages_reused_out_of_order(cuda, orc, model_dir, kind, kw, kvd):
    path = _model(kind, model_dir, kw)
    V = kw["V"]
    rng = np.random.default_rng(11)
    a, b, c = (rng.integers(0, V, 64).astype(np.int32) for _ in range(3))
    m = rt.Model(path, max_batch=2, kv_dtype=kvd, page_size=16, n_pages=6)
    assert m.kv_pages() == (16, 6, 6)
    oms = [orc.model(path).set_kv(kvd), orc.model(path).set_kv(kvd)]
    for t in range(16):  # both sequences: pages 0 (sequence 0) and 1 (sequence 1)
        _check(m, oms, [a[t], b[t]], [t, t])
    for t in range(16, 40):  # sequence 0 alone: pages 2 and 3
        _check(m, oms[:1], [a[t]], [t])
    assert m.kv_pages() == (16, 6, 2)
    m.release_seq(0)  # pages 0, 2, 3 back to the pool
    assert m.kv_pages() == (16, 6, 5)
    # sequence 0 starts again with other tokens while sequence 1 goes on:
    # their pages now come out of order (sequence 1: 1, 2, 4; sequence 0:
    # 0, 3), over rows the first sequence 0 left behind
    oms[0] = orc.model(path).set_kv(kvd)
    for u in range(32):
        _check(m, oms, [c[u], b[16 + u]], [u, 16 + u])
    assert m.kv_pages() == (16, 6, 1)
    # two more pages wanted, one free: refused, nothing taken
    with pytest.raises(rt.LmcError) as e:
        m.forward([c[32], b[48]], [32, 48])
    assert e.value.code == ERR_OOM
    assert m.kv_pages() == (16, 6, 1)
    for u in range(32, 40):  # sequence 0 alone takes the last page
        _check(m, oms[:1], [c[u]], [u])
    assert m.kv_pages() == (16, 6, 0)
    m.release_seq(1)
    assert m.kv_pages() == (16, 6, 3)
    assert rt.lib().lmc_device_status() == 0  # no page id outside the pool was met


@pytest.mark.parametrize("kind,kw", [GPT2, LLAMA])
def test_paged_cache_generate_prefill_replay(cuda, orc, model_dir, kind, kw):
    """Generation with prompt chunks (two rows per step, eight rows per
    chunk), its replay, and a batched prefill after both sequences gave their
    pages back: the oracle's ids and logits, fp16 rows."""
    kvd = rt.KV_F16
    path = _model(kind, model_dir, kw)
    V = kw["V"]
    prompt = np.random.default_rng(12).integers(0, V, 12).astype(np.int32)
    om = orc.model(path).set_kv(kvd)
    lg = None
    for pos, t in enumerate(prompt):
        lg = om.forward(int(t), pos)
    prompt_lg = lg
    ids, pos = [], len(prompt)
    for _ in range(24):
        ids.append(orc.argmax(lg))
        lg = om.forward(ids[-1], pos)
        pos += 1
    m = rt.Model(path, max_batch=2, kv_dtype=kvd, max_rows=8, page_size=16, n_pages=8)
    got = m.generate(np.stack([prompt, prompt]), 24, use_graph=True)
    assert got[0].tolist() == ids and got[1].tolist() == ids
    assert m.kv_pages() == (16, 8, 2)  # positions 0..34: three pages each
    s = m.replay(10)  # positions 35..44: no new page
    assert m.kv_pages() == (16, 8, 2)
    s = m.replay(5)  # positions 45..49: a fourth page each
    assert m.kv_pages() == (16, 8, 0)
    with pytest.raises(rt.LmcError) as e:
        m.replay(20)  # positions 50..69 need a fifth page each
    assert e.value.code == ERR_OOM
    with pytest.raises(rt.LmcError) as e:
        m.replay(200)  # beyond the context
    assert e.value.code == ERR_INVALID
    rt.call("lmc_stream_sync", s)
    assert rt.lib().lmc_device_status() == 0
    m.release_seq(0)
    m.release_seq(1)
    assert m.kv_pages() == (16, 8, 8)
    got_lg, nxt = m.prefill(1, prompt)
    assert rel_err(got_lg, prompt_lg) < 1e-3
    assert nxt == orc.argmax(prompt_lg)
    oms = [orc.model(path).set_kv(kvd), orc.model(path).set_kv(kvd)]
    for p, t in enumerate(prompt):
        oms[1].forward(int(t), p)
    _check(m, oms, [prompt[0], ids[0]], [0, len(prompt)])
    _check(m, oms, [prompt[1], ids[1]], [1, len(prompt) + 1])
    assert rt.lib().lmc_device_status() == 0


def test_paged_cache_rejects_page_size_not_dividing_context(cuda, model_dir):
    path = _model("gpt2", model_dir, GPT2[1])  # context 128
    with pytest.raises(rt.LmcError) as e:
        rt.Model(path, max_batch=1, page_size=256, n_pages=2)
    assert e.value.code == ERR_INVALID
