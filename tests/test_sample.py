"""Top-p sampling (LMc's sample_top_p, src/lmc.c:29-59).

CPU: the oracle's restatement draws the same tokens and leaves the same
xorshift64 state as LMc's own function (compiled from lmc.c into
oracle/_ref), except where the draw lies within 1e-5 of a cdf boundary (LMc
is built with -ffast-math, the oracle without, so sums round differently).
GPU: lmc_sample_top_p (and the generate loop with sampling) against the
oracle, under the same boundary rule."""
import ctypes

import numpy as np
import pytest

from lmc_b200 import runtime as rt
from lmc_b200 import synth

CASES = [(0.7, 0.9), (1.0, 0.5), (0.0, 0.9), (1e-7, 0.9), (1.3, 1.0), (0.5, 0.05), (2.0, 0.99)]
MARGIN = 1e-5


def logits_rows(V, n, seed, scale=2.0):
    rng = np.random.default_rng(seed)
    return rng.normal(0, scale, (n, V)).astype(np.float32)


def test_rng_seed_matches_lmc():
    """rng_seed (src/lmc.c:30-31): seed ^ 0xdeadbeefcafe, never 0."""
    L = rt.lib()
    assert L.lmc_rng_seed(0) == 0xdeadbeefcafe
    assert L.lmc_rng_seed(0xdeadbeefcafe) == 1
    assert L.lmc_rng_seed(12345) == 12345 ^ 0xdeadbeefcafe


@pytest.mark.parametrize("V", [7, 1000, 50257])
def test_oracle_sampler_matches_lmc(orc, V):
    from oracle import Ref
    ref = Ref()
    compared = 0
    for ci, (t, p) in enumerate(CASES):
        st = 777 ^ 0xdeadbeefcafe
        for k, lg in enumerate(logits_rows(V, 12, seed=V + 100 * ci)):
            a, sa, margin = orc.sample_top_p(lg, t, p, st)
            b, sb = ref.sample_top_p(lg, t, p, st)
            assert sa == sb, "the RNG advances once per draw (never for greedy)"
            if margin >= MARGIN:
                assert a == b, (V, t, p, k)
                compared += 1
            st = sa
    assert compared >= (0.5 if V > 10000 else 0.8) * len(CASES) * 12  # large vocabularies: small cdf steps


@pytest.mark.gpu
@pytest.mark.parametrize("V", [7, 1000, 50257, 128256])
def test_device_sampler_matches_oracle(cuda, orc, V):
    torch = cuda
    rows = 4
    compared = 0
    for t, p in CASES:
        lg = logits_rows(V, rows, seed=V)
        states = np.array([rt.lib().lmc_rng_seed(1000 + r) for r in range(rows)], np.uint64)
        d_lg = torch.from_numpy(lg).cuda()
        d_st = torch.from_numpy(states.view(np.int64).copy()).cuda()
        d_out = torch.empty(rows, dtype=torch.int32, device="cuda")
        for draw in range(3):
            rt.call("lmc_sample_top_p", d_lg.data_ptr(), V, rows, t, p, d_st.data_ptr(), d_out.data_ptr(), None)
            torch.cuda.synchronize()
            got = d_out.cpu().numpy()
            new_st = d_st.cpu().numpy().view(np.uint64)
            for r in range(rows):
                tok, st2, margin = orc.sample_top_p(lg[r], t, p, int(states[r]))
                assert int(new_st[r]) == st2
                if margin >= MARGIN:
                    assert int(got[r]) == tok, (V, t, p, draw, r)
                    compared += 1
            states = new_st.copy()
    assert compared >= (0.35 if V > 10000 else 0.8) * len(CASES) * 3 * rows


@pytest.mark.gpu
def test_device_sampler_ties_and_edges(cuda, orc):
    """Equal logits (every probability ties): the draw walks the ties in
    index order; top_p above 1 keeps the whole vocabulary; a tiny top_p keeps
    the most probable token only."""
    torch = cuda
    V = 64
    d_out = torch.empty(1, dtype=torch.int32, device="cuda")
    for lg, t, p in [(np.zeros(V, np.float32), 1.0, 0.5), (np.zeros(V, np.float32), 1.0, 1.5),
                     (np.arange(V, dtype=np.float32), 1.0, 1e-6)]:
        st = rt.lib().lmc_rng_seed(99)
        d_st = torch.tensor([np.uint64(st).view(np.int64)], device="cuda")
        rt.call("lmc_sample_top_p", torch.from_numpy(lg).cuda().data_ptr(), V, 1, t, p, d_st.data_ptr(),
                d_out.data_ptr(), None)
        torch.cuda.synchronize()
        # the draw in float64, ties in index order
        s2 = st
        s2 ^= (s2 << 13) & 0xFFFFFFFFFFFFFFFF
        s2 ^= s2 >> 7
        s2 ^= (s2 << 17) & 0xFFFFFFFFFFFFFFFF
        r = np.float32(s2 >> 11) / np.float32(2.0 ** 53)
        pr = np.exp(lg * (1 / t) - (lg * (1 / t)).max())
        pr = pr / pr.sum()
        order = sorted(range(V), key=lambda i: (-pr[i], i))
        cum, nuc = 0.0, 0
        for i in order:
            cum += pr[i]
            nuc += 1
            if cum >= p:
                break
        ns = sum(pr[i] for i in order[:nuc])
        cdf, want = 0.0, order[nuc - 1]
        for i in order[:nuc]:
            cdf += pr[i] / ns
            if r < cdf:
                want = i
                break
        assert int(d_out.item()) == want, (t, p)


@pytest.mark.gpu
@pytest.mark.parametrize("kind,kw", [
    ("gpt2", dict(L=2, D=256, H=4, S=128, V=1000, seed=31)),
    ("llama", dict(L=2, D=512, H=8, Hkv=2, F=768, S=128, V=1000, seed=31)),
])
@pytest.mark.parametrize("use_graph", [True, False])
def test_generate_sample_matches_oracle(cuda, orc, model_dir, kind, kw, use_graph):
    """lmc_model_generate_sample against the oracle's forward + sampler loop
    (LMc's generate with --temp 0.8 --top-p 0.9): every draw that lies more
    than 1e-5 from a cdf boundary picks the oracle's token; where a draw is
    that close, the oracle continues from the device's token."""
    path = synth.cached_model(kind, model_dir, **kw)
    prompt = np.random.default_rng(2).integers(0, kw["V"], 6).astype(np.int32)
    T, P, seed, n_new = 0.8, 0.9, 4242, 24
    m = rt.Model(path, max_batch=2)
    out = np.empty((2, n_new), np.int32)
    p2 = np.ascontiguousarray(np.stack([prompt, prompt]))
    rt.call("lmc_model_generate_sample", m.h, p2.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), len(prompt), 2, n_new,
            T, P, seed, int(use_graph), out.ctypes.data_as(ctypes.POINTER(ctypes.c_int)))
    for b in range(2):
        om = orc.model(path)
        lg = None
        for pos, t in enumerate(prompt):
            lg = om.forward(int(t), pos)
        st = rt.lib().lmc_rng_seed(seed + b)
        pos, compared = len(prompt), 0
        for i in range(n_new):
            tok, st, margin = orc.sample_top_p(lg, T, P, st)
            if margin >= MARGIN:
                assert int(out[b, i]) == tok, (b, i)
                compared += 1
            lg = om.forward(int(out[b, i]), pos)
            pos += 1
        assert compared >= n_new // 2
    # temperature 0 is the greedy loop
    g = m.generate(p2, n_new, use_graph=use_graph)
    rt.call("lmc_model_generate_sample", m.h, p2.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), len(prompt), 2, n_new,
            0.0, P, seed, int(use_graph), out.ctypes.data_as(ctypes.POINTER(ctypes.c_int)))
    assert out.tolist() == g.tolist()
