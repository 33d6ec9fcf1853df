"""The oracle (oracle/lmc_oracle.c) pinned against LMc itself: the committed
golden fixtures (LMc's own outputs, tests/golden/make_golden.py) and, when
the compiled LMc sources are present (oracle/_ref), random inputs."""
import os
import tempfile

import numpy as np
import pytest

from lmc_b200 import synth
from tests.conftest import ROOT, rel_err

GOLD = os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(GOLD, "kernels.npz"))


@pytest.fixture(scope="module")
def ref():
    from oracle import Ref, ref_library_path
    if not os.path.exists(ref_library_path()):
        pytest.skip("LMc reference build (oracle/_ref) not present")
    return Ref()


@pytest.mark.parametrize("t", synth.ALL_TYPES, ids=lambda t: synth.NAMES[t])
def test_dequant_golden(orc, gold, t):
    blk = gold[f"dq_{synth.NAMES[t]}_blocks"]
    want = gold[f"dq_{synth.NAMES[t]}_out"]
    got = orc.dequant(t, blk, want.size)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_gemv_and_ops_golden(orc, gold):
    w = orc.dequant(synth.Q4_K, gold["gemv_blocks"], 48 * 512).reshape(48, 512)
    assert rel_err(orc.matmul_vec(w, gold["gemv_x"], gold["gemv_bias"]), gold["gemv_y"]) < 1e-6
    x, w, b = gold["ops_x"], gold["ops_w"], gold["ops_b"]
    assert rel_err(orc.layer_norm(x, w, b), gold["ops_layer_norm"]) < 1e-6
    assert rel_err(orc.rms_norm(x, w, 1e-5), gold["ops_rms_norm"]) < 1e-6
    assert rel_err(orc.softmax(x), gold["ops_softmax"]) < 1e-6
    assert np.allclose(orc.gelu(x[:64]), gold["ops_gelu"], rtol=1e-6, atol=1e-7)
    assert np.allclose(orc.silu(x[:64]), gold["ops_silu"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("kind", ["gpt2", "llama"])
def test_model_golden(orc, kind):
    g = np.load(os.path.join(GOLD, f"model_{kind}.npz"))
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "m.gguf")
        g["gguf"].tofile(p)
        m = orc.model(p)
        for pos, t in enumerate(g["tokens"]):
            assert rel_err(m.forward(int(t), pos), g["logits"][pos]) < 1e-5
        m.close()
        m = orc.model(p)
        lg = None
        for pos, t in enumerate(g["prompt"]):
            lg = m.forward(int(t), pos)
        ids, pos = [], len(g["prompt"])
        for _ in range(len(g["ids"])):
            ids.append(orc.argmax(lg))
            lg = m.forward(ids[-1], pos)
            pos += 1
        assert ids == g["ids"].tolist()


@pytest.mark.parametrize("t", synth.ALL_TYPES, ids=lambda t: synth.NAMES[t])
def test_dequant_vs_lmc_random(orc, ref, t):
    be = max(synth.GEOMETRY[t][0], 8)
    for seed in range(4):
        n = be * 512
        blk = synth.random_blocks(t, n, seed=seed)
        assert np.array_equal(orc.dequant(t, blk, n).view(np.uint32), ref.dequant(t, blk, n).view(np.uint32))


def test_edge_scales_vs_lmc(orc, ref):
    """Zero, subnormal, max-finite and negative fp16 scales decode like LMc
    (scales kept finite: LMc's fast-math build is only flag-stable there)."""
    specials = np.array([0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0xFBFF, 0x3C00, 0xBC00], np.uint16)
    for t in synth.BLOCK_TYPES:
        be, bb, offs = synth.GEOMETRY[t]
        nb = len(specials)
        blk = synth.random_blocks(t, be * nb, seed=9)
        body = blk[:-synth.PAD].reshape(nb, bb)
        for o in offs:
            body[:, o:o + 2] = specials.view(np.uint8).reshape(nb, 2)
        blk = np.concatenate([body.reshape(-1), blk[-synth.PAD:]])
        a, b = orc.dequant(t, blk, be * nb), ref.dequant(t, blk, be * nb)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), synth.NAMES[t]


def test_matmul_vs_lmc(orc, ref):
    rng = np.random.default_rng(1)
    for M, K in ((7, 1600), (300, 768), (3, 17)):
        w = rng.normal(0, 1, (M, K)).astype(np.float32)
        x = rng.normal(0, 1, K).astype(np.float32)
        b = rng.normal(0, 1, M).astype(np.float32)
        assert rel_err(orc.matmul_vec(w, x, b), ref.matmul_vec(w, x, b)) < 1e-5


def test_norms_softmax_vs_lmc(orc, ref):
    """LayerNorm, RMSNorm and softmax of the oracle against LMc's compiled
    ops.c / ops_llama.c on random rows of the model widths and on edge rows:
    one element, a constant row (zero variance: rstd = 1/sqrt(eps)), zeros,
    and large magnitudes."""
    rng = np.random.default_rng(11)
    rows = [rng.normal(0, s, n).astype(np.float32) for n, s in ((768, 1.0), (2048, 3.0), (4096, 0.1), (100, 50.0))]
    rows += [np.array([2.5], np.float32), np.full(256, 7.0, np.float32), np.zeros(64, np.float32),
             rng.normal(0, 1e4, 512).astype(np.float32)]
    for x in rows:
        w = rng.normal(1, 0.1, x.size).astype(np.float32)
        b = rng.normal(0, 0.1, x.size).astype(np.float32)
        assert rel_err(orc.layer_norm(x, w, b), ref.layer_norm(x, w, b)) < 1e-5
        if np.any(x):
            assert rel_err(orc.rms_norm(x, w, 1e-5), ref.rms_norm(x, w, 1e-5)) < 1e-5
        else:
            assert np.array_equal(orc.rms_norm(x, w, 1e-5), ref.rms_norm(x, w, 1e-5))
        assert rel_err(orc.softmax(x), ref.softmax(x)) < 1e-5


@pytest.mark.parametrize("kind,kw", [
    ("gpt2", dict(L=2, D=256, H=4, S=64, V=700, seed=21)),
    ("llama", dict(L=2, D=256, H=8, Hkv=2, F=512, S=64, V=700, seed=21)),
])
def test_model_vs_lmc_random(orc, ref, tmp_path, kind, kw):
    """A freshly generated model (not a fixture): the oracle's teacher-forced
    logits match LMc's compiled model_forward within 1e-5 and its greedy ids
    match LMc's generate loop."""
    path = str(tmp_path / f"{kind}.gguf")
    (synth.make_gpt2 if kind == "gpt2" else synth.make_llama)(path, **kw)
    prompt = np.random.default_rng(3).integers(0, kw["V"], 6).astype(np.int32)
    ref.load(path)
    want_ids, _, _ = ref.generate(prompt, 12)
    ref.load(path)
    m = orc.model(path)
    lg = None
    for pos, t in enumerate(prompt):
        lg = m.forward(int(t), pos)
        assert rel_err(lg, ref.forward(int(t), pos)) < 1e-5
    ids, pos = [], len(prompt)
    for _ in range(12):
        ids.append(orc.argmax(lg))
        lg = m.forward(ids[-1], pos)
        pos += 1
    m.close()
    assert ids == want_ids.tolist()


@pytest.mark.parametrize("H,Hkv,Dh,S,pos", [(12, 12, 64, 32, 0), (12, 12, 64, 32, 31), (32, 4, 64, 128, 100),
                                            (32, 8, 128, 64, 40), (6, 2, 16, 8, 5)])
def test_attention_vs_float64(orc, H, Hkv, Dh, S, pos):
    """The oracle's attention read against a float64 statement of LMc's
    (ops.c:128-178, ops_llama.c:88-134): scores q.k / sqrt(Dh) over positions
    0..pos, softmax, weighted V; query head h reads kv head h / (H / Hkv)
    (the code's division, not the modulo its header comment names)."""
    rng = np.random.default_rng(H * 1000 + pos)
    q = rng.normal(0, 1, H * Dh).astype(np.float32)
    kc = rng.normal(0, 1, (Hkv, S, Dh)).astype(np.float32)
    vc = rng.normal(0, 1, (Hkv, S, Dh)).astype(np.float32)
    got = orc.attention(q, kc, vc, H, Hkv, Dh, S, pos).reshape(H, Dh)
    G = H // Hkv
    for h in range(H):
        k = kc[h // G, :pos + 1].astype(np.float64)
        v = vc[h // G, :pos + 1].astype(np.float64)
        s = k @ q[h * Dh:(h + 1) * Dh].astype(np.float64) / np.sqrt(Dh)
        p = np.exp(s - s.max())
        want = (p / p.sum()) @ v
        assert rel_err(got[h], want) < 1e-5, h


def test_rope_and_activations_vs_float64(orc):
    """RoPE table (models.c:101-117: angle = pos / theta^(2d/Dh)), the pair
    rotation (ops_llama.c:39-48) and GELU / SiLU (ops.c:20-29) of the oracle
    against float64 statements of the same formulas."""
    S, Dh, theta = 300, 128, 10000.0
    c, s = orc.rope_cache(S, Dh, theta)
    pos = np.arange(S, dtype=np.float64)[:, None]
    d = np.arange(Dh // 2, dtype=np.float64)[None, :]
    ang = pos / np.power(theta, 2.0 * d / Dh)
    # float32 angles of up to ~300 rad: the table matches to float32 angle rounding
    assert np.max(np.abs(c - np.cos(ang))) < 2e-4 and np.max(np.abs(s - np.sin(ang))) < 2e-4
    rng = np.random.default_rng(2)
    v = rng.normal(0, 1, Dh).astype(np.float32)
    got = orc.rope_apply(v, c[123], s[123])
    x0, x1 = v[0::2].astype(np.float64), v[1::2].astype(np.float64)
    cc, ss = c[123].astype(np.float64), s[123].astype(np.float64)
    want = np.empty(Dh)
    want[0::2], want[1::2] = x0 * cc - x1 * ss, x0 * ss + x1 * cc
    assert np.max(np.abs(got - want)) < 1e-5
    x = np.linspace(-20, 20, 401).astype(np.float32)
    xd = x.astype(np.float64)
    assert np.allclose(orc.gelu(x), xd / (1 + np.exp(-1.702 * xd)), rtol=1e-5, atol=1e-6)
    assert np.allclose(orc.silu(x), xd / (1 + np.exp(-xd)), rtol=1e-5, atol=1e-6)


def test_kv_row_forms(orc):
    """The compact KV row forms the device cache offers: fp16 rounding equals
    IEEE half rounding (numpy), and the int8 row quantization keeps every
    value within half a step (scale / 2) with the maximum at +-127."""
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.normal(0, 1, 4000), rng.normal(0, 1e-5, 1000), rng.normal(0, 3e4, 1000),
                        [65504.0, 65519.0, 65520.0, -65520.0, 6e-8, 3e-8, 0.0]]).astype(np.float32)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).astype(np.float32)
    got = orc.kv_round_rows(x[None], 1)[0]
    assert np.array_equal(got, want)
    for scale in (1.0, 1e-3, 50.0):
        r = rng.normal(0, scale, 128).astype(np.float32)
        q, sc = orc.kv_q8_row(r)
        assert np.abs(q).max() == 127 and np.abs(q.astype(np.int32)).max() <= 127
        assert np.float32(sc) == np.float32(np.abs(r).max() / np.float32(127.0))
        assert np.abs(q * np.float32(sc) - r).max() <= sc / 2 * (1 + 1e-6)
    q, sc = orc.kv_q8_row(np.zeros(64, np.float32))
    assert sc == 0.0 and not q.any()
