"""CUDA kernels against the oracle, through the C ABI (liblmc_b200.so).

Dequant must be bit-exact; GEMV / ops / attention within the norm-wise
relative error 1e-3 of the fp32 reference (the tolerance LMc parity is
stated in), with tighter bounds where the math allows."""
import numpy as np
import pytest

from lmc_b200 import runtime as rt
from lmc_b200 import synth
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
RTOL = 1e-3


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def gpu_dequant(torch, t, blk, n):
    d = dev(torch, blk)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    rt.call("lmc_dequant", t, d.data_ptr(), n, out.data_ptr(), None)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("t", synth.ALL_TYPES, ids=lambda t: synth.NAMES[t])
def test_dequant_bit_exact(cuda, orc, t):
    be = max(synth.GEOMETRY[t][0], 8)
    for seed, nblk in ((0, 1), (1, 37), (2, 4096)):
        n = be * nblk
        blk = synth.random_blocks(t, n, seed=seed)
        a = orc.dequant(t, blk, n)
        b = gpu_dequant(cuda, t, blk, n)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (synth.NAMES[t], nblk)


def test_dequant_f16_all_patterns(cuda, orc):
    blk = np.concatenate([np.arange(65536, dtype=np.uint16).view(np.uint8), np.zeros(16, np.uint8)])
    a = orc.dequant(synth.F16, blk, 65536)
    b = gpu_dequant(cuda, synth.F16, blk, 65536)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_dequant_iq4xs_reads_next_block(cuda, orc):
    """IQ4_XS code bytes 126-127 of block i come from block i+1 (LMc
    quant.c:506,515): changing the next block's first bytes changes them."""
    n = 512
    blk = synth.random_blocks(synth.IQ4_XS, n, seed=5)
    a = gpu_dequant(cuda, synth.IQ4_XS, blk, n)
    blk2 = blk.copy()
    blk2[136] ^= 0xFF
    b = gpu_dequant(cuda, synth.IQ4_XS, blk2, n)
    assert not np.array_equal(a[252:256], b[252:256])
    assert np.array_equal(orc.dequant(synth.IQ4_XS, blk2, n).view(np.uint32), b.view(np.uint32))


def test_dequant_rejects_bad_size(cuda):
    d = cuda.zeros(1024, dtype=cuda.uint8, device="cuda")
    out = cuda.empty(300, dtype=cuda.float32, device="cuda")
    with pytest.raises(rt.LmcError):
        rt.call("lmc_dequant", synth.Q4_K, d.data_ptr(), 300, out.data_ptr(), None)
    with pytest.raises(rt.LmcError):
        rt.call("lmc_dequant", 99, d.data_ptr(), 256, out.data_ptr(), None)


def ref_gemv(orc, t, blk, M, K, x, bias=None):
    w = orc.dequant(t, blk, M * K).reshape(M, K)
    return np.stack([orc.matmul_vec(w, xb, bias) for xb in x])


GEMV_CASES = [
    (synth.Q4_K, 3072, 768), (synth.Q6_K, 768, 3072), (synth.Q8_0, 1000, 512), (synth.Q8_0, 3072, 768),
    (synth.Q4_K, 6400, 1600), (synth.Q5_K, 1600, 6400),  # 6400x1600: K-quant blocks straddle rows
] + [(t, 256, 512) for t in synth.ALL_TYPES] + [(t, 96, 1600) for t in synth.BLOCK_TYPES]


@pytest.mark.parametrize("t,M,K", GEMV_CASES, ids=lambda v: str(v))
@pytest.mark.parametrize("B", [1, 3, 8])
def test_gemv(cuda, orc, t, M, K, B):
    rng = np.random.default_rng(M + K + B)
    blk = synth.random_blocks(t, M * K, seed=M ^ K)
    x = rng.normal(0, 1, (B, K)).astype(np.float32)
    bias = rng.normal(0, 1, M).astype(np.float32)
    want = ref_gemv(orc, t, blk, M, K, x, bias)
    q = rt.QTensor(t, M, K, blk)
    dx, db = dev(cuda, x), dev(cuda, bias)
    y = cuda.empty((B, M), dtype=cuda.float32, device="cuda")
    q.matmul(dx, y, batch=B, bias=db)
    got = y.cpu().numpy()
    assert rel_err(got, want) < RTOL
    # the generic kernel on the raw blocks agrees too
    y2 = cuda.empty((B, M), dtype=cuda.float32, device="cuda")
    rt.call("lmc_matmul_blocks", t, rt.lib().lmc_qtensor_blocks(q.h), M, K, dx.data_ptr(), K, db.data_ptr(),
            y2.data_ptr(), M, B, 0, None)
    assert rel_err(y2.cpu().numpy(), want) < RTOL


# Shapes of the tensor-core path (Q4_K / Q6_K / Q8_0, cols % 256 == 0) that
# exercise its work split: long rows (K = 14336), ragged row count, many row
# tiles per cluster, and batch widths 2 and 5 (two rows per fragment, and an
# odd row in the last fragment).  At batch 1 the rows of more than two
# activation tasks a thread (K > 4096, Q6_K K > 2048) take a register-held
# activation variant: four slots for three or four tasks (Q6_K K = 3072,
# Q8_0 K = 5120 with some threads at three tasks and the others at two), the
# longest one up to its limits (K = 14336; Q6_K K = 16384; Q6_K K = 4352
# gives some threads five tasks and the others four), and Q4_K K = 16384
# the default one again.
TILED_CASES = [(synth.Q4_K, 4096, 14336), (synth.Q6_K, 50257, 768), (synth.Q8_0, 2048, 4096),
               (synth.Q4_K, 14336, 2048), (synth.Q8_0, 520, 768), (synth.Q8_0, 1024, 14336),
               (synth.Q6_K, 1040, 16384), (synth.Q6_K, 2048, 4352), (synth.Q4_K, 512, 16384),
               (synth.Q6_K, 768, 3072), (synth.Q8_0, 600, 5120)]


@pytest.mark.parametrize("t,M,K", TILED_CASES, ids=lambda v: str(v))
@pytest.mark.parametrize("B", [1, 2, 5])
def test_gemv_tiled_shapes(cuda, orc, t, M, K, B):
    rng = np.random.default_rng(M * 7 + K + B)
    blk = synth.random_blocks(t, M * K, seed=M + 3 * K)
    x = rng.normal(0, 1, (B, K)).astype(np.float32)
    want = ref_gemv(orc, t, blk, M, K, x)
    q = rt.QTensor(t, M, K, blk)
    assert q.tiled
    y = cuda.empty((B, M), dtype=cuda.float32, device="cuda")
    dx = dev(cuda, x)
    q.matmul(dx, y, batch=B)
    assert rel_err(y.cpu().numpy(), want) < RTOL
    assert rt.lib().lmc_device_status() == 0


# Batched GEMM on the tcgen05 tensor cores (batch widths above the GEMV's 8
# rows).  The weights enter as fp16 (relative rounding <= 2^-11) and x as fp16
# hi + lo, fp32 accumulation: the norm-wise relative error is ~3e-4, checked
# against the 1e-3 bound of the GEMV.
GEMM_CASES = [(synth.Q4_K, 3072, 768, 64), (synth.Q6_K, 768, 3072, 64), (synth.Q8_0, 1000, 512, 200),
              (synth.Q4_0, 6400, 1600, 16), (synth.Q5_1, 512, 1024, 512), (synth.Q3_K, 520, 1024, 9),
              (synth.Q5_K, 640, 2048, 100), (synth.IQ4_XS, 384, 1024, 64), (synth.F16, 256, 512, 33),
              (synth.Q2_K, 256, 768, 24), (synth.IQ3_XXS, 300, 512, 40), (synth.Q4_1, 256, 4096, 130)]


@pytest.mark.parametrize("t,M,K,N", GEMM_CASES, ids=lambda v: str(v))
def test_gemm(cuda, orc, t, M, K, N):
    rng = np.random.default_rng(M + 3 * K + N)
    blk = synth.random_blocks(t, M * K, seed=M + K)
    x = rng.normal(0, 1, (N, K)).astype(np.float32)
    bias = rng.normal(0, 1, M).astype(np.float32)
    want = ref_gemv(orc, t, blk, M, K, x, bias)
    q = rt.QTensor(t, M, K, blk)
    y = cuda.empty((N, M), dtype=cuda.float32, device="cuda")
    dx, db = dev(cuda, x), dev(cuda, bias)
    q.matmul(dx, y, batch=N, bias=db)
    assert rel_err(y.cpu().numpy(), want) < RTOL
    assert rt.lib().lmc_device_status() == 0


def test_gemm_epilogues(cuda, orc):
    t, M, K, N = synth.Q4_K, 640, 1024, 24
    rng = np.random.default_rng(5)
    blk = synth.random_blocks(t, M * K, seed=5)
    x = rng.normal(0, 1, (N, K)).astype(np.float32)
    bias = rng.normal(0, 1, M).astype(np.float32)
    base = ref_gemv(orc, t, blk, M, K, x, bias)
    q = rt.QTensor(t, M, K, blk)
    y = cuda.empty((N, M), dtype=cuda.float32, device="cuda")
    q.matmul(dev(cuda, x), y, batch=N, bias=dev(cuda, bias), epilogue=rt.EPI_GELU)
    assert rel_err(y.cpu().numpy(), orc.gelu(base)) < RTOL
    resid = rng.normal(0, 1, (N, M)).astype(np.float32)
    y = dev(cuda, resid)
    q.matmul(dev(cuda, x), y, batch=N, bias=dev(cuda, bias), epilogue=rt.EPI_ACCUM)
    assert rel_err(y.cpu().numpy(), resid + base) < RTOL


def test_gemv_epilogues(cuda, orc):
    t, M, K, B = synth.Q4_K, 512, 1024, 2
    rng = np.random.default_rng(3)
    blk = synth.random_blocks(t, M * K, seed=3)
    x = rng.normal(0, 1, (B, K)).astype(np.float32)
    bias = rng.normal(0, 1, M).astype(np.float32)
    base = ref_gemv(orc, t, blk, M, K, x, bias)
    q = rt.QTensor(t, M, K, blk)
    y = cuda.empty((B, M), dtype=cuda.float32, device="cuda")
    q.matmul(dev(cuda, x), y, batch=B, bias=dev(cuda, bias), epilogue=rt.EPI_GELU)
    assert rel_err(y.cpu().numpy(), orc.gelu(base)) < RTOL
    resid = rng.normal(0, 1, (B, M)).astype(np.float32)
    y = dev(cuda, resid)
    q.matmul(dev(cuda, x), y, batch=B, bias=dev(cuda, bias), epilogue=rt.EPI_ACCUM)
    assert rel_err(y.cpu().numpy(), resid + base) < RTOL


def test_layer_rms_norm_softmax(cuda, orc):
    rng = np.random.default_rng(0)
    for dim in (768, 2048, 4096, 100):
        x = rng.normal(0, 2, (3, dim)).astype(np.float32)
        w = rng.normal(1, 0.1, dim).astype(np.float32)
        b = rng.normal(0, 0.1, dim).astype(np.float32)
        out = cuda.empty((3, dim), dtype=cuda.float32, device="cuda")
        dx, dw, db = dev(cuda, x), dev(cuda, w), dev(cuda, b)  # keep the buffers alive across the call
        rt.call("lmc_layer_norm", out.data_ptr(), dx.data_ptr(), dw.data_ptr(), db.data_ptr(), dim, 3, None)
        want = np.stack([orc.layer_norm(r, w, b) for r in x])
        assert rel_err(out.cpu().numpy(), want) < 1e-5
        rt.call("lmc_rms_norm", out.data_ptr(), dx.data_ptr(), dw.data_ptr(), dim, 3, 1e-5, None)
        want = np.stack([orc.rms_norm(r, w, 1e-5) for r in x])
        assert rel_err(out.cpu().numpy(), want) < 1e-5
        s = dev(cuda, x * 3)
        rt.call("lmc_softmax", s.data_ptr(), dim, 3, None)
        want = np.stack([orc.softmax(r * 3) for r in x])
        assert rel_err(s.cpu().numpy(), want) < 1e-5


def test_activations_rope(cuda, orc):
    rng = np.random.default_rng(1)
    x = rng.normal(0, 3, 5000).astype(np.float32)
    for name, fn in (("lmc_gelu", orc.gelu), ("lmc_silu", orc.silu)):
        d = dev(cuda, x)
        rt.call(name, d.data_ptr(), x.size, None)
        assert np.allclose(d.cpu().numpy(), fn(x), rtol=1e-6, atol=1e-6)
    u = rng.normal(0, 1, 5000).astype(np.float32)
    d, du = dev(cuda, x), dev(cuda, u)
    rt.call("lmc_swiglu", d.data_ptr(), du.data_ptr(), x.size, None)
    assert np.allclose(d.cpu().numpy(), orc.silu(x) * u, rtol=1e-6, atol=1e-6)
    c, s = orc.rope_cache(64, 64, 10000.0)
    v = rng.normal(0, 1, (4, 64)).astype(np.float32)
    d, dc, ds = dev(cuda, v), dev(cuda, c[37]), dev(cuda, s[37])
    rt.call("lmc_rope_apply", d.data_ptr(), dc.data_ptr(), ds.data_ptr(), 64, 4, None)
    want = np.stack([orc.rope_apply(r, c[37], s[37]) for r in v])
    assert np.allclose(d.cpu().numpy(), want, rtol=1e-6, atol=1e-6)


def test_argmax_first_max(cuda, orc):
    rng = np.random.default_rng(2)
    x = rng.normal(0, 1, (4, 50257)).astype(np.float32)
    x[1, 17] = x[1, 40000] = 99.0  # tie: the first index wins (lmc.c:45-47)
    x[2, :] = 1.0
    x[3, 50256] = 50.0
    idx = cuda.empty(4, dtype=cuda.int32, device="cuda")
    dx = dev(cuda, x)
    rt.call("lmc_argmax", dx.data_ptr(), 50257, 4, idx.data_ptr(), None)
    assert idx.cpu().numpy().tolist() == [orc.argmax(r) for r in x] == [orc.argmax(x[0]), 17, 0, 50256]


@pytest.mark.parametrize("H,Hkv,Dh,S,pos,kvd", [
    (12, 12, 64, 1024, 0, rt.KV_F32), (12, 12, 64, 1024, 135, rt.KV_F32),
    (32, 4, 64, 2048, 700, rt.KV_F32), (32, 8, 128, 4096, 1500, rt.KV_F32),
    (32, 4, 64, 2048, 511, rt.KV_F16), (8, 8, 64, 64, 63, rt.KV_F32),
    # fp16 caches: the tensor-core body (head 64/128, 1-8 query heads per kv
    # head, short and long contexts) and the CUDA-core body (16 query heads
    # per kv head; head 96)
    (32, 8, 128, 4096, 1500, rt.KV_F16), (12, 12, 64, 1024, 135, rt.KV_F16), (32, 4, 64, 2048, 14, rt.KV_F16),
    (32, 2, 64, 512, 300, rt.KV_F16), (6, 2, 96, 256, 200, rt.KV_F16), (6, 2, 96, 256, 200, rt.KV_F32)])
def test_attention(cuda, orc, H, Hkv, Dh, S, pos, kvd):
    rng = np.random.default_rng(pos + H)
    B = 2
    kc = rng.normal(0, 1, (B, Hkv, S, Dh)).astype(np.float32)
    vc = rng.normal(0, 1, (B, Hkv, S, Dh)).astype(np.float32)
    if kvd == rt.KV_F16:
        kc, vc = kc.astype(np.float16).astype(np.float32), vc.astype(np.float16).astype(np.float32)
    q = rng.normal(0, 1, (B, H * Dh)).astype(np.float32)
    kn = rng.normal(0, 1, (B, Hkv * Dh)).astype(np.float32)
    vn = rng.normal(0, 1, (B, Hkv * Dh)).astype(np.float32)
    poss = np.array([pos, max(pos // 2, 0)], np.int32)
    want = []
    for b in range(B):
        k2, v2 = kc[b].copy(), vc[b].copy()
        kr, vr = kn[b].reshape(Hkv, Dh), vn[b].reshape(Hkv, Dh)
        if kvd == rt.KV_F16:
            kr, vr = kr.astype(np.float16).astype(np.float32), vr.astype(np.float16).astype(np.float32)
        k2[:, poss[b]], v2[:, poss[b]] = kr, vr
        want.append(orc.attention(q[b], k2, v2, H, Hkv, Dh, S, int(poss[b])))
    want = np.stack(want)
    cdt = cuda.float16 if kvd == rt.KV_F16 else cuda.float32
    dk, dv = dev(cuda, kc).to(cdt), dev(cuda, vc).to(cdt)
    out = cuda.empty((B, H * Dh), dtype=cuda.float32, device="cuda")
    wsb = rt.lib().lmc_attention_workspace_bytes(B, H, Dh, S)
    ws = cuda.empty(max(wsb, 4), dtype=cuda.uint8, device="cuda")
    dq, dkn, dvn, dpos = dev(cuda, q), dev(cuda, kn), dev(cuda, vn), dev(cuda, poss)
    rt.call("lmc_attention_decode", out.data_ptr(), dq.data_ptr(), dkn.data_ptr(), dvn.data_ptr(), dk.data_ptr(),
            dv.data_ptr(), kvd, dpos.data_ptr(), B, H, Hkv, Dh, S, ws.data_ptr(), wsb, None)
    assert rel_err(out.cpu().numpy(), want) < 1e-5
    # the new row was appended to the cache
    assert np.allclose(dk[1, :, poss[1]].float().cpu().numpy().reshape(-1),
                       kn[1].astype(np.float16 if kvd == rt.KV_F16 else np.float32).astype(np.float32))


def q8_cache(orc, rows):
    """[..., Dh] fp32 rows -> (the int8-row cache bytes [..., Dh + 16], the
    values it holds as fp32)."""
    Dh = rows.shape[-1]
    flat = rows.reshape(-1, Dh)
    raw = np.zeros((flat.shape[0], Dh + 16), np.uint8)
    vals = np.empty_like(flat)
    for i, r in enumerate(flat):
        q, sc = orc.kv_q8_row(r)
        raw[i, :Dh] = q.view(np.uint8)
        raw[i, Dh:Dh + 4] = np.frombuffer(np.float32(sc).tobytes(), np.uint8)
        vals[i] = q.astype(np.float32) * np.float32(sc)
    return raw.reshape(rows.shape[:-1] + (Dh + 16,)), vals.reshape(rows.shape)


@pytest.mark.parametrize("H,Hkv,Dh,S,pos", [
    (12, 12, 64, 1024, 0), (12, 12, 64, 1024, 135), (32, 4, 64, 2048, 700), (32, 8, 128, 4096, 1500),
    (6, 2, 96, 256, 200)])
def test_attention_int8_rows(cuda, orc, H, Hkv, Dh, S, pos):
    """LMC_KV_Q8: rows of int8 codes and one fp32 scale.  The appended rows'
    codes and scales are the oracle's quantization bit for bit; the output
    is attention over the values the cache holds (rel-err 1e-5)."""
    rng = np.random.default_rng(pos + 7 * H)
    B = 2
    base = rng.normal(0, 1, (B, Hkv, S, Dh)).astype(np.float32)
    kraw, kvals = q8_cache(orc, base)
    vraw, vvals = q8_cache(orc, rng.normal(0, 1, (B, Hkv, S, Dh)).astype(np.float32))
    q = rng.normal(0, 1, (B, H * Dh)).astype(np.float32)
    kn = rng.normal(0, 1, (B, Hkv * Dh)).astype(np.float32)
    vn = rng.normal(0, 1, (B, Hkv * Dh)).astype(np.float32)
    kn[0, :Dh] = 0.0  # an all-zero row: scale 0, codes 0
    poss = np.array([pos, max(pos // 2, 0)], np.int32)
    want, knew = [], []
    for b in range(B):
        k2, v2 = kvals[b].copy(), vvals[b].copy()
        kq, kv_ = q8_cache(orc, kn[b].reshape(Hkv, Dh))
        vq, vv_ = q8_cache(orc, vn[b].reshape(Hkv, Dh))
        k2[:, poss[b]], v2[:, poss[b]] = kv_, vv_
        knew.append((kq, vq))
        want.append(orc.attention(q[b], k2, v2, H, Hkv, Dh, S, int(poss[b])))
    want = np.stack(want)
    dk, dv = dev(cuda, kraw), dev(cuda, vraw)
    out = cuda.empty((B, H * Dh), dtype=cuda.float32, device="cuda")
    wsb = rt.lib().lmc_attention_workspace_bytes(B, H, Dh, S)
    ws = cuda.empty(max(wsb, 4), dtype=cuda.uint8, device="cuda")
    dq, dkn, dvn, dpos = dev(cuda, q), dev(cuda, kn), dev(cuda, vn), dev(cuda, poss)
    rt.call("lmc_attention_decode", out.data_ptr(), dq.data_ptr(), dkn.data_ptr(), dvn.data_ptr(), dk.data_ptr(),
            dv.data_ptr(), rt.KV_Q8, dpos.data_ptr(), B, H, Hkv, Dh, S, ws.data_ptr(), wsb, None)
    assert rel_err(out.cpu().numpy(), want) < 1e-5
    kc, vc = dk.cpu().numpy(), dv.cpu().numpy()
    for b in range(B):
        assert (kc[b, :, poss[b], :Dh + 4] == knew[b][0][:, :Dh + 4]).all()
        assert (vc[b, :, poss[b], :Dh + 4] == knew[b][1][:, :Dh + 4]).all()
    assert rt.lib().lmc_device_status() == 0


@pytest.mark.parametrize("kvd", [rt.KV_F32, rt.KV_F16, rt.KV_Q8])
@pytest.mark.parametrize("H,Hkv,Dh,P,pos", [(12, 12, 64, 16, 135), (32, 4, 64, 64, 700), (32, 8, 128, 256, 1500),
                                           (8, 8, 64, 16, 0)])
def test_attention_paged(cuda, orc, kvd, H, Hkv, Dh, P, pos):
    """lmc_attention_decode_paged: the pages of two sequences scattered over
    a pool (in shuffled order) give the same output as the contiguous cache
    (the oracle on the rows the cache holds), and the new row lands in the
    page the table names."""
    rng = np.random.default_rng(pos + P)
    B, maxp = 2, (pos + P) // P + 1
    S = maxp * P
    npages = 2 * B * maxp + 3
    cont = rng.normal(0, 1, (B, Hkv, S, Dh)).astype(np.float32)
    vcont = rng.normal(0, 1, (B, Hkv, S, Dh)).astype(np.float32)
    if kvd == rt.KV_Q8:
        kraw, kvals = q8_cache(orc, cont)
        vraw, vvals = q8_cache(orc, vcont)
    else:
        dt = np.float16 if kvd == rt.KV_F16 else np.float32
        kraw, vraw = cont.astype(dt), vcont.astype(dt)
        kvals, vvals = kraw.astype(np.float32), vraw.astype(np.float32)
    RB = kraw.shape[-1]
    table = rng.permutation(npages)[:B * maxp].astype(np.int32).reshape(B, maxp)
    kpool = np.zeros((npages, Hkv, P, RB), kraw.dtype)
    vpool = np.zeros((npages, Hkv, P, RB), vraw.dtype)
    for b in range(B):
        for j in range(maxp):
            kpool[table[b, j]] = kraw[b, :, j * P:(j + 1) * P]
            vpool[table[b, j]] = vraw[b, :, j * P:(j + 1) * P]
    q = rng.normal(0, 1, (B, H * Dh)).astype(np.float32)
    kn = rng.normal(0, 1, (B, Hkv * Dh)).astype(np.float32)
    vn = rng.normal(0, 1, (B, Hkv * Dh)).astype(np.float32)
    poss = np.array([pos, max(pos // 3, 0)], np.int32)
    want = []
    for b in range(B):
        k2, v2 = kvals[b].copy(), vvals[b].copy()
        k2[:, poss[b]] = orc.kv_round_rows(kn[b].reshape(Hkv, Dh), kvd)
        v2[:, poss[b]] = orc.kv_round_rows(vn[b].reshape(Hkv, Dh), kvd)
        want.append(orc.attention(q[b], k2, v2, H, Hkv, Dh, S, int(poss[b])))
    want = np.stack(want)
    dk, dv, dt_ = dev(cuda, kpool), dev(cuda, vpool), dev(cuda, table)
    out = cuda.empty((B, H * Dh), dtype=cuda.float32, device="cuda")
    wsb = rt.lib().lmc_attention_workspace_bytes(B, H, Dh, S)
    ws = cuda.empty(max(wsb, 4), dtype=cuda.uint8, device="cuda")
    dq, dkn, dvn, dpos = dev(cuda, q), dev(cuda, kn), dev(cuda, vn), dev(cuda, poss)
    rt.call("lmc_attention_decode_paged", out.data_ptr(), dq.data_ptr(), dkn.data_ptr(), dvn.data_ptr(),
            dk.data_ptr(), dv.data_ptr(), kvd, npages, dt_.data_ptr(), maxp, P, dpos.data_ptr(), B, H, Hkv, Dh,
            ws.data_ptr(), wsb, None)
    assert rel_err(out.cpu().numpy(), want) < 1e-5
    kp = dk.cpu().numpy()
    for b in range(B):
        page, off = table[b, poss[b] // P], poss[b] % P
        got_row = kp[page, :, off]
        if kvd == rt.KV_Q8:
            got_vals = got_row[:, :Dh].view(np.int8).astype(np.float32) * got_row[:, Dh:Dh + 4].copy().view(np.float32)
        else:
            got_vals = got_row.astype(np.float32)
        assert np.array_equal(got_vals, orc.kv_round_rows(kn[b].reshape(Hkv, Dh), kvd))
    assert rt.lib().lmc_device_status() == 0


def test_softmax_edge_rows(cuda, orc):
    """Softmax rows as LMc's softmax (src/ops.c:31-43) treats them: masked
    entries (-inf) give 0, one element gives 1, a constant row is uniform,
    values near the float range do not overflow (the max is subtracted
    first).  LMc's sum < 1e-30 branch cannot be taken by finite rows (the
    maximum contributes e^0 = 1); the oracle restates it as written."""
    rows = [
        np.array([0.5, -np.inf, 2.0, -np.inf, -1.0], np.float32),
        np.array([7.0], np.float32),
        np.full(33, 3.25, np.float32),
        np.array([3e38, -3e38, 1e38, 0.0], np.float32),
        np.array([-1e30, -1e30 + 1e23, -1e30], np.float32),
    ]
    for r in rows:
        d = dev(cuda, r[None])
        rt.call("lmc_softmax", d.data_ptr(), r.size, 1, None)
        got = d.cpu().numpy()[0]
        want = orc.softmax(r)
        assert np.all(np.isfinite(got))
        assert np.allclose(got, want, rtol=1e-6, atol=1e-7), (r, got, want)
        assert abs(float(got.sum()) - 1.0) < 1e-5
