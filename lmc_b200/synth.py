"""Seeded synthetic GGUF data: random blocks, simple quantizers, GGUF writer.

No public model, dataset or benchmark is involved anywhere in this project:
every weight and token is drawn here from numpy's PCG64 generator
(`numpy.random.default_rng(seed)`), so the same seed gives the same bytes on
every host.  The GPU path and the CPU reference read the same files.

Block geometry and type IDs follow LMc src/quant.h:27-99.  The quantizers are
plain per-block absmax / min-max quantizers (LMc ships none: it only reads
GGUF files); parity is always checked on the dequantized bytes, so their
quality only matters for keeping activations in a sane range.
"""
import os
import struct

import numpy as np

F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, IQ3_XXS, IQ3_S, IQ4_XS = 10, 11, 12, 13, 14, 18, 21, 23

# type -> (elements per block, bytes per block, byte offsets of fp16 scales)
GEOMETRY = {
    F32: (1, 4, ()),
    F16: (1, 2, ()),
    Q4_0: (32, 18, (0,)),
    Q4_1: (32, 20, (0, 2)),
    Q5_0: (32, 22, (0,)),
    Q5_1: (32, 24, (0, 2)),
    Q8_0: (32, 34, (0,)),
    Q2_K: (256, 84, (80, 82)),
    Q3_K: (256, 110, (108,)),
    Q4_K: (256, 144, (0, 2)),
    Q5_K: (256, 176, (0, 2)),
    Q6_K: (256, 210, (208,)),
    IQ3_XXS: (256, 98, (0,)),
    IQ3_S: (256, 110, (0,)),
    IQ4_XS: (256, 136, (0,)),
}
NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0", Q5_1: "Q5_1",
         Q8_0: "Q8_0", Q2_K: "Q2_K", Q3_K: "Q3_K", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K",
         IQ3_XXS: "IQ3_XXS", IQ3_S: "IQ3_S", IQ4_XS: "IQ4_XS"}
BLOCK_TYPES = [Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, IQ3_XXS, IQ3_S, IQ4_XS]
ALL_TYPES = [F32, F16] + BLOCK_TYPES
# Bytes readable past the last block: IQ4_XS decoding reads 2 bytes of the
# next block (LMc quant.c:506,515), so every block buffer carries a pad.
PAD = 16


def tensor_bytes(t, n_elements):
    be, bb, _ = GEOMETRY[t]
    if n_elements % be:
        raise ValueError(f"{NAMES[t]}: {n_elements} elements is not a multiple of {be}")
    return n_elements // be * bb


def fp16_abs_normal(rng, n, std=1e-3):
    """fp16 bit patterns of |N(0, std)| (always finite)."""
    return np.abs(rng.normal(0.0, std, n)).astype(np.float16).view(np.uint16)


def random_blocks(t, n_elements, seed=0, scale_std=1e-3):
    """Uniform random codes with fp16 scales drawn as |N(0, scale_std)|.

    All fields other than the fp16 scales (codes, packed 6-bit sub-block
    scales and mins, high-bit masks, sign bytes, lattice indices) are uniform
    random bytes; F32/F16 tensors get N(0,1) values.  Returns a uint8 array
    of tensor_bytes(t, n) + PAD bytes (the pad is zero).
    """
    rng = np.random.default_rng(seed)
    if t == F32:
        return np.concatenate([rng.normal(0, 1, n_elements).astype(np.float32).view(np.uint8),
                               np.zeros(PAD, np.uint8)])
    if t == F16:
        return np.concatenate([rng.normal(0, 1, n_elements).astype(np.float16).view(np.uint8),
                               np.zeros(PAD, np.uint8)])
    be, bb, offs = GEOMETRY[t]
    nb = n_elements // be
    raw = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    for o in offs:
        raw[:, o:o + 2] = fp16_abs_normal(rng, nb, scale_std).view(np.uint8).reshape(nb, 2)
    return np.concatenate([raw.reshape(-1), np.zeros(PAD, np.uint8)])


# ---------------------------------------------------------------------------
# quantizers (fp32 -> blocks), vectorized over blocks
# ---------------------------------------------------------------------------
def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16)


def quantize_q8_0(w):
    w = np.asarray(w, np.float32).reshape(-1, 32)
    amax = np.abs(w).max(1)
    d = _f16(amax / 127.0)
    dd = d.astype(np.float32)
    inv = np.where(dd > 0, 1.0 / np.where(dd > 0, dd, 1), 0)
    q = np.clip(np.rint(w * inv[:, None]), -127, 127).astype(np.int8)
    out = np.empty((w.shape[0], 34), np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def _pack_k4_scales(sc, mn):
    """Inverse of LMc get_scale_min_k4 (quant.c:44-53): 8 six-bit (sc, m)
    pairs per block -> 12 bytes."""
    nb = sc.shape[0]
    s = np.zeros((nb, 12), np.uint8)
    for j in range(4):
        s[:, j] = (sc[:, j] & 63) | ((sc[:, j + 4] >> 4) << 6)
        s[:, j + 4] = (mn[:, j] & 63) | ((mn[:, j + 4] >> 4) << 6)
        s[:, j + 8] = (sc[:, j + 4] & 15) | ((mn[:, j + 4] & 15) << 4)
    return s


def quantize_q4_k(w):
    w = np.asarray(w, np.float32).reshape(-1, 8, 32)
    nb = w.shape[0]
    lo = np.minimum(w.min(2), 0.0)
    hi = w.max(2)
    scale = (hi - lo) / 15.0
    mins = -lo
    d = _f16(scale.max(1) / 63.0)
    dmin = _f16(mins.max(1) / 63.0)
    dd, dm = d.astype(np.float32), dmin.astype(np.float32)
    sc = np.clip(np.rint(scale / np.where(dd > 0, dd, 1)[:, None]), 0, 63).astype(np.uint8)
    mn = np.clip(np.rint(mins / np.where(dm > 0, dm, 1)[:, None]), 0, 63).astype(np.uint8)
    step = dd[:, None] * sc.astype(np.float32)
    off = dm[:, None] * mn.astype(np.float32)
    q = np.clip(np.rint((w + off[:, :, None]) / np.where(step > 0, step, 1)[:, :, None]), 0, 15).astype(np.uint8)
    out = np.empty((nb, 144), np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(-1, 2)
    out[:, 4:16] = _pack_k4_scales(sc, mn)
    q = q.reshape(nb, 4, 2, 32)  # (pair g, lo/hi, l)
    out[:, 16:] = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(nb, 128)
    return out.reshape(-1)


def quantize_q6_k(w):
    w = np.asarray(w, np.float32).reshape(-1, 16, 16)
    nb = w.shape[0]
    sub = np.abs(w).max(2) / 31.0
    d = _f16(sub.max(1) / 127.0)
    dd = d.astype(np.float32)
    sc = np.clip(np.rint(sub / np.where(dd > 0, dd, 1)[:, None]), -128, 127).astype(np.int8)
    step = dd[:, None] * sc.astype(np.float32)
    q = np.clip(np.rint(w / np.where(step != 0, step, 1)[:, :, None]), -32, 31).astype(np.int32) + 32
    q = q.reshape(nb, 2, 4, 32)  # (pass, k, l): element 128p + 32k + l
    q1, q2, q3, q4 = q[:, :, 0], q[:, :, 1], q[:, :, 2], q[:, :, 3]
    out = np.empty((nb, 210), np.uint8)
    ql = np.empty((nb, 2, 64), np.uint8)
    ql[:, :, :32] = (q1 & 15) | ((q3 & 15) << 4)
    ql[:, :, 32:] = (q2 & 15) | ((q4 & 15) << 4)
    qh = (q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6)
    out[:, 0:128] = ql.reshape(nb, 128)
    out[:, 128:192] = qh.astype(np.uint8).reshape(nb, 64)
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    return out.reshape(-1)


QUANTIZERS = {Q8_0: quantize_q8_0, Q4_K: quantize_q4_k, Q6_K: quantize_q6_k,
              F32: lambda w: np.asarray(w, np.float32).reshape(-1).view(np.uint8),
              F16: lambda w: np.asarray(w, np.float32).astype(np.float16).reshape(-1).view(np.uint8)}


# ---------------------------------------------------------------------------
# GGUF v3 writer (layout read by LMc gguf.c:114-353)
# ---------------------------------------------------------------------------
def _gguf_str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, arch, meta_u32, meta_f32, tensors):
    """tensors: list of (name, dims (innermost first), type, raw bytes).

    Tensor data starts at the 32-byte-aligned end of the header
    (gguf.c:285-287) and every tensor offset is 32-byte aligned.
    """
    hdr = bytearray()
    n_kv = 1 + len(meta_u32) + len(meta_f32)
    hdr += struct.pack("<IIQQ", 0x46554747, 3, len(tensors), n_kv)
    hdr += _gguf_str("general.architecture") + struct.pack("<I", 8) + _gguf_str(arch)
    for k, v in meta_u32.items():
        hdr += _gguf_str(k) + struct.pack("<II", 4, int(v))
    for k, v in meta_f32.items():
        hdr += _gguf_str(k) + struct.pack("<If", 6, float(v))
    offs, off = [], 0
    for name, dims, t, raw in tensors:
        offs.append(off)
        off += (len(raw) + 31) // 32 * 32
    for (name, dims, t, raw), o in zip(tensors, offs):
        hdr += _gguf_str(name) + struct.pack("<I", len(dims))
        hdr += b"".join(struct.pack("<Q", d) for d in dims)
        hdr += struct.pack("<IQ", t, o)
    pad = (-len(hdr)) % 32
    with open(path, "wb") as f:
        f.write(bytes(hdr) + b"\0" * pad)
        for (name, dims, t, raw), o in zip(tensors, offs):
            f.write(bytes(raw))
            f.write(b"\0" * ((-len(raw)) % 32))
    return path


def _q(t, w):
    be = GEOMETRY[t][0]
    if w.size % be:
        raise ValueError(f"{w.size} not a multiple of {be}")
    return QUANTIZERS[t](w)


def make_gpt2(path, L=12, D=768, H=12, S=1024, V=50257, F=None, seed=0,
              wtype=Q4_K, down_type=Q6_K, out_type=Q6_K, emb_type=Q6_K, std=0.02):
    """GPT-2-architecture GGUF: LayerNorm + GELU, learned positions, fused QKV.

    Weights are N(0, std) then quantized (attention and ffn_up in `wtype`,
    ffn_down in `down_type`, output in `out_type`, token embedding in
    `emb_type`); norms and biases fp32 (LN weights 1 + N(0, std), biases
    N(0, std)); position embedding F32 N(0, std).  output.weight is always
    written (LMc copies wte into lm_head before loading, gguf.c:302-304).
    """
    F = F or 4 * D
    rng = np.random.default_rng(seed)
    nrm = lambda *s: rng.normal(0.0, std, s).astype(np.float32)
    T = []
    T.append(("token_embd.weight", (D, V), emb_type, _q(emb_type, nrm(V, D))))
    T.append(("position_embd.weight", (D, S), F32, _q(F32, nrm(S, D))))
    for l in range(L):
        p = f"blk.{l}."
        T += [(p + "attn_norm.weight", (D,), F32, _q(F32, 1.0 + nrm(D))),
              (p + "attn_norm.bias", (D,), F32, _q(F32, nrm(D))),
              (p + "attn_qkv.weight", (D, 3 * D), wtype, _q(wtype, nrm(3 * D, D))),
              (p + "attn_qkv.bias", (3 * D,), F32, _q(F32, nrm(3 * D))),
              (p + "attn_output.weight", (D, D), wtype, _q(wtype, nrm(D, D))),
              (p + "attn_output.bias", (D,), F32, _q(F32, nrm(D))),
              (p + "ffn_norm.weight", (D,), F32, _q(F32, 1.0 + nrm(D))),
              (p + "ffn_norm.bias", (D,), F32, _q(F32, nrm(D))),
              (p + "ffn_up.weight", (D, F), wtype, _q(wtype, nrm(F, D))),
              (p + "ffn_up.bias", (F,), F32, _q(F32, nrm(F))),
              (p + "ffn_down.weight", (F, D), down_type, _q(down_type, nrm(D, F))),
              (p + "ffn_down.bias", (D,), F32, _q(F32, nrm(D)))]
    T += [("output_norm.weight", (D,), F32, _q(F32, 1.0 + nrm(D))),
          ("output_norm.bias", (D,), F32, _q(F32, nrm(D))),
          ("output.weight", (D, V), out_type, _q(out_type, nrm(V, D)))]
    meta = {"gpt2.block_count": L, "gpt2.attention.head_count": H, "gpt2.embedding_length": D,
            "gpt2.feed_forward_length": F, "gpt2.context_length": S, "gpt2.vocab_size": V}
    return write_gguf(path, "gpt2", meta, {}, T)


def make_llama(path, L=22, D=2048, H=32, Hkv=4, F=5632, S=2048, V=32000, theta=10000.0,
               eps=1e-5, seed=0, wtype=Q4_K, out_type=Q6_K, emb_type=Q6_K, std=0.02, blocks="quantized"):
    """LLaMA-architecture GGUF: RMSNorm, RoPE, GQA, SwiGLU; RMS weights
    1 + N(0, std).  blocks="quantized": matrices N(0, std) then quantized;
    blocks="random": matrices are random blocks (uniform codes, fp16 scales
    |N(0, 1e-3)|, as random_blocks) -- the same bytes per weight, written in
    seconds for the billion-parameter shapes used by the throughput runs."""
    rng = np.random.default_rng(seed)
    nrm = lambda *s: rng.normal(0.0, std, s).astype(np.float32)
    salt = [0]

    def mat(t, rows, cols):
        if blocks == "random":
            salt[0] += 1
            return random_blocks(t, rows * cols, seed=seed * 7919 + salt[0])[:tensor_bytes(t, rows * cols)]
        return _q(t, nrm(rows, cols))

    Dh = D // H
    T = [("token_embd.weight", (D, V), emb_type, mat(emb_type, V, D))]
    for l in range(L):
        p = f"blk.{l}."
        T += [(p + "attn_norm.weight", (D,), F32, _q(F32, 1.0 + nrm(D))),
              (p + "attn_q.weight", (D, H * Dh), wtype, mat(wtype, H * Dh, D)),
              (p + "attn_k.weight", (D, Hkv * Dh), wtype, mat(wtype, Hkv * Dh, D)),
              (p + "attn_v.weight", (D, Hkv * Dh), wtype, mat(wtype, Hkv * Dh, D)),
              (p + "attn_output.weight", (D, D), wtype, mat(wtype, D, D)),
              (p + "ffn_norm.weight", (D,), F32, _q(F32, 1.0 + nrm(D))),
              (p + "ffn_gate.weight", (D, F), wtype, mat(wtype, F, D)),
              (p + "ffn_up.weight", (D, F), wtype, mat(wtype, F, D)),
              (p + "ffn_down.weight", (F, D), wtype, mat(wtype, D, F))]
    T += [("output_norm.weight", (D,), F32, _q(F32, 1.0 + nrm(D))),
          ("output.weight", (D, V), out_type, mat(out_type, V, D))]
    meta = {"llama.block_count": L, "llama.attention.head_count": H, "llama.attention.head_count_kv": Hkv,
            "llama.embedding_length": D, "llama.feed_forward_length": F, "llama.context_length": S,
            "llama.vocab_size": V}
    return write_gguf(path, "llama", meta, {"llama.rope.freq_base": theta,
                                            "llama.attention.layer_norm_rms_epsilon": eps}, T)


def cached_model(kind, directory, **kw):
    """Write (once) and return the path of a synthetic model file."""
    key = "_".join(f"{k}{v}" for k, v in sorted(kw.items()))
    path = os.path.join(directory, f"{kind}_{key}.gguf")
    if not os.path.exists(path):
        os.makedirs(directory, exist_ok=True)
        tmp = path + ".tmp"
        (make_gpt2 if kind == "gpt2" else make_llama)(tmp, **kw)
        os.replace(tmp, path)
    return path
