"""The latency GEMV's unit bodies (lmc_b200/csrc/ff_unit.cuh), compiled as
host C++ via tests/host_ff_unit.cpp, against the oracle: the tiled layout
restated here from its description (16 rows x 256 columns per unit, block
headers first, code words interleaved by lane), the units dotted with fp32
activations the way each lane of the kernel does, and the sums within
rel-err 1e-5 of LMc's dequantize-then-dot for Q4_K, Q6_K and Q8_0 at batch
1 and 2, with ragged row tiles (rows beyond the matrix are zero).  Runs
without a GPU: it checks the arithmetic (codes as 1 + q/16 or 1 + q/64
floats, the sum of x taken out once per chunk), not the device."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from lmc_b200 import synth
from tests.conftest import rel_err

HERE = os.path.dirname(os.path.abspath(__file__))
UNIT = {synth.Q4_K: 2304, synth.Q6_K: 3360, synth.Q8_0: 4352}
QT = {synth.Q4_K: 4, synth.Q6_K: 6, synth.Q8_0: 8}


@pytest.fixture(scope="module")
def hostlib(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("hff") / "hff.so")
    subprocess.check_call(["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fno-strict-aliasing", "-fPIC",
                           "-shared", "-o", out, os.path.join(HERE, "host_ff_unit.cpp")])
    L = ctypes.CDLL(out)
    L.host_ff_gemv.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                               ctypes.c_int, ctypes.c_void_p]
    return L


def code_word(n, t):
    """u32 index of lane t's code word n: 16-byte word n / 4 of 32 lanes."""
    return ((n >> 2) * 32 + t) * 4 + (n & 3)


def q4k_code(blk, k):  # src/quant.c:293: 64-weight groups, low nibbles then high
    g, w = k >> 6, k & 63
    b = int(blk[16 + 32 * g + (w & 31)])
    return b >> 4 if w & 32 else b & 15


def q6k_code(blk, k):  # src/quant.c:403-406: 4 low bits from ql, 2 high from qh
    p, r = k >> 7, k & 127
    kk, l = r >> 5, r & 31
    lo = (int(blk[64 * p + (32 if kk & 1 else 0) + l]) >> ((kk >> 1) * 4)) & 15
    hi = (int(blk[128 + 32 * p + l]) >> (2 * kk)) & 3
    return lo | hi << 4


def tile(t, blocks, M, K):
    """The tiled copy of a row-major matrix of GGUF blocks: RT x KB units."""
    KB, RT, U = K // 256, (M + 15) // 16, UNIT[t]
    out = np.zeros(RT * KB * U, np.uint8)
    be = 32 if t == synth.Q8_0 else 256  # weights per block
    bb = synth.tensor_bytes(t, be)
    per_row = (K // be) * bb

    def block(r, i):  # block i of row r (Q8_0: blocks of 32)
        if r >= M:
            return None
        o = r * per_row + i * bb
        return blocks[o:o + bb]

    for rt in range(RT):
        for kb in range(KB):
            u = out[(rt * KB + kb) * U:(rt * KB + kb + 1) * U]
            w32 = np.zeros((U - 256) // 4 if t != synth.Q6_K else (U - 288) // 4, np.uint32)
            if t == synth.Q4_K:
                for r in range(16):
                    b = block(rt * 16 + r, kb)
                    if b is not None:
                        u[16 * r:16 * r + 16] = b[:16]  # d, dmin, 12 scale / min bytes
                for lane in range(32):
                    g, c = lane >> 2, lane & 3
                    b0, b1 = block(rt * 16 + g, kb), block(rt * 16 + g + 8, kb)
                    for j in range(8):
                        p = q = 0
                        for i in range(4):
                            k0 = 32 * j + 4 * c + i
                            if b0 is not None:
                                p |= (q4k_code(b0, k0) | q4k_code(b0, k0 + 16) << 4) << (8 * i)
                            if b1 is not None:
                                q |= (q4k_code(b1, k0) | q4k_code(b1, k0 + 16) << 4) << (8 * i)
                        w32[code_word(2 * j, lane)] = p
                        w32[code_word(2 * j + 1, lane)] = q
                u[256:] = w32.view(np.uint8)
            elif t == synth.Q6_K:
                for r in range(16):
                    b = block(rt * 16 + r, kb)
                    if b is not None:
                        u[16 * r:16 * r + 16] = b[192:208]  # int8 scales
                        u[256 + 2 * r:256 + 2 * r + 2] = b[208:210]  # d
                lo = np.zeros(512, np.uint32)
                hi = np.zeros(256, np.uint32)
                for lane in range(32):
                    g, c = lane >> 2, lane & 3
                    b0, b1 = block(rt * 16 + g, kb), block(rt * 16 + g + 8, kb)
                    code0 = (lambda k: q6k_code(b0, k)) if b0 is not None else (lambda k: 0)
                    code1 = (lambda k: q6k_code(b1, k)) if b1 is not None else (lambda k: 0)
                    for j in range(16):
                        p = 0
                        for i in range(4):
                            k = 16 * j + 4 * c + i
                            p |= ((code0(k) & 15) | (code1(k) & 15) << 4) << (8 * i)
                        lo[code_word(j, lane)] = p
                    for jp in range(8):
                        h = 0
                        for i in range(4):
                            k = 32 * jp + 4 * c + i
                            h |= ((code0(k) >> 4) | (code1(k) >> 4) << 2 | (code0(k + 16) >> 4) << 4
                                  | (code1(k + 16) >> 4) << 6) << (8 * i)
                        hi[code_word(jp, lane)] = h
                u[288:288 + 2048] = lo.view(np.uint8)
                u[288 + 2048:] = hi.view(np.uint8)
            else:
                for r in range(16):
                    for j in range(8):
                        b = block(rt * 16 + r, kb * 8 + j)
                        if b is not None:
                            u[16 * r + 2 * j:16 * r + 2 * j + 2] = b[:2]  # d of block j
                for lane in range(32):
                    g, c = lane >> 2, lane & 3
                    for j in range(8):
                        b0, b1 = block(rt * 16 + g, kb * 8 + j), block(rt * 16 + g + 8, kb * 8 + j)
                        for i in range(4):
                            w = 0
                            src = [(b0, 4 * c), (b1, 4 * c), (b0, 16 + 4 * c), (b1, 16 + 4 * c)][i]
                            if src[0] is not None:
                                codes = src[0][2:]
                                for e in range(4):
                                    w |= int(codes[src[1] + e]) << (8 * e)
                            w32[(j * 32 + lane) * 4 + i] = w
                u[256:] = w32.view(np.uint8)
    return out


@pytest.mark.parametrize("t", [synth.Q4_K, synth.Q6_K, synth.Q8_0], ids=lambda t: synth.NAMES[t])
@pytest.mark.parametrize("nb", [1, 2])
def test_unit_bodies_match_the_oracle(hostlib, orc, t, nb):
    M, K = 40, 512  # three row tiles, the last one half empty
    blocks = synth.random_blocks(t, M * K, seed=7)
    W = orc.dequant(t, blocks, M * K).reshape(M, K).astype(np.float64)
    x = np.random.default_rng(3).normal(0, 1, (nb, K)).astype(np.float32)
    units = tile(t, blocks, M, K)
    RT = (M + 15) // 16
    y = np.zeros((nb, RT * 16), np.float32)
    assert hostlib.host_ff_gemv(QT[t], units.ctypes.data, RT, K // 256, x.ctypes.data, nb, y.ctypes.data) == 0
    want = x.astype(np.float64) @ W.T
    for b in range(nb):
        # the bodies round near 2^-24 per term (1-3e-7 here): 1e-5, a hundredth
        # of the 1e-3 bar, still catches a single misplaced code word (~1e-2)
        assert rel_err(y[b, :M], want[b]) < 1e-5
        assert not y[b, M:].any()  # rows past the matrix stay zero
