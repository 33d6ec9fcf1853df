"""The CUDA block decoders (lmc_b200/csrc/lmc_blocks.cuh), compiled as host
C++ via tests/host_decoders.cpp, are bit-exact to the oracle for every format.
Runs without a GPU: it checks the decoder logic, not the device."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from lmc_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def hostlib(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("hd") / "hd.so")
    subprocess.check_call(["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-o", out,
                           os.path.join(HERE, "host_decoders.cpp")])
    L = ctypes.CDLL(out)
    L.host_decode8.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    return L


def decode(L, t, blk, n):
    out = np.empty(n, np.float32)
    assert L.host_decode8(t, blk.ctypes.data, out.ctypes.data, n) == 0
    return out


@pytest.mark.parametrize("t", synth.ALL_TYPES, ids=lambda t: synth.NAMES[t])
def test_decoder_bit_exact(hostlib, orc, t):
    be = max(synth.GEOMETRY[t][0], 8)
    for seed in range(3):
        n = be * 777
        blk = synth.random_blocks(t, n, seed=seed)
        a = orc.dequant(t, blk, n)
        b = decode(hostlib, t, blk, n)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), synth.NAMES[t]


def test_f16_all_patterns(hostlib, orc):
    """Every fp16 bit pattern (subnormals, Inf, NaN payloads) decodes like
    LMc's f16_to_f32 (quant.c:19-38)."""
    blk = np.concatenate([np.arange(65536, dtype=np.uint16).view(np.uint8), np.zeros(16, np.uint8)])
    a = orc.dequant(synth.F16, blk, 65536)
    b = decode(hostlib, synth.F16, blk, 65536)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
