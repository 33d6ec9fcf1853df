"""The C ABI library builds, loads and exports every entry point that
include/*.h declares; calls that need no GPU behave as documented."""
import ctypes
import os
import re
import subprocess

import pytest

from lmc_b200 import runtime as rt
from lmc_b200 import synth
from tests.conftest import ROOT


def declared_functions():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(lmc_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    assert os.path.exists(rt.LIB_PATH), "liblmc_b200.so not built"
    out = subprocess.check_output(["nm", "-D", "--defined-only", rt.LIB_PATH], text=True)
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    missing = declared_functions() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    assert len(declared_functions()) >= 25


def test_bindings_cover_header():
    assert declared_functions() <= set(rt.SIGNATURES) | {"lmc_model_graph_kernels"} | set(rt.SIGNATURES)


def test_block_geometry_matches_lmc_table():
    L = rt.lib()
    for t, (be, bb, _) in synth.GEOMETRY.items():
        e, b = ctypes.c_int(), ctypes.c_int()
        assert L.lmc_block_geometry(t, ctypes.byref(e), ctypes.byref(b)) == 0
        assert (e.value, b.value) == (be, bb)
    e, b = ctypes.c_int(), ctypes.c_int()
    assert L.lmc_block_geometry(9, ctypes.byref(e), ctypes.byref(b)) == -2  # Q8_1: not in LMc
    assert b"unsupported" in L.lmc_last_error()


def test_init_without_gpu_fails_loudly():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(rt.LmcError) as e:
        rt.init(0)
    assert e.value.code == -3


def test_model_load_errors_are_status_codes(tmp_path):
    h = ctypes.c_void_p()
    L = rt.lib()
    assert L.lmc_model_load(str(tmp_path / "missing.gguf").encode(), 1, 0, ctypes.byref(h)) == -5
    assert b"cannot open" in L.lmc_last_error()
    assert L.lmc_model_load(b"x", 0, 0, ctypes.byref(h)) == -1
