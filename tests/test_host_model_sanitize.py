"""The library's host runtime (lmc_b200/host/lmc_model.c) under
AddressSanitizer and UndefinedBehaviorSanitizer on a machine without a GPU:
tests/host_model_sanitize.c, linked with an instrumented build of
lmc_model.c and the library's CUDA objects, loads well-formed GGUF files
(the load stops at the first device allocation and must release
everything it took) and malformed ones (bad magic, truncated metadata or
tensor table, a wrapped tensor offset, no tensor data, arrays nested past
any real file, dimensions negative as ints, a missing file),
contiguous and paged; every call must end in a status code with no
out-of-bounds access, leak or undefined operation."""
import os
import struct
import subprocess

import pytest

from lmc_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
BUILD = os.path.join(ROOT, "lmc_b200", "_build")
SAN = ["-fsanitize=address,undefined", "-fno-sanitize-recover=all", "-fno-omit-frame-pointer"]


def test_host_runtime_is_clean_under_asan_and_ubsan(tmp_path):
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present: this checks the load paths that stop before the device")
    except ImportError:
        pass
    objs = [os.path.join(BUILD, f) for f in sorted(os.listdir(BUILD))] if os.path.isdir(BUILD) else []
    objs = [o for o in objs if o.endswith(".o") and not os.path.basename(o).startswith("host_")]
    if not objs:
        pytest.skip("library objects not built (make -C lmc_b200)")
    from tests.test_abi import _table_end, crafted_gguf_cases
    d = str(tmp_path)
    m_o, drv_o, exe = (os.path.join(d, n) for n in ("lmc_model.o", "drv.o", "drv"))
    cuda = "/usr/local/cuda"
    subprocess.check_call(["gcc", "-std=c99", "-O1", "-g"] + SAN + ["-I" + cuda + "/include", "-c",
                          os.path.join(ROOT, "lmc_b200", "host", "lmc_model.c"), "-o", m_o])
    subprocess.check_call(["gcc", "-std=c99", "-O1", "-g"] + SAN + ["-c", os.path.join(HERE, "host_model_sanitize.c"),
                                                                    "-o", drv_o])
    subprocess.check_call(["g++"] + SAN + ["-o", exe, drv_o, m_o] + objs +
                          ["-L" + cuda + "/lib64", "-lcudart", "-lnccl", "-lm", "-Wl,-rpath," + cuda + "/lib64"])
    good = [synth.make_llama(os.path.join(d, "ok.gguf"), L=1, D=64, H=4, Hkv=2, F=128, S=16, V=64, seed=1),
            synth.make_gpt2(os.path.join(d, "g.gguf"), L=1, D=64, H=4, S=16, V=64, seed=1)]
    raw = open(good[0], "rb").read()
    end, first_off = _table_end(raw)
    bad = {"magic": b"GGUX" + raw[4:], "meta": raw[:60], "table": raw[:end - 3], "nodata": raw[:end],
           "offset": raw[:first_off] + struct.pack("<Q", 2 ** 64 - 16) + raw[first_off + 8:],
           "cut": raw[:len(raw) // 2]}
    bad.update({name[:-5]: data for name, data, _, _ in crafted_gguf_cases()})
    paths = list(good)
    for k, v in bad.items():
        p = os.path.join(d, k + ".gguf")
        with open(p, "wb") as f:
            f.write(v)
        paths.append(p)
    paths.append(os.path.join(d, "missing.gguf"))
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1", UBSAN_OPTIONS="print_stacktrace=1")
    r = subprocess.run([exe] + paths, capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    codes = [int(ln.split()[0]) for ln in r.stdout.splitlines()]
    assert len(codes) == 2 * len(paths) + 1
    assert all(c < 0 for c in codes[:-1]) and codes[-1] == 0  # no device here: every load fails, cleanly
    out = r.stdout
    for word in (b"not a GGUF", b"truncated metadata", b"truncated tensor table", b"no tensor data",
                 b"data past end of file", b"cannot open", b"model dimension"):
        assert word.decode() in out, word
