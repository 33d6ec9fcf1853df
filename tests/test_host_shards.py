"""The tensor-parallel shard loader of lmc_b200/host/lmc_model.c, run on the
CPU: the loader is linked with host stand-ins for the device side
(tests/host_shard_fakes.c) that write every uploaded block stream to a file.
For 1, 2, 4 and 8 ranks, every rank's uploads must be exactly the bytes cut
here from the GGUF file by the tensor-parallel layout: q/k/v rows by heads,
gate/up rows and ffn_down columns by ffn rows, attn_output columns by heads,
lm_head rows by ceil(V/N), the embedding whole; and the ranks' shards of each
tensor must put the whole tensor back together.  Built again under ASan and
UBSan, whole loads and frees must be clean, and the paged cache's page pool
must count as forward calls take pages and sequences give them back."""
import os
import struct
import subprocess

import numpy as np
import pytest

from lmc_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CUDA_INC = "/usr/local/cuda/include"
GEOM = {synth.Q4_K: (256, 144), synth.Q6_K: (256, 210), synth.Q8_0: (32, 34), synth.F32: (1, 4)}


def tensors(raw):
    """name -> (dims innermost first, type, absolute byte offset) of a GGUF v3
    file with u32 / f32 / string metadata (what synth writes)."""
    n_t, n_kv = struct.unpack_from("<QQ", raw, 8)
    p = 24
    for _ in range(n_kv):
        p += 8 + struct.unpack_from("<Q", raw, p)[0]
        typ = struct.unpack_from("<I", raw, p)[0]
        p += 4
        p += 8 + struct.unpack_from("<Q", raw, p)[0] if typ == 8 else 4
    out = []
    for _ in range(n_t):
        nl = struct.unpack_from("<Q", raw, p)[0]
        name = raw[p + 8:p + 8 + nl].decode()
        p += 8 + nl
        nd = struct.unpack_from("<I", raw, p)[0]
        dims = struct.unpack_from("<%dQ" % nd, raw, p + 4)
        p += 4 + 8 * nd
        t, off = struct.unpack_from("<IQ", raw, p)
        p += 12
        out.append((name, dims, t, off))
    data = (p + 31) // 32 * 32
    return [(n, d, t, data + o) for n, d, t, o in out]


def row_bytes(t, cols):
    be, bb = GEOM[t]
    assert cols % be == 0
    return cols // be * bb


def expected(raw, cfg, rank, n):
    """The block streams rank `rank` of `n` uploads, in file order."""
    D, H, Hkv, F, V = cfg["D"], cfg["H"], cfg["Hkv"], cfg["F"], cfg["V"]
    Dh = D // H
    hl, hkvl, fl = H // n, Hkv // n, F // n
    vr = -(-V // n)
    v0 = rank * vr
    vl = min(vr, V - v0)
    out = []
    for name, dims, t, off in tensors(raw):
        if t == synth.F32:
            continue  # vectors are copied whole (no qtensor)
        cols, rows = dims[0], dims[1]
        rb = row_bytes(t, cols)
        whole = raw[off:off + rows * rb]

        def rows_of(r0, nr):
            return whole[r0 * rb:(r0 + nr) * rb]

        def cols_of(c0, nc):
            a, b = row_bytes(t, c0) if c0 else 0, row_bytes(t, nc)
            return b"".join(whole[i * rb + a:i * rb + a + b] for i in range(rows))

        kind = name.split(".")[-2]
        if n == 1 or name == "token_embd.weight":
            out.append((name, whole))
        elif name == "output.weight":
            out.append((name, rows_of(v0, vl)))
        elif kind == "attn_q":
            out.append((name, rows_of(rank * hl * Dh, hl * Dh)))
        elif kind in ("attn_k", "attn_v"):
            out.append((name, rows_of(rank * hkvl * Dh, hkvl * Dh)))
        elif kind == "attn_output":
            out.append((name, cols_of(rank * hl * Dh, hl * Dh)))
        elif kind in ("ffn_gate", "ffn_up"):
            out.append((name, rows_of(rank * fl, fl)))
        elif kind == "ffn_down":
            out.append((name, cols_of(rank * fl, fl)))
        else:
            raise AssertionError(name)
    return out


SAN = ["-fsanitize=address,undefined", "-fno-sanitize-recover=all", "-fno-omit-frame-pointer"]


def build_loader(d, extra=()):
    if not os.path.isdir(CUDA_INC):
        pytest.skip("CUDA headers not present")
    layout = d / "layout.c"
    layout.write_text('#include <stddef.h>\n#include "%s"\n'
                      "const size_t qt_layout[5] = {offsetof(struct lmc_qtensor, rows), "
                      "offsetof(struct lmc_qtensor, bytes), offsetof(struct lmc_qtensor, tiled), "
                      "offsetof(struct lmc_qtensor, gemm_wscale), sizeof(struct lmc_qtensor)};\n"
                      % os.path.join(ROOT, "lmc_b200", "csrc", "lmc_internal.h"))
    exe = str(d / "loader")
    subprocess.check_call(["gcc", "-std=gnu99", "-O1", "-g", "-w", "-I" + CUDA_INC] + list(extra) + ["-o", exe,
                           os.path.join(ROOT, "lmc_b200", "host", "lmc_model.c"),
                           os.path.join(HERE, "host_shard_fakes.c"), str(layout), "-lm"])
    return exe


@pytest.fixture(scope="module")
def loader(tmp_path_factory):
    return build_loader(tmp_path_factory.mktemp("shards"))


@pytest.fixture(scope="module")
def loader_san(tmp_path_factory):
    """The same loader under AddressSanitizer (leaks included) and
    UndefinedBehaviorSanitizer."""
    return build_loader(tmp_path_factory.mktemp("shards_san"), SAN)


def run(exe, args, **env):
    e = dict(os.environ, LMC_TP_PEER="0", ASAN_OPTIONS="detect_leaks=1", UBSAN_OPTIONS="print_stacktrace=1", **env)
    r = subprocess.run([exe] + args, capture_output=True, text=True, env=e, timeout=300)
    assert r.returncode == 0, (r.stdout[-1000:] + r.stderr[-3000:])
    return r.stdout


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_shard_loader_uploads_the_tensor_parallel_layout(loader, tmp_path, n):
    # width 2048: every rank's attn_output / ffn_down columns start on a
    # 256-weight block at 8 ranks; vocabulary 70 leaves the last lm_head
    # shard short (ceil(70 / 8) = 9 rows, the last rank 7)
    cfg = dict(L=2, D=2048, H=16, Hkv=8, F=2048, S=16, V=70, seed=3)
    path = synth.make_llama(str(tmp_path / "m.gguf"), **cfg)
    raw = open(path, "rb").read()
    dump = tmp_path / "dump"
    dump.mkdir()
    env = dict(os.environ, LMC_TP_PEER="0", LMC_FAKE_DUMP=str(dump))
    r = subprocess.run([loader, path, str(n)], capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    ranks, cur = [], None
    for ln in r.stdout.splitlines():
        f = ln.split()
        if f[0] == "R":
            cur = []
            ranks.append(cur)
        elif f[0] == "rc":
            assert f[1] == "0", ln
        elif f[0] == "Q":
            cur.append((int(f[1]), int(f[3]), int(f[4])))
    assert len(ranks) == n
    per_tensor = {}
    for rank, got in enumerate(ranks):
        want = expected(raw, cfg, rank, n)
        assert len(got) == len(want), (rank, len(got), len(want))
        for (seq, rows, cols), (name, data) in zip(got, want):
            blob = (dump / ("%04d.bin" % seq)).read_bytes()
            assert blob == data, (rank, name)
            per_tensor.setdefault(name, []).append((rows, cols, blob))
    # the shards put each tensor back together
    for name, dims, t, off in tensors(raw):
        if t == synth.F32:
            continue
        cols, rows = dims[0], dims[1]
        rb = row_bytes(t, cols)
        whole = np.frombuffer(raw[off:off + rows * rb], np.uint8).reshape(rows, rb)
        parts = per_tensor[name]
        if n == 1 or name == "token_embd.weight":
            assert all(p[2] == whole.tobytes() for p in parts)
        elif parts[0][1] == cols:  # row shards
            assert b"".join(p[2] for p in parts) == whole.tobytes(), name
        else:  # column shards
            back = np.concatenate([np.frombuffer(p[2], np.uint8).reshape(rows, -1) for p in parts], axis=1)
            assert back.tobytes() == whole.tobytes(), name


def test_whole_load_and_free_are_clean_under_asan(loader_san, tmp_path):
    """Every host allocation of a load (tables, staging, the fused
    q|k|v and gate|up tensors, the RoPE table, the tensor-parallel geometry)
    released by lmc_model_free, nothing read or written out of bounds."""
    gp = synth.make_gpt2(str(tmp_path / "g.gguf"), L=2, D=256, H=4, S=32, V=100, seed=1)
    lp = synth.make_llama(str(tmp_path / "l.gguf"), L=2, D=512, H=8, Hkv=4, F=512, S=32, V=64, seed=1)
    for path, n in ((gp, 1), (lp, 1), (lp, 2)):
        out = run(loader_san, [path, str(n)])
        assert out.count("rc 0") == n, out[-500:]


def test_paged_cache_page_accounting(loader_san, tmp_path):
    """The paged cache's pool as forward calls take pages and sequences give
    them back (each forward stops at its first kernel launch, after taking its
    pages): all-or-nothing refusal when the pool is short, release returns
    every page, a bad sequence is refused; clean under the sanitizers."""
    path = synth.make_llama(str(tmp_path / "p.gguf"), L=1, D=64, H=4, Hkv=2, F=128, S=64, V=64, seed=1)
    out = run(loader_san, [path, "1", "paged"])
    steps = [tuple(int(v) for v in ln.split()[1:]) for ln in out.splitlines() if ln.startswith("P ")]
    launch, ok, oom, invalid = -2, 0, -4, -1
    assert steps == [(launch, 4), (launch, 2), (ok, 5), (launch, 2), (oom, 2), (launch, 1), (ok, 4), (invalid, 4)]


def test_model_entry_points_refuse_bad_arguments(loader_san, tmp_path):
    """lmc_model_forward / _prefill / _generate / _replay on a loaded model
    refuse negative or out-of-range positions, tokens and sequences, and
    sizes whose sum would overflow an int (the checks are written without
    the sum; UBSan would stop the run on a signed overflow)."""
    path = synth.make_llama(str(tmp_path / "a.gguf"), L=1, D=64, H=4, Hkv=2, F=128, S=64, V=64, seed=1)
    out = run(loader_san, [path, "1", "args"])
    codes = [int(ln.split()[1]) for ln in out.splitlines() if ln.startswith("A ")]
    assert codes == [-1] * 9, out[-800:]
