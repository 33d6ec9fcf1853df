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


def _load_status(path, tp_rank=0, tp_size=1):
    h = ctypes.c_void_p()
    nid = ctypes.create_string_buffer(128)
    rc = rt.lib().lmc_model_load_ex(str(path).encode(), 1, 1, 0, tp_rank, tp_size,
                                    ctypes.cast(nid, ctypes.c_void_p) if tp_size > 1 else None, ctypes.byref(h))
    return rc, rt.lib().lmc_last_error()


def _table_end(raw):
    """(end of the tensor table, position of the first tensor's offset field)
    in a GGUF v3 file with u32 / f32 / string metadata (what synth writes)."""
    import struct
    n_t, n_kv = struct.unpack_from("<QQ", raw, 8)
    p = 24
    for _ in range(n_kv):
        p += 8 + struct.unpack_from("<Q", raw, p)[0]  # key
        typ = struct.unpack_from("<I", raw, p)[0]
        p += 4
        p += 8 + struct.unpack_from("<Q", raw, p)[0] if typ == 8 else 4
    first_off = None
    for _ in range(n_t):
        p += 8 + struct.unpack_from("<Q", raw, p)[0]  # name
        nd = struct.unpack_from("<I", raw, p)[0]
        p += 4 + 8 * nd + 4
        first_off = p if first_off is None else first_off
        p += 8
    return p, first_off


def _gguf_kv(key, typ, payload):
    import struct
    k = key.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<I", typ) + payload


def _gguf(kvs):
    """A GGUF v3 file with no tensors and the given encoded metadata pairs."""
    import struct
    return struct.pack("<IIQQ", 0x46554747, 3, 0, len(kvs)) + b"".join(kvs)


def crafted_gguf_cases():
    """(name, bytes, status, message) of metadata a crafted file can hold:
    arrays nested 200000 deep (a reader that recurses per level runs out of
    stack) and dimensions that are negative as ints (2^31 / -1 traps)."""
    import struct
    deep = struct.pack("<IQ", 9, 1) * 200000 + struct.pack("<IQ", 4, 0)
    u32 = lambda v: struct.pack("<I", v)
    arch = _gguf_kv("general.architecture", 8, struct.pack("<Q", 5) + b"llama")
    return [
        ("nested.gguf", _gguf([_gguf_kv("x.nested", 9, deep)]), -5, b"truncated metadata"),
        ("negdim.gguf", _gguf([arch, _gguf_kv("llama.block_count", 4, u32(1)),
                               _gguf_kv("llama.embedding_length", 4, u32(2 ** 31)),
                               _gguf_kv("llama.attention.head_count", 4, u32(2 ** 32 - 1))]),
         -5, b"model dimension"),
        ("hugedim.gguf", _gguf([arch, _gguf_kv("llama.block_count", 4, u32(1)),
                                _gguf_kv("llama.embedding_length", 4, u32(1 << 30)),
                                _gguf_kv("llama.attention.head_count", 4, u32(4))]),
         -5, b"model dimension"),
    ]


def test_model_load_rejects_crafted_metadata(tmp_path):
    """Metadata no real file has is refused with a status code, not a
    crash: arrays nested beyond any real file, dimensions that are negative
    or absurdly large as the reader's ints."""
    for name, data, code, word in crafted_gguf_cases():
        p = tmp_path / name
        p.write_bytes(data)
        rc, msg = _load_status(p)
        assert rc == code and word in msg, (name, rc, msg)


def test_model_load_rejects_malformed_gguf(tmp_path):
    """Malformed GGUF headers are reported as status codes with a message
    (the header is parsed before anything is uploaded, so no GPU is needed):
    bad magic, unknown version, truncated metadata, truncated tensor table,
    missing block/head/width keys, heads not a multiple of kv heads."""
    import struct
    from lmc_b200 import synth
    good = synth.make_llama(str(tmp_path / "ok.gguf"), L=1, D=64, H=4, Hkv=2, F=128, S=16, V=64, seed=1)
    raw = open(good, "rb").read()

    def case(name, data):
        p = tmp_path / name
        p.write_bytes(data)
        return _load_status(p)

    rc, msg = case("magic.gguf", b"GGUX" + raw[4:])
    assert rc == -5 and b"not a GGUF v1-3 file" in msg
    rc, msg = case("ver.gguf", raw[:4] + struct.pack("<I", 7) + raw[8:])
    assert rc == -5 and b"not a GGUF v1-3 file" in msg
    rc, msg = case("meta.gguf", raw[:60])
    assert rc == -5 and b"truncated metadata" in msg
    # header only: metadata intact, the tensor table cut in its first entry
    hdr_end = raw.index(b"token_embd.weight") + 8
    rc, msg = case("table.gguf", raw[:hdr_end])
    assert rc == -5 and b"truncated tensor table" in msg
    # a crafted tensor offset (2^64 - 16: offset + size wraps around) and a
    # file that ends at its tensor table (the aligned data start lies past
    # the end): refused before anything is read or uploaded
    end, first_off = _table_end(raw)
    rc, msg = case("offset.gguf", raw[:first_off] + struct.pack("<Q", 2 ** 64 - 16) + raw[first_off + 8:])
    assert rc == -5 and b"data past end of file" in msg
    assert end % 32, "the header must not end on the data alignment for this case"
    rc, msg = case("nodata.gguf", raw[:end])
    assert rc == -5 and b"no tensor data after the header" in msg
    p = synth.write_gguf(str(tmp_path / "nokeys.gguf"), "llama", {"llama.block_count": 1}, {}, [])
    rc, msg = _load_status(p)
    assert rc == -5 and b"missing L/H/D metadata" in msg
    p = synth.write_gguf(str(tmp_path / "kv.gguf"), "llama",
                         {"llama.block_count": 1, "llama.attention.head_count": 6, "llama.embedding_length": 96,
                          "llama.attention.head_count_kv": 4}, {}, [])
    rc, msg = _load_status(p)
    assert rc == -5 and b"not a multiple of kv heads" in msg


def test_model_load_rejects_unshardable_tensor_parallel(tmp_path):
    """Tensor parallel is for LLaMA models whose heads, kv heads and ffn rows
    divide by the group size; other requests fail before any upload."""
    from lmc_b200 import synth
    g = synth.make_gpt2(str(tmp_path / "g.gguf"), L=1, D=64, H=4, S=16, V=64, seed=1)
    rc, msg = _load_status(g, 0, 2)
    assert rc == -2 and b"LLaMA models only" in msg
    p = synth.make_llama(str(tmp_path / "l.gguf"), L=1, D=96, H=6, Hkv=3, F=192, S=16, V=64, seed=1)
    rc, msg = _load_status(p, 0, 2)
    assert rc == -2 and b"not divisible by 2" in msg
    rc, msg = _load_status(p, 2, 2)
    assert rc == -1 and b"shard 2 of 2" in msg


def test_entry_points_validate_arguments_first():
    """Every entry point checks its arguments before it touches the device:
    null pointers, sizes that are not whole blocks, empty shapes and
    oversized requests come back as LMC_ERR_INVALID with a message, the way
    LMc's LMC_FATAL checks fire before any work."""
    L = rt.lib()
    p = ctypes.c_void_p(256)  # never dereferenced: the checks fail first
    calls = [
        ("lmc_dequant", (12, None, 256, None, None), b"null"),
        ("lmc_dequant", (12, p, 300, p, None), b"not a multiple of 256"),
        ("lmc_qtensor_upload", (12, 0, 256, None, 0, None), b"args"),
        ("lmc_layer_norm", (None, None, None, None, 768, 1, None), b"args"),
        ("lmc_rms_norm", (None, None, None, 768, 1, 1e-5, None), b"args"),
        ("lmc_softmax", (None, 10, 1, None), b"args"),
        ("lmc_argmax", (None, 10, 1, None, None), b"args"),
        ("lmc_gelu", (None, 10, None), b"null"),
        ("lmc_model_forward", (None, None, None, 1, None, None), b"args"),
        ("lmc_model_generate", (None, None, 1, 1, 1, 0, None), b"args"),
        ("lmc_model_prefill", (None, 0, None, 1, 0, None, None), b"sequence"),
        # 64 sequences x 32 heads x 128 dims over 32768 positions: the
        # split-context scratch exceeds the fixed array
        ("lmc_attention_decode_noalloc", (p, p, p, p, p, p, 0, p, 64, 32, 8, 128, 32768, None), b"attention_noalloc"),
        # null pointers and H not a multiple of Hkv: rejected before the
        # entry point looks up its scratch array (a CUDA call)
        ("lmc_attention_decode_noalloc", (None, p, p, p, p, p, 0, p, 1, 32, 8, 128, 1024, None), b"null"),
        ("lmc_attention_decode_noalloc", (p, p, p, p, p, None, 0, p, 1, 32, 8, 128, 1024, None), b"null"),
        ("lmc_attention_decode_noalloc", (p, p, p, p, p, p, 0, p, 1, 30, 8, 128, 1024, None), b"Hkv=8"),
        # paged cache: a page size that is not a power of two, an empty pool
        ("lmc_attention_decode_paged", (p, p, p, p, p, p, 0, 8, p, 4, 24, p, 1, 32, 8, 128, p, 0, None),
         b"attention_paged"),
        ("lmc_attention_decode_paged", (p, p, p, p, p, p, 0, 0, p, 4, 64, p, 1, 32, 8, 128, p, 0, None),
         b"attention_paged"),
        # paged model cache: page size 24 (not a power of two), 8 (below
        # 16), no pages; checked before the file is opened
        ("lmc_model_load_paged", (b"x.gguf", 1, 1, 0, 24, 4, 0, 1, None, ctypes.byref(ctypes.c_void_p())),
         b"KV pages"),
        ("lmc_model_load_paged", (b"x.gguf", 1, 1, 0, 8, 4, 0, 1, None, ctypes.byref(ctypes.c_void_p())),
         b"KV pages"),
        ("lmc_model_load_paged", (b"x.gguf", 1, 1, 0, 16, 0, 0, 1, None, ctypes.byref(ctypes.c_void_p())),
         b"KV pages"),
        ("lmc_model_load_paged", (b"x.gguf", 1, 1, 0, 0, 4, 0, 1, None, ctypes.byref(ctypes.c_void_p())),
         b"page size"),
        ("lmc_model_release_seq", (None, 0), b"release_seq"),
        ("lmc_model_kv_pages", (None, None, None, None), b"kv_pages"),
        ("lmc_set_wait_limit", (ctypes.c_longlong(-5),), b"set_wait_limit"),
        ("lmc_wait_selftest", (7,), b"wait_selftest"),
        ("lmc_sample_top_p", (None, 10, 1, 1.0, 0.9, None, None, None), b"sample_top_p"),
    ]
    for name, args, word in calls:
        rc = getattr(L, name)(*args)
        assert rc == -1, (name, rc)
        assert word in L.lmc_last_error(), (name, L.lmc_last_error())
    assert L.lmc_model_free(None) == 0 and L.lmc_qtensor_free(None) == 0
