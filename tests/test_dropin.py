"""The ops.h drop-in layer (include/lmc_ops.h, lmc_b200/dropin/lmc_ops.c).

One LMc-side program (lmc_b200/dropin/example_main.c, written against LMc's
headers only) is linked twice: with LMc's own gguf.c / ops.c / ops_llama.c
(oracle/_ref/example_native, LMc compiled from source) and with the drop-in
layer on the B200 (lmc_b200/dropin/_build/example_dropin).  The greedy ids of
its generate loop must be identical, and every ops.h kernel it calls
(matmul_vec, layer_norm, rms_norm, softmax, gelu, silu, rope_apply,
attention_forward, llama_attention_forward, swiglu_ffn_forward,
transformer_block_forward) must agree within rel-err 1e-3."""
import os
import subprocess

import numpy as np
import pytest

from lmc_b200 import synth
from tests.conftest import ROOT, rel_err

NATIVE = os.path.join(ROOT, "oracle", "_ref", "example_native")
DROPIN = os.path.join(ROOT, "lmc_b200", "dropin", "_build", "example_dropin")
ARCHIVE = os.path.join(ROOT, "lmc_b200", "dropin", "_build", "liblmc_ops_dropin.a")
OPS_H = ["load_model", "model_forward", "matmul_vec", "layer_norm", "rms_norm", "softmax", "gelu", "silu",
         "rope_apply", "attention_forward", "llama_attention_forward", "swiglu_ffn_forward",
         "transformer_block_forward", "detect_format", "find_default_model"]

MODELS = [
    ("gpt2", dict(L=2, D=256, H=4, S=128, V=1000, seed=21)),
    ("llama", dict(L=2, D=512, H=8, Hkv=2, F=768, S=128, V=1000, seed=21)),
]


def need(path):
    if not os.path.exists(path):
        pytest.skip(f"{os.path.relpath(path, ROOT)} not built (make -C oracle ref; make -C lmc_b200/dropin)")


def run(exe, *args):
    out = subprocess.run([exe, *map(str, args)], capture_output=True, text=True, timeout=600)
    return out.returncode, out.stdout, out.stderr


def parse(stdout):
    res = {}
    for line in stdout.splitlines():
        if line.startswith("["):
            continue
        f = line.split()
        if len(f) >= 2 and f[1].isdigit():
            res[f[0]] = np.array([float(v) for v in f[2:]], np.float64)
    return res


def test_dropin_archive_defines_ops_h():
    """The layer defines LMc's ops.h / gguf.h entry points and needs none of
    LMc's gguf.c / ops.c / ops_llama.c symbols."""
    need(ARCHIVE)
    out = subprocess.check_output(["nm", ARCHIVE], text=True)
    defined = {l.split()[-1] for l in out.splitlines() if " T " in l}
    undefined = {l.split()[-1] for l in out.splitlines() if " U " in l}
    assert set(OPS_H) <= defined
    assert not (undefined & {"dequant_q4k", "load_model_gguf", "llama_model_forward", "gguf_name_to_ptr"})


def test_example_native_matches_lmc_generate(model_dir):
    """The example program on LMc itself gives LMc's generate() ids (the same
    ids ref_shim's driver of LMc produces)."""
    need(NATIVE)
    from oracle import Ref
    kind, kw = MODELS[0]
    path = synth.cached_model(kind, model_dir, **kw)
    prompt = [5, 17, 900, 3, 999, 0]
    rc, out, err = run(NATIVE, path, "gen", 12, *prompt)
    assert rc == 0, err
    ids = parse(out)["ids"].astype(int).tolist()
    ref = Ref()
    ref.load(path)
    want, _, _ = ref.generate(np.array(prompt, np.int32), 12)
    assert ids == want.tolist()


def test_detect_format_matches_lmc(tmp_path, model_dir):
    """gguf.h's detect_format through the layer gives LMc's answer for
    names that decide by suffix, files that decide by their magic (GGUF, LMc's
    .bin header), unreadable and missing files.  No model is loaded."""
    need(NATIVE)
    need(DROPIN)
    import struct
    gguf = synth.cached_model(MODELS[0][0], model_dir, **MODELS[0][1])
    plain = tmp_path / "model_without_suffix"
    plain.write_bytes(open(gguf, "rb").read()[:64])
    legacy = tmp_path / "legacy_weights"
    legacy.write_bytes(struct.pack("<I", 0x47505432) + b"\0" * 60)
    junk = tmp_path / "junk"
    junk.write_bytes(b"abc")
    paths = [str(p) for p in (plain, legacy, junk)] + [str(tmp_path / "x.gguf"), str(tmp_path / "y.bin"),
                                                       str(tmp_path / "missing"), gguf]
    rc_n, out_n, err_n = run(NATIVE, "format", *paths)
    rc_d, out_d, err_d = run(DROPIN, "format", *paths)
    assert rc_n == 0 and rc_d == 0, (err_n, err_d)
    assert out_d == out_n
    assert [int(l.split()[1]) for l in out_n.splitlines()] == [2, 1, 0, 2, 1, 0, 2]


def test_dropin_fails_loudly_without_gpu(model_dir):
    need(DROPIN)
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    kind, kw = MODELS[0]
    rc, out, err = run(DROPIN, synth.cached_model(kind, model_dir, **kw), "gen", 4, 1, 2)
    assert rc == 1 and "[FATAL]" in err and "ids" not in out


@pytest.mark.gpu
@pytest.mark.parametrize("kind,kw", MODELS)
def test_dropin_ops_match_lmc(cuda, model_dir, kind, kw):
    need(NATIVE)
    need(DROPIN)
    path = synth.cached_model(kind, model_dir, **kw)
    rc, out_n, err = run(NATIVE, path, "ops")
    assert rc == 0, err
    rc, out_d, err = run(DROPIN, path, "ops")
    assert rc == 0, err
    want, got = parse(out_n), parse(out_d)
    assert set(want) == set(got) and len(want) >= 10
    for name in want:
        assert got[name].shape == want[name].shape, name
        assert rel_err(got[name], want[name]) < 1e-3, name


@pytest.mark.gpu
@pytest.mark.parametrize("kind,kw", MODELS + [("gpt2", dict(seed=0))])
def test_dropin_generate_matches_lmc(cuda, model_dir, kind, kw):
    """32 greedy ids of LMc's generate loop through the drop-in equal LMc's
    (the last case is GPT-2 Small, the decode benchmark's model)."""
    need(NATIVE)
    need(DROPIN)
    path = synth.cached_model(kind, model_dir, **kw)
    V = kw.get("V", 50257)
    prompt = np.random.default_rng(4).integers(0, V, 8).tolist()
    rc, out_n, err = run(NATIVE, path, "gen", 32, *prompt)
    assert rc == 0, err
    rc, out_d, err = run(DROPIN, path, "gen", 32, *prompt)
    assert rc == 0, err
    assert parse(out_d)["ids"].tolist() == parse(out_n)["ids"].tolist()
