"""The C oracle under AddressSanitizer and UndefinedBehaviorSanitizer
(LMc's own build has neither; its sources have latent undefined behaviour
the restatement must not inherit, such as the IQ4_XS read past the last
block, which the oracle is given exactly): tests/oracle_sanitize.c calls
every entry point with buffers of their exact sizes, loads and runs a tiny
GPT-2 and a tiny LLaMA model in every K/V row form, and checks that GGUF
files cut short inside their tensor data fail to load.  Any out-of-bounds
access, leak or undefined operation fails the run."""
import os
import subprocess

import pytest

from lmc_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def test_oracle_is_clean_under_asan_and_ubsan(tmp_path):
    exe = str(tmp_path / "oracle_sanitize")
    build = subprocess.run(["gcc", "-std=c99", "-O1", "-g", "-fsanitize=address,undefined",
                            "-fno-sanitize-recover=all", "-fno-omit-frame-pointer", "-ffp-contract=off",
                            "-o", exe, os.path.join(HERE, "oracle_sanitize.c"),
                            os.path.join(ROOT, "oracle", "lmc_oracle.c"), "-lm"], capture_output=True, text=True)
    if build.returncode and "sanitize" in build.stderr:
        pytest.skip("compiler without ASan/UBSan: " + build.stderr[-200:])
    assert build.returncode == 0, build.stderr[-2000:]
    d = str(tmp_path)
    good = [synth.cached_model("gpt2", d, L=2, D=64, H=2, S=16, V=300, seed=1),
            synth.cached_model("llama", d, L=2, D=64, H=4, Hkv=2, F=128, S=16, V=300, seed=1)]
    data = open(good[0], "rb").read()
    bad = []
    # the header alone, inside the metadata, half the tensors, and 40 bytes
    # short (past the end padding of at most 31 bytes, into the last tensor)
    for i, n in enumerate((10, 200, len(data) // 2, len(data) - 40)):
        p = str(tmp_path / f"cut{i}.gguf")
        with open(p, "wb") as f:
            f.write(data[:n])
        bad.append(p)
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1", UBSAN_OPTIONS="print_stacktrace=1")
    r = subprocess.run([exe] + good + ["--bad"] + bad, capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0 and r.stdout.strip() == "ok", (r.stdout + r.stderr)[-3000:]
