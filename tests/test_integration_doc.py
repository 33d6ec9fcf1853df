"""The integration guide's code works as written: the C ABI shim of its §2
compiles as C99 against include/lmc_cuda.h and LMc's own headers (with LMc's
declarations of the functions it replaces in scope), and the link line of its
§1 builds LMc's own CLI (src/lmc.c) against the drop-in layer with no symbol
missing or defined twice."""
import os
import re
import subprocess

import pytest

from __graft_entry__ import LMC_SRC
from tests.conftest import ROOT

DROPIN_LIB = os.path.join(ROOT, "lmc_b200", "dropin", "_build", "liblmc_ops_dropin.a")


def test_integration_shim_compiles_against_lmc_headers(tmp_path):
    if not os.path.isdir(LMC_SRC):
        pytest.skip("LMc sources not present")
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    block = [b for b in re.findall(r"```c\n(.*?)```", doc, re.S) if "model_forward" in b][0]
    assert "load_model" in block and "model_forward" in block
    src = tmp_path / "shim.c"
    src.write_text('#include "utils.h"\n#include "models.h"\n#include "ops.h"\n#include "gguf.h"\n' + block)
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", "-I", os.path.join(ROOT, "include"),
                        "-I", LMC_SRC, str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_lmc_cli_links_against_dropin(tmp_path):
    """The guide's link line, run: LMc's lmc.c, utils.c, models.c,
    tokenizer.c and llama_tok.c with the drop-in archive and liblmc_b200."""
    if not os.path.isdir(LMC_SRC):
        pytest.skip("LMc sources not present")
    if not os.path.exists(DROPIN_LIB):
        pytest.skip("drop-in layer not built (make -C lmc_b200/dropin)")
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    sh = re.findall(r"```sh\n(.*?)```", doc, re.S)[0]
    line = re.search(r"gcc -std=c99.*?-lm", sh, re.S).group(0).replace("\\\n", " ")
    line = line.replace("$LMC/src", LMC_SRC).replace("$PWD", ROOT).replace("lmc_b200_cli", str(tmp_path / "cli"))
    r = subprocess.run(line + " -w", shell=True, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert os.path.exists(tmp_path / "cli")
