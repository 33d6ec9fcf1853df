"""The LMc-side shim shown in INTEGRATION.md (the first C block: load_model
and model_forward over the C ABI) compiles as C99 against include/lmc_cuda.h
and LMc's own headers, with LMc's declarations of the functions it replaces
in scope, so a signature drift on either side shows up here."""
import os
import re
import subprocess

import pytest

from __graft_entry__ import LMC_SRC
from tests.conftest import ROOT


def test_integration_shim_compiles_against_lmc_headers(tmp_path):
    if not os.path.isdir(LMC_SRC):
        pytest.skip("LMc sources not present")
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    block = re.findall(r"```c\n(.*?)```", doc, re.S)[0]
    assert "load_model" in block and "model_forward" in block
    src = tmp_path / "shim.c"
    src.write_text('#include "utils.h"\n#include "models.h"\n#include "ops.h"\n#include "gguf.h"\n' + block)
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", "-I", os.path.join(ROOT, "include"),
                        "-I", LMC_SRC, str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
