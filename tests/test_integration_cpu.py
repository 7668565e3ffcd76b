"""The yalm-side shim that INTEGRATION.md gives (src/b200.cpp of a yalm checkout) compiles against
yalm's own headers and include/yalm_b200.h, so a maintainer can paste it as written.  Syntax only,
no linking; skipped where yalm's sources are not present."""
import os
import re
import shutil
import subprocess

import pytest

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_integration_shim_compiles_against_yalm_headers(tmp_path):
    src = os.path.join(oracle.REF_SRC, "src")
    if not os.path.exists(os.path.join(src, "model.h")) or not shutil.which("g++"):
        pytest.skip("yalm's sources or g++ not present")
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    blocks = re.findall(r"```cpp\n(.*?)```", text, re.S)
    assert blocks, "INTEGRATION.md has no C++ shim"
    shim = tmp_path / "b200.cpp"
    shim.write_text(blocks[0])
    # yalm's src/ holds a time.h, so its directories go on the quote path only (as its own
    # relative includes resolve), not ahead of the system headers
    cmd = ["g++", "-std=c++20", "-fsyntax-only", "-mavx2", "-mf16c", "-mfma",
           "-I/usr/local/cuda/include", "-iquote", src, "-iquote", os.path.join(oracle.REF_SRC, "vendor"),
           "-I" + os.path.join(ROOT, "include"), str(shim)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
