"""The yalm-side binding (yalm_b200/integration/: yalm.patch and b200.cpp) against yalm's sources, on
the CPU: the patch applies cleanly to a copy of a yalm checkout, and the patched sources with the
shim compile.  The linked CLI runs in tests/test_integration_gpu.py.  Skipped where yalm's sources
are not present (the GPU box uses the prebuilt binary)."""
import os
import shutil
import subprocess

import pytest

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INTEG = os.path.join(ROOT, "yalm_b200", "integration")


@pytest.fixture
def patched_checkout(tmp_path):
    if not oracle.REF_SRC or not shutil.which("g++") or not shutil.which("patch"):
        pytest.skip("yalm's sources, g++ or patch not present")
    dst = tmp_path / "yalm"
    dst.mkdir()
    for d in ("src", "vendor"):
        shutil.copytree(os.path.join(oracle.REF_SRC, d), dst / d)
    shutil.copy(os.path.join(oracle.REF_SRC, "Makefile"), dst / "Makefile")
    subprocess.run(["chmod", "-R", "u+w", str(dst)], check=True)
    r = subprocess.run(["patch", "-s", "-d", str(dst), "-p1", "-i", os.path.join(INTEG, "yalm.patch")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    shutil.copy(os.path.join(INTEG, "b200.cpp"), dst / "src" / "b200.cpp")
    return dst


@pytest.mark.parametrize("src", ["b200.cpp", "model.cpp", "main.cpp"])
def test_patched_yalm_compiles(patched_checkout, src):
    d = patched_checkout
    # yalm's src/ holds a time.h, so its directories go on the quote path only (as its own relative
    # includes resolve), not ahead of the system headers
    cmd = ["g++", "-std=c++20", "-fsyntax-only", "-mavx2", "-mf16c", "-mfma", "-fopenmp",
           "-I/usr/local/cuda/include", "-iquote", str(d / "src"), "-I" + str(d / "vendor"),
           "-I" + os.path.join(ROOT, "include"), str(d / "src" / src)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]


def test_patch_adds_the_device_only(patched_checkout):
    """The patch touches model.h, model.cpp, main.cpp and the Makefile, and adds no CPU-path change:
    every hunk only adds lines."""
    text = open(os.path.join(INTEG, "yalm.patch")).read()
    files = [l.split()[-1][2:] for l in text.splitlines() if l.startswith("+++ ")]
    assert sorted(files) == ["Makefile", "src/main.cpp", "src/model.cpp", "src/model.h"]
    removed = [l for l in text.splitlines() if l.startswith("-") and not l.startswith("--- ")]
    assert removed == []
