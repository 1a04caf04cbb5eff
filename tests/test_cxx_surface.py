"""The C++ surface of include/inference_b200.h (the reference's class names over the C ABI):
its two test programs, the reference's tst/test_block.cpp and tst/test_loader.cpp checks written
against that header, compile and link here; on a GPU they run and pass."""
import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "qwen3.cpp_b200" / "lib"
CXX = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"


@pytest.fixture(scope="module")
def cxx_tests(q3lib, tmp_path_factory):
    import build
    out = tmp_path_factory.mktemp("cxx")
    exes = {}
    for name in ("test_block_b200", "test_loader_b200"):
        exe = out / name
        cmd = [CXX, "-std=gnu++23", "-O1", "-I", str(ROOT / "include"),
               str(ROOT / "tests" / "cxx" / f"{name}.cpp"), "-o", str(exe), f"-L{LIB}",
               "-lq3b200_cxx", "-lq3b200", f"-Wl,-rpath,{LIB}",
               f"-Wl,-rpath,{build.cuda_home() / 'lib64'}"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        exes[name] = exe
    return exes


def test_cxx_programs_link(cxx_tests):
    for exe in cxx_tests.values():
        assert exe.exists() and os.access(exe, os.X_OK)


@pytest.mark.gpu
def test_cxx_block_checks(cxx_tests):
    r = subprocess.run([str(cxx_tests["test_block_b200"])], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "block tests passed" in r.stdout


@pytest.mark.gpu
def test_cxx_loader_and_generate(cxx_tests, full_weights):
    r = subprocess.run([str(cxx_tests["test_loader_b200"]), str(full_weights)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "loader tests passed" in r.stdout
