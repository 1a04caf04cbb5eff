#!/usr/bin/env python3
"""Build the B200 Qwen3 library in-tree.

    python qwen3.cpp_b200/build.py [--force]

Compiles every csrc/*.cu for sm_100a with nvcc into qwen3.cpp_b200/lib/libq3b200.so (the C ABI of
include/q3_b200.h) and the C++ reference-surface layer csrc/inference_b200.cpp (include/
inference_b200.h) with g++ into qwen3.cpp_b200/lib/libq3b200_cxx.so. Objects go to
qwen3.cpp_b200/_build/. A target is rebuilt when any of its sources or headers is newer.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "lib"
SO = LIB / "libq3b200.so"
CXX_SO = LIB / "libq3b200_cxx.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and Path(c).exists():
            return c
    raise FileNotFoundError("nvcc not found")


def cuda_home() -> Path:
    return Path(nvcc()).resolve().parent.parent


def host_cxx() -> str:
    # The image exports CXX pointing at a gcc without libgomp; the system g++ is complete.
    for c in ("/usr/bin/g++", shutil.which("g++")):
        if c and Path(c).exists():
            return c
    raise FileNotFoundError("g++ not found")


def _newest(paths) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} {cmd[-1]}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    hdr_time = _newest(headers)
    cus = sorted(CSRC.glob("*.cu"))
    objs = []
    jobs = []
    for cu in cus:
        obj = BUILD / (cu.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(cu.stat().st_mtime, hdr_time):
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(cu),
                   "-o", str(obj)]
            jobs.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for f in [ex.submit(_run, j) for j in jobs]:
            f.result()
    if force or jobs or not SO.exists() or SO.stat().st_mtime < _newest(objs):
        _run([nvcc(), *ARCH, "-shared", "-o", str(SO), *map(str, objs)])
    cxx_src = CSRC / "inference_b200.cpp"
    if cxx_src.exists():
        deps = [cxx_src, SO, *INCLUDE.glob("*.h")]
        if force or not CXX_SO.exists() or CXX_SO.stat().st_mtime < _newest(deps):
            # -Wno-free-nonheap-object: a known false positive of g++ 13 in std::vector growth.
            _run([host_cxx(), "-std=gnu++23", "-O2", "-fPIC", "-shared", "-Wno-free-nonheap-object",
                  "-I", str(INCLUDE), "-I", str(cuda_home() / "include"), str(cxx_src), "-o", str(CXX_SO),
                  f"-L{LIB}", "-lq3b200", f"-L{cuda_home() / 'lib64'}", "-lcudart",
                  "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{cuda_home() / 'lib64'}"])
    if verbose:
        print(f"built {SO}")
    return SO


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    build(args.force, verbose=True)


if __name__ == "__main__":
    main()
