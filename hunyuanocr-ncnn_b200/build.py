"""Build recipe: compiles the CUDA library for sm_100a in-tree (no JIT cache).

    python hunyuanocr-ncnn_b200/build.py

produces hunyuanocr-ncnn_b200/libhy_decode.so from csrc/ with nvcc
(-gencode arch=compute_100a,code=sm_100a). nvcc cross-compiles without a GPU.
"""

from __future__ import annotations

import hashlib
import json
import os
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libhy_decode.so")
RECORD = os.path.join(HERE, "libhy_decode.build.json")   # what the last in-tree build compiled, and how
SOURCES = [os.path.join(HERE, "csrc", "hy_capi.cu"), os.path.join(HERE, "csrc", "hy_package.cpp")]
DEPS = [os.path.join(HERE, "csrc", f) for f in os.listdir(os.path.join(HERE, "csrc"))] + [
    os.path.join(REPO, "include", "hy_decode.h")]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-shared", "-I" + os.path.join(REPO, "include")]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in DEPS + [__file__])


def build(force: bool = False, verbose: bool = False, defines=(), out: str = LIB) -> str:
    """Build the library (into `out`; `defines` such as "HY_TRACE_CTAS=148" become -D flags,
    for instrumented builds kept beside the in-tree one)."""
    if out == LIB and not defines and not force and up_to_date():
        return LIB
    cmd = [NVCC, *FLAGS, *[f"-D{d}" for d in defines], "-o", out, *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    t0 = time.time()
    subprocess.run(cmd, check=True)
    if out == LIB:
        write_record(cmd, time.time() - t0)
    return out


def write_record(cmd, seconds: float) -> None:
    """Record of a fresh in-tree build: the nvcc command and version, the digest of
    every source it read, and of the library it wrote."""
    def digest(p):
        with open(p, "rb") as f:
            return hashlib.sha256(f.read()).hexdigest()

    ver = subprocess.run([NVCC, "--version"], capture_output=True, text=True).stdout.strip().splitlines()
    rec = {"built_at": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()), "seconds": round(seconds, 1),
           "nvcc": ver[-1] if ver else "", "command": cmd,
           "sources": {os.path.relpath(p, REPO): digest(p) for p in sorted(set(SOURCES + DEPS))},
           "library": {"path": os.path.relpath(LIB, REPO), "sha256": digest(LIB), "bytes": os.path.getsize(LIB)}}
    with open(RECORD, "w") as f:
        json.dump(rec, f, indent=1)


SHIM_TEST_SRC = os.path.join(REPO, "tests", "cpp", "test_shim.cpp")
SHIM_TEST_BIN = os.path.join(REPO, "tests", "cpp", "test_shim")


def build_shim_test(force: bool = False) -> str:
    """Compile the C++17 layer's test program (tests/cpp/test_shim.cpp, over
    include/hunyuan_ocr_cuda.h) against the in-tree library."""
    deps = [SHIM_TEST_SRC, LIB, os.path.join(REPO, "include", "hunyuan_ocr_cuda.h"),
            os.path.join(REPO, "include", "hy_decode.h")]
    if not force and os.path.exists(SHIM_TEST_BIN) and all(
            os.path.getmtime(d) <= os.path.getmtime(SHIM_TEST_BIN) for d in deps):
        return SHIM_TEST_BIN
    cxx = os.environ.get("CXX", "g++")
    subprocess.run([cxx, "-std=c++17", "-O1", "-Wall", "-Wextra", "-I" + os.path.join(REPO, "include"), SHIM_TEST_SRC,
                    "-L" + HERE, "-lhy_decode", "-Wl,-rpath," + HERE, "-o", SHIM_TEST_BIN], check=True)
    return SHIM_TEST_BIN


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description="build libhy_decode.so for sm_100a")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", action="store_true", help="print the command and ptxas resource usage")
    ap.add_argument("--define", action="append", default=[], help="NAME=VALUE, passed as -D (repeatable)")
    ap.add_argument("--out", default=LIB, help="output path (default: the in-tree library)")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.v, defines=a.define, out=a.out))
