"""Build libks_b200.so in-tree with nvcc for sm_100a.

    python -m kernelswift_b200.build [--verbose]

One translation unit (csrc/ks_capi.cu) holds every kernel and the C ABI.  The
result is written next to this file so it travels with the source tree.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libks_b200.so")
SOURCES = ["ks_capi.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def command(ptxas_verbose: bool = False, out: str = OUT) -> list[str]:
    cmd = [nvcc(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
           "-I", os.path.join(ROOT, "include"), "-I", CSRC, "-o", out]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    return cmd + [os.path.join(CSRC, s) for s in SOURCES]


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(ROOT, "include", "ks_b200.h"))
    return all(os.path.getmtime(d) <= t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    tmp = OUT + ".tmp"
    res = subprocess.run(command(verbose, tmp), capture_output=True, text=True)
    if verbose or res.returncode:
        sys.stderr.write(res.stdout + res.stderr)
    if res.returncode:
        raise RuntimeError(f"nvcc failed with code {res.returncode}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
