"""Build liba11spec.so (the C-ABI CUDA library) for sm_100a, in-tree.

Usage: python a11-llm-optimizer_b200/build.py [--force] [--verbose]
The library lands next to the Python package (a11spec/liba11spec.so) so that
it travels with the repository snapshot and is what the package loads.
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT = os.path.join(HERE, "a11spec", "liba11spec.so")
CPP = os.path.join(HERE, "cpp")
VERIFIER_OUT = os.path.join(CPP, "libspec_verifier.so")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def deps():
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))) + [
        os.path.join(INCLUDE, "a11spec.h")]


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(p) <= t for p in deps())


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    if not force and up_to_date():
        return OUT
    cmd = [NVCC, *NVCC_FLAGS, *extra, "-I", INCLUDE, "-o", OUT + ".tmp", *sources()]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
    if verbose:
        print(r.stdout + r.stderr, file=sys.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


def build_verifier(force: bool = False) -> str:
    """libspec_verifier.so: the A11::Engine::SpeculativeTreeVerifier C++ interface
    over liba11spec (g++, links liba11spec.so and the CUDA runtime)."""
    src = os.path.join(CPP, "speculative_verifier.cpp")
    hdr = os.path.join(CPP, "include", "engine", "speculative_verifier.hpp")
    if not force and os.path.exists(VERIFIER_OUT) and all(
            os.path.getmtime(p) <= os.path.getmtime(VERIFIER_OUT) for p in (src, hdr, OUT)):
        return VERIFIER_OUT
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-I", os.path.join(CPP, "include"), "-I", INCLUDE,
           "-I", os.path.join(CUDA_HOME, "include"), "-o", VERIFIER_OUT, src, "-L", os.path.dirname(OUT),
           "-la11spec", "-Wl,-rpath,$ORIGIN/../a11spec", "-L", os.path.join(CUDA_HOME, "lib64"), "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("g++ failed:\n" + r.stdout + r.stderr)
    return VERIFIER_OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    print(build_verifier(force=args.force))
