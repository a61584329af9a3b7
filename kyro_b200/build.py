"""Build kyro_b200/libkyro_spec.so from kyro_b200/csrc/*.cu with nvcc for sm_100a.

Usage: python -m kyro_b200.build [--force] [--verbose]

Each translation unit compiles to an object under kyro_b200/_build/, then
nvcc links them into one shared library with the CUDA runtime linked
statically (the library exports only the C ABI of include/kyro_spec.h).
sampler.cu is compiled with --fmad=false: its arithmetic must round exactly
like the CPU restatement it is checked against.
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
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libkyro_spec.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-ffp-contract=off",
          "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]
PER_FILE = {"sampler.cu": ["--fmad=false"]}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))] + [
        os.path.join(ROOT, "include", "kyro_spec.h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    hdrs = headers()
    objs = []
    for src in sources():
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src[:-3] + ".o")
        objs.append(o)
        if force or _stale(o, [s] + hdrs + [__file__]):
            cmd = [cc, *ARCH, *COMMON, *PER_FILE.get(src, []), "-c", s, "-o", o]
            if verbose:
                cmd += ["-Xptxas", "-v"]
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    sys.exit(main())
