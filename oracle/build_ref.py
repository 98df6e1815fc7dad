"""Build recipe for oracle/_ref: the reference's own kernels, run on the host.

TEST INFRASTRUCTURE ONLY. Compiles oracle/ref_harness/ref_kernels.cpp, which
includes alpakaNN's device kernels (include/alpaka/nn/onAcc/internal/nn/*.hpp)
unmodified from the reference tree, against the host-only alpaka stand-in in
oracle/ref_harness/alpaka/alpaka.hpp, into oracle/_ref/libann_ref.so. Same
floating-point flags as the oracle: no contraction, no fast-math.

The reference tree is read where it lies (REFERENCE_ROOT, default
/root/reference); nothing is copied. Without it, build() returns the library
already built, or None.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "ref_harness", "ref_kernels.cpp")
STANDIN = os.path.join(HERE, "ref_harness")
OUT_DIR = os.path.join(HERE, "_ref")
OUT = os.path.join(OUT_DIR, "libann_ref.so")
REFERENCE_ROOT = os.environ.get("REFERENCE_ROOT", "/root/reference")
KERNELS = os.path.join(REFERENCE_ROOT, "include", "alpaka", "nn", "onAcc", "internal", "nn")


def build(force: bool = False):
    include = os.path.join(REFERENCE_ROOT, "include")
    if not os.path.isdir(KERNELS):
        return OUT if os.path.exists(OUT) else None
    deps = [SRC, os.path.join(STANDIN, "alpaka", "alpaka.hpp")] + [
        os.path.join(KERNELS, f) for f in os.listdir(KERNELS)]
    if not force and os.path.exists(OUT) and all(os.path.getmtime(OUT) >= os.path.getmtime(d) for d in deps):
        return OUT
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = ["g++", "-std=c++20", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-Wall",
           "-I", STANDIN, "-I", include, "-o", OUT, SRC]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
