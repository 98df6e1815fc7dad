"""Build the C++ drop-in test program (tests/cpp/test_dropin.cpp) against
include/alpakann_b200/onHost.hpp and the in-tree libann_b200.so."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT_DIR = os.path.join(HERE, "_build")
EXE = os.path.join(OUT_DIR, "test_dropin")
SRC = os.path.join(HERE, "test_dropin.cpp")
LIB_DIR = os.path.join(ROOT, "alpakann_b200", "_build")
CUDA = "/usr/local/cuda"


E2E_SRC = os.path.join(HERE, "decode_e2e.cpp")
E2E_LIB = os.path.join(OUT_DIR, "libdecode_e2e.so")


def build_e2e(force: bool = False) -> str:
    """tests/cpp/decode_e2e.cpp -> libdecode_e2e.so: the decode step through the
    C++ drop-in header with host buffers (bench.py's end-to-end figure)."""
    os.makedirs(OUT_DIR, exist_ok=True)
    deps = [E2E_SRC, os.path.join(ROOT, "include", "alpakann_b200", "onHost.hpp"),
            os.path.join(ROOT, "include", "ann_b200.h")]
    if not force and os.path.exists(E2E_LIB) and all(os.path.getmtime(E2E_LIB) >= os.path.getmtime(d) for d in deps):
        return E2E_LIB
    cmd = ["g++", "-std=c++20", "-O2", "-Wall", "-fPIC", "-shared", "-I", os.path.join(ROOT, "include"), "-I",
           f"{CUDA}/include", E2E_SRC, "-o", E2E_LIB, "-L", LIB_DIR, "-lann_b200", f"-Wl,-rpath,{LIB_DIR}",
           "-L", f"{CUDA}/lib64", "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
    subprocess.run(cmd, check=True)
    return E2E_LIB


def build(force: bool = False) -> str:
    build_e2e(force)
    os.makedirs(OUT_DIR, exist_ok=True)
    deps = [SRC, os.path.join(ROOT, "include", "alpakann_b200", "onHost.hpp"), os.path.join(ROOT, "include",
                                                                                             "ann_b200.h")]
    if not force and os.path.exists(EXE) and all(os.path.getmtime(EXE) >= os.path.getmtime(d) for d in deps):
        return EXE
    cmd = ["g++", "-std=c++20", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"), "-I", f"{CUDA}/include", SRC,
           "-o", EXE, "-L", LIB_DIR, "-lann_b200", f"-Wl,-rpath,{LIB_DIR}", "-L", f"{CUDA}/lib64", "-lcudart",
           f"-Wl,-rpath,{CUDA}/lib64"]
    subprocess.run(cmd, check=True)
    return EXE


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
