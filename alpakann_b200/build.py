"""Build the sm_100a CUDA library of alpakann_b200 in-tree.

alpakann_b200/csrc/*.cu -> alpakann_b200/_build/obj/*.o -> alpakann_b200/_build/libann_b200.so
alpakann_b200/csrc/*.cpp (host-only code: file loading, hashing) -> g++ -> same library

nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3, C++20, static
cudart inside the shared library (no dependency on the runtime version a
host process such as PyTorch happens to load), cuBLAS resolved at run time.
"""
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
OBJ_DIR = os.path.join(OUT_DIR, "obj")
LIB = os.path.join(OUT_DIR, "libann_b200.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++20", "-Xcompiler", "-fPIC,-Wall", "--expt-relaxed-constexpr",
                     "-I", INCLUDE, "-I", CSRC]


CXX_FLAGS = ["-O3", "-std=c++20", "-fPIC", "-Wall", "-I", INCLUDE, "-I", CSRC, "-I", "/usr/local/cuda/include"]


def cxx():
    for cand in (os.environ.get("CXX"), shutil.which("g++")):
        if cand and (os.path.exists(cand) or shutil.which(cand)):
            return cand
    raise RuntimeError("g++ not found")


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, extra):
    base = os.path.basename(src)
    obj = os.path.join(OBJ_DIR, base.rsplit(".", 1)[0] + (".o" if base.endswith(".cu") else ".cpp.o"))
    if _stale(obj, [src] + headers() + [__file__]):
        if base.endswith(".cu"):
            cmd = [nvcc()] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
        else:
            cmd = [cxx()] + CXX_FLAGS + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed for {base}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    if force:
        for f in os.listdir(OBJ_DIR):
            os.remove(os.path.join(OBJ_DIR, f))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), srcs))
    if _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="--ptxas" in sys.argv))
