"""Build libwxb200.so from csrc/ for sm_100a, in the source tree.

    python -m wxb200._build          (with whisper-xdna_b200/ on sys.path)

nvcc compiles each translation unit in parallel into _build/ at the repository
root and links one shared library next to this file. The CUDA runtime is
linked statically and the driver API is reached through
cudaGetDriverEntryPoint, so the library loads on machines without a GPU.
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
ROOT = PKG.parents[1]
BUILD = ROOT / "_build"
LIB = PKG / "libwxb200.so"
SOURCES = ["capi.cu", "rowops.cu", "gemm.cu", "attention.cu", "encoder.cu", "noalloc.cu",
           "mel.cu", "quant.cu"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3",
              "-std=c++17", "-Xcompiler", "-fPIC"]


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def _stale(obj, src):
    if not obj.exists():
        return True
    deps = [src] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + \
        [ROOT / "include" / "wxb200.h"]
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose=False, force=False):
    BUILD.mkdir(exist_ok=True)
    nvcc = _nvcc()

    def compile_one(name):
        src = CSRC / name
        obj = BUILD / (name[:-3] + ".o")
        if not force and not _stale(obj, src):
            return obj, ""
        cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {name}:\n{r.stdout}\n{r.stderr}")
        return obj, r.stderr

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(compile_one, SOURCES))
    objs = [o for o, _ in results]
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
               "-o", str(LIB), *map(str, objs), "-lcudart_static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        for _, log in results:
            if log:
                print(log)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
