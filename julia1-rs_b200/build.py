"""Build libj1.so (CUDA kernels + native host) in-tree for sm_100a with nvcc.

Usage: python julia1-rs_b200/build.py [--force]

Objects go to julia1-rs_b200/_build/, the library to julia1-rs_b200/lib/libj1.so.
Sources are recompiled only when newer than their object (or a header changed).
"""
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libj1.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", os.path.join(ROOT, "include")]
SOURCES = ["gemm.cu", "gemm_resid.cu", "attention.cu", "rows.cu", "attention_noalloc.cu", "checkpoint.cpp", "model.cpp", "engine.cpp", "router.cpp", "tokenizer.cpp"]


def _newest_header():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(ROOT, "include", "j1.h"))
    return max(os.path.getmtime(h) for h in hs)


def _compile(src, force, hdr_time):
    s = os.path.join(CSRC, src)
    o = os.path.join(BUILD, src + ".o")
    if not force and os.path.exists(o) and os.path.getmtime(o) >= max(os.path.getmtime(s), hdr_time):
        return o, None
    cmd = [NVCC] + ARCH + COMMON + ["-c", s, "-o", o]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return o, "compile failed: %s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr)
    return o, None


def build(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    hdr = _newest_header()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        results = list(ex.map(lambda s: _compile(s, force, hdr), SOURCES))
    errs = [e for _, e in results if e]
    if errs:
        raise RuntimeError("\n".join(errs))
    objs = [o for o, _ in results]
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        # Export only the j1_* C ABI from the shared library.
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-Xcompiler", "-fPIC", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed: %s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
