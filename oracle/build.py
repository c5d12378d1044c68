"""Build recipes for the oracle (test infrastructure only).

  python oracle/build.py          -> oracle/_build/libj1oracle.so  (CPU restatement, j1_oracle.cpp)
  python oracle/build.py --ref    -> also oracle/_ref/kernels.cubin (the reference's own
                                     src/cuda/kernels.cu, compiled unmodified for sm_100a
                                     from the reference tree when it is present; the
                                     GPU box has no reference tree and uses the prebuilt cubin)

Outputs are git-ignored but travel to the GPU box with the repository snapshot.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
REF = os.path.join(HERE, "_ref")
LIB = os.path.join(BUILD, "libj1oracle.so")
CUBIN = os.path.join(REF, "kernels.cubin")
# The reference checkout: $J1_REFERENCE_DIR, else a directory named "reference" beside this
# repository's root. Without one (the GPU box) the prebuilt cubin is used.
REFERENCE_DIR = os.environ.get("J1_REFERENCE_DIR") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
REFERENCE_KERNELS = os.path.join(REFERENCE_DIR, "src", "cuda", "kernels.cu")


def build_oracle(force=False):
    src = os.path.join(HERE, "j1_oracle.cpp")
    os.makedirs(BUILD, exist_ok=True)
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(src):
        return LIB
    # -ffp-contract=off: no implicit FMA contraction, matching the reference's Rust float semantics.
    cmd = ["g++", "-O3", "-std=c++17", "-fopenmp", "-fPIC", "-shared", "-ffp-contract=off", "-o", LIB, src]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed: %s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    return LIB


def build_reference_kernels(force=False):
    """Compile the reference's kernels.cu (hidden 384 only) as-is; returns the cubin path or None."""
    if not os.path.exists(REFERENCE_KERNELS):
        return CUBIN if os.path.exists(CUBIN) else None
    os.makedirs(REF, exist_ok=True)
    if not force and os.path.exists(CUBIN) and os.path.getmtime(CUBIN) >= os.path.getmtime(REFERENCE_KERNELS):
        return CUBIN
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    # Same flags as the reference's build.rs:26 (-O3 -std=c++17 -lineinfo), one arch: sm_100a.
    cmd = [nvcc, "--cubin", "-O3", "-std=c++17", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a", "-o",
           CUBIN, REFERENCE_KERNELS]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("reference kernels build failed: %s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    return CUBIN


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    if "--ref" in sys.argv:
        print(build_reference_kernels(force="--force" in sys.argv))
