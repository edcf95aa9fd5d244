"""Build recipe of libtalm_b200.so: one nvcc invocation for sm_100a, output in-tree.

    python -m talm_b200.build            # builds talm_b200/_lib/libtalm_b200.so
    python -m talm_b200.build --verbose  # also prints ptxas register / spill report

The library is a single translation unit (csrc/talm.cu includes the kernel files), linked
against the static CUDA runtime; the driver's tensor-map encoder is looked up at run time, so
the library loads on machines without an NVIDIA driver (the symbol check of the CPU tests).
"""

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
LIB_NAME = "libtalm_b200.so"
LIB_PATH = os.path.join(OUT_DIR, LIB_NAME)
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC)
                  if f.endswith((".cu", ".cuh")))


def up_to_date():
    if not os.path.exists(LIB_PATH):
        return False
    built = os.path.getmtime(LIB_PATH)
    deps = sources() + [os.path.join(HERE, "..", "include", "talm.h")]
    return all(os.path.getmtime(p) <= built for p in deps if os.path.exists(p))


def build(force=False, verbose=False):
    """Compile csrc/talm.cu into _lib/libtalm_b200.so (skipped when up to date)."""
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-O2", "-o", tmp,
           os.path.join(CSRC, "talm.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr[-4000:]}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
