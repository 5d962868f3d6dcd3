"""Build the CUDA C-ABI library in-tree: sam-rs_b200/libsamrs_b200.so (sm_100a only).

    python sam-rs_b200/build.py [--force] [--verbose]

nvcc cross-compiles for sm_100a without a GPU. The .so is git-ignored but travels with the source
tree to the GPU box, where the package loads it (and fails loudly if it is missing).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT = os.path.join(HERE, "libsamrs_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fvisibility=hidden"]


def sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh"))] + \
        [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and os.path.exists(OUT):
        newest = max(os.path.getmtime(p) for p in sources())
        if os.path.getmtime(OUT) >= newest:
            return OUT
    cmd = [NVCC, *ARCH, *FLAGS, os.path.join(CSRC, "samrs_abi.cu"), "-o", OUT + ".tmp", "-lcuda"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
