"""Build recipe for the CPU oracle (test infrastructure; see relpos_oracle.c's header).

    python oracle/build_oracle.py      -> oracle/liboracle.so

The reference (apiplant/sam-rs) is Rust and its CPU path cannot be compiled here (no cargo/rustc); the
oracle is the C restatement in relpos_oracle.c. The reference's CUDA kernels are plain CUDA C and are
compiled by build_ref_cuda.py into oracle/_ref/ (the parity tests run them).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "relpos_oracle.c")
OUT = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    cmd = ["gcc", "-O3", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared", "-std=gnu11",
           SRC, "-o", OUT + ".tmp", "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
