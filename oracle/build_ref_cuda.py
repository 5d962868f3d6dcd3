"""Build recipe for the reference's own CUDA kernels (test infrastructure, never part of the product).

    python oracle/build_ref_cuda.py      -> oracle/_ref/sam.cubin

The reference (apiplant/sam-rs) is Rust and cannot be built here. Its CUDA kernels are different: they are
one self-contained CUDA C file, kernels/sam.cu, which includes only the CUDA headers. They are:
  * relpos_softmax_i{1..32}_{f32,f16,bf16}: the softmax of the reference's CUDA attention path;
  * qkv_split_*, bias_residual_*, bias_gelu_*: the elementwise ops around it.
This script compiles that file where it lies, with the flags of the reference's build.rs
(`-O3 --use_fast_math -std=c++17`), for sm_100. build.rs emits PTX for compute_{cap} and lets the driver
JIT it; this script emits the cubin for the same target ahead of time.
The output goes only to oracle/_ref/, which git ignores. oracle/ref_cuda.py loads it through the CUDA
driver API, as candle's custom-module loader does (src/kernels.rs:1079, `get_or_load_custom_func`).
The reference tree is read at build time only. Without it, nothing is built and the tests that need the
cubin are skipped.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SRC = os.environ.get("SAMRS_REFERENCE_ROOT", os.path.join(os.sep, "root", "reference"))
SRC = os.path.join(REF_SRC, "kernels", "sam.cu")
OUT_DIR = os.path.join(HERE, "_ref")
OUT = os.path.join(OUT_DIR, "sam.cubin")


def build(force: bool = False):
    """Compile the reference's kernels/sam.cu into oracle/_ref/sam.cubin; None if the source is absent."""
    if not os.path.exists(SRC):
        return None
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    os.makedirs(OUT_DIR, exist_ok=True)
    nvcc = os.path.join(os.environ.get("CUDA_PATH", "/usr/local/cuda"), "bin", "nvcc")
    cmd = [nvcc, "-cubin", "-O3", "--use_fast_math", "-std=c++17", "-gencode", "arch=compute_100,code=sm_100",
           SRC, "-o", OUT + ".tmp"]
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
