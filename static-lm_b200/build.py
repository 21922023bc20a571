"""Build recipe of libslm_b200.so (sm_100a) -- used by __graft_entry__.build().

nvcc -gencode arch=compute_100a,code=sm_100a, --fmad=false so that every f32
multiply and add is rounded on its own as in the reference (fused
multiply-adds appear only where written as __fmaf_rn), no fast-math.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libslm_b200.so")
SOURCES = ["kernels_vec.cu", "kernels_gemv.cu", "kernels_attn.cu", "kernels_attn_tc.cu", "kernels_attn_flash.cu",
           "kernels_attn_cluster.cu", "runtime.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "--fmad=false",
         "-std=c++17", "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
         "-shared", "-cudart", "shared"]


def build(verbose: bool = False, extra=None) -> str:
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    newest = max(os.path.getmtime(p) for p in srcs + headers +
                 [os.path.join(HERE, "..", "include", "slm_b200.h"), os.path.abspath(__file__)])
    if os.path.exists(OUT) and os.path.getmtime(OUT) >= newest and not extra:
        return OUT
    cmd = [NVCC] + FLAGS + (extra or []) + ["-o", OUT] + srcs
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(verbose=True, extra=sys.argv[1:] or None)
