"""Build libunoq_cuda.so in-tree (unoq-dsp_b200/lib/) for sm_100a with nvcc.

Usage: python unoq-dsp_b200/build.py [--debug]
The shared library is the product's native core: C ABI (include/unoq_cuda.h) over the CUDA
engine and kernels in csrc/. It links only the CUDA runtime (static); NCCL is opened at run time for multi-GPU runs.
"""
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
LIB = HERE / "lib" / "libunoq_cuda.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["plan.cpp", "device_state.cpp", "k_simt.cu", "k_bytes.cu", "k_dw.cu", "k_conv_small.cu", "conv_tc.cu", "conv_rows.cu", "conv_taps.cu", "dw_tc.cu", "k_decode.cu", "gather.cu", "engine.cu", "abi.cu", "k_gemm.cu", "ops_abi.cu", "k_peak.cu"]


def build(debug=False, verbose=False):
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    common = ARCH + ["-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                     "-I", str(CSRC), "-I", str(ROOT / "include")]
    common += ["-O0", "-g"] if debug else ["-O3"]
    objs = []
    for src in SOURCES:
        obj = objdir / (src + ".o")
        path = CSRC / src
        deps = [path] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + list((ROOT / "include").glob("*.h"))
        if not obj.exists() or any(d.stat().st_mtime > obj.stat().st_mtime for d in deps):
            cmd = [NVCC] + common + ["-x", "cu" if src.endswith(".cu") else "c++", "-c", str(path), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd))
            subprocess.run(cmd, check=True)
        objs.append(str(obj))
    cmd = [NVCC] + ARCH + ["-shared", "-o", str(LIB)] + objs + ["-cudart", "static", "-lpthread", "-ldl", "-lrt"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(debug="--debug" in sys.argv, verbose=True))
