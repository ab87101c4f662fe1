"""Builds tests/csrc/exp2_check.cu (test harness for the kernels' FMA-pipe exponentials) into
tests/_build/libexp2check.so with nvcc for sm_100a.  Called by __graft_entry__.build() and, when the library is
missing or older than its sources, by tests/test_gpu_exp2_poly.py."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc", "exp2_check.cu")
PTX_HEADER = os.path.join(os.path.dirname(HERE), "nano-vllm-spec-decode_b200", "csrc", "nva_ptx.cuh")
OUT = os.path.join(HERE, "_build", "libexp2check.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def build(force: bool = False) -> str:
    fresh = os.path.exists(OUT) and all(os.path.getmtime(OUT) >= os.path.getmtime(p) for p in (SRC, PTX_HEADER))
    if force or not fresh:
        os.makedirs(os.path.dirname(OUT), exist_ok=True)
        subprocess.check_call([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-shared",
                               "-Xcompiler", "-fPIC", "-diag-suppress", "20044", "-I", os.path.dirname(PTX_HEADER), SRC, "-o", OUT])
    return OUT


if __name__ == "__main__":
    print(build(force=True))
