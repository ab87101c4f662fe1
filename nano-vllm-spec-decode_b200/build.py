"""Build libnvattn.so in-tree with nvcc for sm_100a (no torch extension machinery: the library is a plain C ABI).

    python nano-vllm-spec-decode_b200/build.py [--force] [--jobs N]

Each .cu file in csrc/ is compiled to an object with relocatable device code (the device error word is shared
across files), then nvcc device-links and links them into nvattn/libnvattn.so.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "nvattn", "libnvattn.so")
BUILD = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _newer(target, deps):
    return os.path.exists(target) and all(os.path.getmtime(target) >= os.path.getmtime(d) for d in deps)


def build(force: bool = False, jobs: int = 8, verbose: bool = False) -> str:
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
                     glob.glob(os.path.join(HERE, "..", "include", "*.h")))
    os.makedirs(BUILD, exist_ok=True)
    objs = []

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        if not force and _newer(obj, [src] + headers):
            return obj, ""
        cmd = [NVCC, *ARCH, *FLAGS, "-I", os.path.join(HERE, "..", "include"), "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        return obj, r.stderr

    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for obj, log in ex.map(compile_one, srcs):
            objs.append(obj)
            if verbose and log:
                print(log, file=sys.stderr)
    if force or not _newer(OUT, objs):
        cmd = [NVCC, *ARCH, "-shared", "-rdc=true", "-Xcompiler", "-fPIC", *objs, "-o", OUT]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))
