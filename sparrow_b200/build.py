"""Build recipe for the CUDA library (sm_100a only).

`python -m sparrow_b200.build` compiles csrc/vmlm_cuda.cu into
sparrow_b200/lib/libvmlm_cuda.so with nvcc; the CUDA runtime is linked
statically and the driver's tensor-map encoder is resolved at run time, so the
library needs nothing but the NVIDIA driver where it runs.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc", "vmlm_cuda.cu")
OUT = os.path.join(HERE, "lib", "libvmlm_cuda.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-shared",
]


def sources():
    csrc = os.path.join(HERE, "csrc")
    files = [os.path.join(csrc, f) for f in os.listdir(csrc)]
    files.append(os.path.join(ROOT, "include", "vmlm_cuda.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(f) <= t for f in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    nvcc = os.environ.get("NVCC", "nvcc")
    cmd = [nvcc, *NVCC_FLAGS, "-o", OUT + ".tmp", SRC]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
