"""Build libad_b200.so in-tree with nvcc for sm_100a.

``python -m ad_b200.build`` (also called by ``__graft_entry__.build()``).
The library links the CUDA runtime statically and NVRTC dynamically; the CUDA
driver is reached through ``cudaGetDriverEntryPoint`` and NCCL is dlopen'ed, so
the library loads on a machine without a GPU driver.
"""
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "libad_b200.so")
SOURCES = [os.path.join(PKG, "csrc", "runtime.cu"), os.path.join(PKG, "csrc", "noalloc.cu")]
HEADERS = [os.path.join(ROOT, "include", "ad_b200.h")]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(s) > t for s in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    tmp = LIB + f".{os.getpid()}.tmp"
    cmd = [NVCC, "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
           "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
           "-I", os.path.join(ROOT, "include"), *SOURCES, "-o", tmp, "-lnvrtc", "-ldl", "-lpthread"]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + r.stdout[-3000:] + r.stderr[-6000:])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
