"""Build libgeoattn.so in-tree with nvcc for sm_100a (no torch extension machinery; plain C ABI)."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libgeoattn.so")
SOURCES = ("geoattn.cu",)
HEADERS = ("geoattn_kernels.cuh", "sm100.cuh", "tma_host.h")
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo", "-shared",
              "-Xcompiler", "-fPIC"]


def nvcc():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _stale():
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(HERE, "..", "include", "geoattn.h"))
    return any(os.path.getmtime(f) > t for f in deps)


def build(force=False, verbose=False):
    """Compile csrc/geoattn.cu into libgeoattn.so next to this file; returns the path."""
    if not force and not _stale():
        return OUT
    cmd = [nvcc(), *NVCC_FLAGS, "-o", OUT + ".tmp", os.path.join(CSRC, "geoattn.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True, capture_output=not verbose)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force=True, verbose=True))
