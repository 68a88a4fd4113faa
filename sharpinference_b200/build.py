"""Builds libsharpinfer_cuda.so in-tree for sm_100a (nvcc + g++, no JIT).

Usage: python -m sharpinference_b200.build [--force]
The shared library lands next to this file so it travels with the repo.
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OUT = HERE / "libsharpinfer_cuda.so"
BUILD = HERE / "_build"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
              "--expt-relaxed-constexpr", f"-I{INCLUDE}"]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math", "-Wall", "-Wextra",
             f"-I{CUDA_HOME / 'include'}", f"-I{INCLUDE}"]


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _fingerprint() -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*")) + list(INCLUDE.glob("*.h"))):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(ARCH + NVCC_FLAGS + CXX_FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False) -> Path:
    stamp = BUILD / "stamp"
    fp = _fingerprint()
    if OUT.exists() and stamp.exists() and stamp.read_text() == fp and not force:
        return OUT
    BUILD.mkdir(exist_ok=True)
    objs = []
    for src in _sources():
        obj = BUILD / (src.name + ".o")
        if src.suffix == ".cu":
            cmd = [NVCC, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        else:
            cmd = ["g++", *CXX_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = OUT.with_suffix(".so.tmp")
    link = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs,
            "-Xlinker", "--no-undefined", "-lpthread", "-ldl", "-lrt"]
    if verbose:
        print(" ".join(link), flush=True)
    subprocess.run(link, check=True)
    os.replace(tmp, OUT)
    stamp.write_text(fp)
    return OUT


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)
