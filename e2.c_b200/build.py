"""Build libe2cuda.so in-tree: sm_100a CUDA kernels (nvcc) + the C11 host library (gcc), one shared
library with the C ABI of include/e2cuda.h. The CUDA runtime is linked statically; the driver is
reached through cudaGetDriverEntryPoint, so the library needs only libcuda at run time.

    python e2.c_b200/build.py          # incremental (sources newer than their objects)
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libe2cuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cuda_home() -> Path:
    for c in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if c and (Path(c) / "bin" / "nvcc").exists():
            return Path(c)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    raise RuntimeError("nvcc not found")


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} {cmd[-1]}")


def build(verbose: bool = False) -> Path:
    cuda = _cuda_home()
    nvcc = str(cuda / "bin" / "nvcc")
    BUILD.mkdir(exist_ok=True)
    inc = [f"-I{CSRC}", f"-I{ROOT / 'include'}"]
    headers = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "e2cuda.h"]
    hdr_mtime = max(h.stat().st_mtime for h in headers)
    objs = []
    for src in sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.c")):
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_mtime):
            continue
        if src.suffix == ".cu":
            cmd = [nvcc, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
                   *inc, "-c", str(src), "-o", str(obj)]
        else:
            cmd = ["gcc", "-std=c11", "-O2", "-fPIC", "-Wall", "-Wextra", "-Wno-unused-parameter",
                   "-D_POSIX_C_SOURCE=200809L", f"-I{cuda / 'include'}", *inc, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        _run(cmd)
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        _run([nvcc, *ARCH, "-shared", "-cudart=static", "-o", str(LIB), *map(str, objs), "-lrt", "-ldl", "-lpthread"])
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
