"""Build libotq.so in-tree with nvcc for sm_100a (no torch extension machinery: the library is
a plain C ABI, loaded with ctypes)."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
ROOT = PKG.parent
LIB = PKG / "libotq.so"
SOURCES = ["abi.cu", "quantize.cu", "quantize4.cu", "gemv.cu", "g32.cu", "prefill.cu", "argmax.cu"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-ftz=false", "-prec-div=true", "-prec-sqrt=true", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (Path(c).exists() or c == "nvcc"):
            return c
    raise RuntimeError("nvcc not found")


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile every .cu to an object (in parallel), then link the shared library."""
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    deps = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [ROOT / "include" / "otq.h"]
    newest_dep = max(p.stat().st_mtime for p in deps)
    procs = []
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = objdir / (s.stem + ".o")
        objs.append(o)
        if o.exists() and o.stat().st_mtime > max(s.stat().st_mtime, newest_dep):
            continue
        cmd = [nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"), "-c", str(s), "-o", str(o)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                            text=True)))
    for src, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode:
            sys.stdout.write(out)
        if p.returncode:
            raise RuntimeError(f"nvcc failed on {src}")
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(LIB),
               *map(str, objs), "-cudart", "static"]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIB)
