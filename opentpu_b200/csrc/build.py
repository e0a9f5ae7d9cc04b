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
SOURCES = ["abi.cu", "quantize.cu", "quantize4.cu", "gemv.cu", "g32.cu", "prefill.cu", "w8a8.cu",
           "argmax.cu", "step.cu"]
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
               *map(str, objs), "-cudart", "static", "-Xlinker", "-soname=libotq.so"]
        subprocess.run(cmd, check=True)
    build_torch_ops(verbose)
    return LIB


TORCH_OPS = PKG / "libotq_torch.so"


def build_torch_ops(verbose: bool = False) -> Path:
    """torch.ops.otq.* (csrc/torch_ops.cpp): a C++ file against PyTorch's headers, linked to
    libotq.so (found next to it at run time) and to PyTorch's own libraries."""
    import torch
    src = CSRC / "torch_ops.cpp"
    deps = [src, ROOT / "include" / "otq.h", LIB]
    if TORCH_OPS.exists() and TORCH_OPS.stat().st_mtime > max(p.stat().st_mtime for p in deps):
        return TORCH_OPS
    tdir = Path(torch.__file__).resolve().parent
    cuda = Path(nvcc()).resolve().parent.parent if nvcc() != "nvcc" else Path("/usr/local/cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-I", str(tdir / "include"), "-I", str(tdir / "include" / "torch" / "csrc" / "api" /
                                                   "include"),
           "-I", str(cuda / "include"), str(src), "-o", str(TORCH_OPS),
           "-L", str(tdir / "lib"), "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_cuda", "-L", str(PKG), "-lotq", "-Wl,-rpath,$ORIGIN",
           f"-Wl,-rpath,{tdir / 'lib'}"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return TORCH_OPS


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIB)
