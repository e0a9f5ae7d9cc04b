"""torch.ops.otq.*: the quantized linear layer as registered PyTorch operators.

Importing this module loads libotq.so (by absolute path, through the ctypes binding, so the one
copy of the library holds the device status word) and then libotq_torch.so
(csrc/torch_ops.cpp, TORCH_LIBRARY(otq)), which registers, for CUDA tensors:

    torch.ops.otq.quantize_act(x, row_mode=False, group=32) -> (q, S, d)      QACT
    torch.ops.otq.mm(q, S, d, rows, srows, fmt, flags, K, k0=0) -> y           MM
    torch.ops.otq.qlinear(x, rows, srows, fmt, flags, K, k0=0, row_mode=False) -> y   QACT + MM
    torch.ops.otq.gemm_w8a16(x_bf16, rows, srows, flags) -> y                   prefill GEMM
    torch.ops.otq.linear_g32(x, codes, scales) -> y                             int4-g32 GEMV
    torch.ops.otq.argmax(x) -> index [1]                                        greedy token

fmt and flags are MM's WF codes and flag bits (linear.PackedWeight.mx_fmt / .flags give them
for a packed weight). The outputs come from PyTorch's allocator, so the ops can be captured in a
CUDA graph once each shape has run. There is no CPU kernel: CPU tensors raise.
"""
from __future__ import annotations

from pathlib import Path

import torch

from . import _lib

LIB = Path(__file__).resolve().parent / "libotq_torch.so"
_loaded = False


def load():
    """Register torch.ops.otq (idempotent); raises if the extension is not built."""
    global _loaded
    if _loaded:
        return
    _lib.load()
    if not LIB.exists():
        raise RuntimeError(f"{LIB} is missing: build it with `python -m opentpu_b200.csrc.build`")
    torch.ops.load_library(str(LIB))
    _loaded = True


def qlinear(x, w):
    """torch.ops.otq.qlinear (or linear_g32 for an int4-g32 weight) of a linear.PackedWeight."""
    load()
    if w.fmt == "int4-g32":
        return torch.ops.otq.linear_g32(x, w.rows, w.srows)
    from . import _lib as L
    return torch.ops.otq.qlinear(x, w.rows, w.srows, L.FMT[w.mx_fmt], w.flags, w.K, w.k0, False)


load()
