"""The prefill linear layer on bf16 activations restated in numpy (oracle; test infrastructure
only).

BASELINE configuration 4 runs the int8 per-row weights of `quant.quantize(W, "int8", g=K)`
(opentpu/quant.py:218-224; bytes as runtime.quantize_rows(W, D, row=True), runtime.py:66-76)
against bf16 activations. The reference has no bf16 path of its own: its float model of the
layer is `deq @ x` (opentpu/reference.py:14-17, the pattern of tests/test_quant.py:276-287), and
that is what this evaluates, in float64, with x taken exactly as its bf16 values.
"""
from __future__ import annotations

import numpy as np


def bf16_round(x) -> np.ndarray:
    """fp32 -> the nearest bf16 (ties to even), returned as float32 (the bf16 values exactly)."""
    b = np.ascontiguousarray(np.asarray(x, np.float32)).view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def deq_rows(rows, srows, K: int, unit: bool = False) -> np.ndarray:
    """int8-row bytes -> the dequantized float64 weight q * Sw [N, K] (Sw = 1 with UNIT)."""
    q = np.asarray(rows)[:, :K].view(np.int8).astype(np.float64)
    if unit:
        return q
    sw = np.ascontiguousarray(np.asarray(srows)[:, :4]).view(np.float32).astype(np.float64)
    return q * sw


def gemm_w8a16(x, rows, srows, K: int, unit: bool = False):
    """(y, bound): y = x @ deq^T in float64 and the magnitude |x| @ |deq|^T that an fp32
    accumulation's error is measured against (x: the bf16 values as float32, [M, K])."""
    x = np.asarray(x, np.float64)
    d = deq_rows(rows, srows, K, unit)
    return x @ d.T, np.abs(x) @ np.abs(d).T
