"""The reference's 4-bit group-32 fp16-scale weight format (its "survey" quantizer) restated in
numpy (oracle; test infrastructure only).

`quant.quantize(W, "int4", g=32, scale="fp16")` (opentpu/quant.py:225-227 -> quant_block
132-142 -> _quant_rows 144-170, fp16 rounding 94-99, element grid 119-122): per group of 32
elements of a row, s = fp16(min(amax / 7, 65504)) (1 where amax or s is 0), the element
w = clip(rint(x / s), -7, 7) and the dequantized value w * s. The reference returns only the
dequantized matrix and the scales (`codes` is empty, quant.py:242); the packed form used here
is two's-complement nibbles (element 2i in the low nibble, the convention of
quant.py:275-285) and the scales as fp16.
"""
from __future__ import annotations

import numpy as np

GROUP = 32


def quantize_g32(W):
    """(codes int8 [N, K] in [-7, 7], scales float16 [N, K/32], deq float32 [N, K])."""
    W = np.asarray(W, np.float32)
    N, K = W.shape
    if K % GROUP:
        raise ValueError(f"K={K} is not a multiple of {GROUP}")
    x = W.reshape(N, K // GROUP, GROUP).astype(np.float64)
    amax = np.abs(x).max(-1)
    s = np.minimum(amax * 1.0 / 7.0, 65504).astype(np.float16).astype(np.float64)
    s = np.where((amax == 0) | (s == 0), 1.0, s)
    codes = np.clip(np.rint(x / s[..., None]), -7, 7)
    deq = (codes * s[..., None]).reshape(N, K).astype(np.float32)
    return codes.reshape(N, K).astype(np.int8), s.astype(np.float16), deq


def pack_g32(codes) -> np.ndarray:
    """int8 codes [N, K] -> nibble bytes [N, K/2], element 2i in the low nibble."""
    c = (np.asarray(codes, np.int8).astype(np.int16) & 15).astype(np.uint8)
    return (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)


def unpack_g32(packed, K: int) -> np.ndarray:
    b = np.asarray(packed, np.uint8)
    c = np.stack([b & 15, b >> 4], -1).reshape(b.shape[0], -1)[:, :K].astype(np.int16)
    return np.where(c >= 8, c - 16, c).astype(np.int8)


def linear_g32(x, codes, scales) -> np.ndarray:
    """y = x @ deq.T in float64 (the reference's `deq @ x` pattern, tests/test_quant.py:276-287
    and reference.py:14-17): the tolerance oracle for the weight-only 4-bit GEMV."""
    codes = np.asarray(codes, np.float64)
    N, K = codes.shape
    deq = (codes.reshape(N, K // GROUP, GROUP)
           * np.asarray(scales, np.float64)[..., None]).reshape(N, K)
    return np.atleast_2d(np.asarray(x, np.float64)) @ deq.T
