"""The exact tensor-core MM's decomposition, checked on the CPU against the oracle's MM.

The reference's MM (opentpu/isasim.py:749-910) for RSC / UNIT weights accumulates, per output,
acc = sum over groups with d <= 16 of 2^(16 - d) * sum_k q_k w_k in exact integers. The
tensor-core path (csrc/w8a8.cu) instead scales each kept byte by 2^(D - d), D the row's largest
kept offset, splits it into balanced base-256 int8 planes, multiplies each plane with the
weights in int32, and recombines (c0 + 256 c1 + 65536 c2) * 2^(16 - D). This test restates that
decomposition in numpy and asserts it is the oracle's integer for every output, with the digit
ranges and int32 bounds the kernel relies on, on rows that need one, two and three planes,
dropped groups, zero groups and zero rows, and in QACT ROW mode."""
import numpy as np
import pytest

from oracle import fp32 as F
from oracle import mx as X


def _planes(q, d):
    """(planes [3, M, K] int64, D [M]) as the QACT-planes kernel builds them."""
    d = d.astype(np.int64)
    kept = d <= 16
    D = np.where(kept, d, 0).max(axis=1)
    sh = np.where(kept, D[:, None] - d, 0)
    a = np.where(np.repeat(kept, 32, axis=1),
                 q.astype(np.int64) * np.repeat(np.left_shift(1, sh), 32, axis=1), 0)
    out = []
    r = a
    for j in range(3):
        p = ((r + 128) & 255) - 128 if j < 2 else r
        out.append(p)
        r = (r - p) >> 8
    return np.stack(out), D


def _rows(rng, M, K, wide):
    x = rng.normal(0.0, 1.0, size=(M, K)).astype(np.float32)
    if wide:   # groups over 21 binades: offsets past 16 (dropped) and 3-plane rows
        g = K // 32
        sc = np.exp2(-rng.integers(0, 21, size=(M, g))).astype(np.float32)
        sc[:, 0] = 1.0
        x = (x.reshape(M, g, 32) * sc[..., None]).reshape(M, K)
        x[0, 32:64] = 0.0
        x[M // 2] = 0.0
    return x


@pytest.mark.parametrize("wide,row_mode", [(False, False), (True, False), (True, True)])
def test_planes_reproduce_the_reference_integer(wide, row_mode):
    rng = np.random.default_rng(11 + 2 * wide + row_mode)
    M, N, K = 24, 40, 640
    x = _rows(rng, M, K, wide)
    W = rng.normal(0.0, 0.02, size=(N, K)).astype(np.float32)
    rows, srows = X.quantize_rows_rsc(W)
    q, S, d = F.quantize_rows(x, 32, row_mode)
    _, acc_ref = X.mm_plain(q, S, d, rows, srows, "int8", K)
    planes, D = _planes(q, d)
    assert planes[:2].min() >= -128 and planes[:2].max() <= 127
    assert np.abs(planes[2]).max() <= 127
    w = rows[:, :K].view(np.int8).astype(np.int64)
    c = [p @ w.T for p in planes]
    assert max(np.abs(ci).max() for ci in c) < 2 ** 31   # each plane's MMA is an exact int32
    acc = (c[0] + 256 * c[1] + 65536 * c[2]) * np.left_shift(1, 16 - D)[:, None]
    assert np.array_equal(acc, acc_ref)
    counts = np.where(D == 0, 1, np.where(D <= 8, 2, 3))
    if row_mode:
        assert counts.max() == 1
    elif wide:
        assert counts.max() == 3
        assert (planes[2] != 0).any()
    else:
        assert counts.max() <= 2 and not (planes[2] != 0).any()
