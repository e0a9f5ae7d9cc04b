"""openTPU's MX weight formats and its MM instruction restated in numpy (oracle; test
infrastructure only).

References (paths inside the reference project):
- formats and scale rows: `docs/isa.md` "Weight formats", `opentpu/quant.py:245-457`;
- quantizers: `opentpu/quant.py:316-524` (int8x, int4x / fp4x6, per-row nvfp4);
- MM: `docs/isa.md` "MM", `opentpu/isasim.py:749-910`, scalar model `tests/test_mx.py:131-151`;
- float64 emulation: `opentpu/quant.py:896-1067` (fake_act, fake_w, mx_matmul).
"""
from __future__ import annotations

import numpy as np

from . import fp32 as F

FORMATS = ("int8", "int4", "fp4", "nvfp4")          # WF 0..3 (isa.py:26-27)
WINDOW = {"int8": 16, "int4": 11, "fp4": 11, "nvfp4": 13}    # isa.py:28 MX_W
SUB = 4            # sub-blocks (QACT offset groups) per K-block (quant.py:261 NSUB)
NV_GROUPS = 8      # nvfp4 E4M3 groups per K-block (quant.py:262 NVG)
M_MAX = 63         # int4 / fp4 6-bit multiplier (quant.py:265 MMAX)
DW_MAX = 255
# nibble -> integer element (quant.py:257-259); E2M1 codes are stored as twice their value
NIBBLE = {
    "int4": np.array([0, 1, 2, 3, 4, 5, 6, 7, -8, -7, -6, -5, -4, -3, -2, -1], np.int8),
    "fp4": np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], np.int8),
}
NIBBLE["nvfp4"] = NIBBLE["fp4"]
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
E2M1_TOP, E4M3_TOP = 6.0, 448.0
# squared-error search factors around the round-to-nearest scale (quant.py:125 SEARCH)
SEARCH = np.linspace(0.64, 1.12, 13)


def _e4m3_grid() -> np.ndarray:
    """The 127 finite non-negative E4M3 values by code (quant.py:41-47)."""
    codes = np.arange(127)
    e, m = codes >> 3, codes & 7
    return np.where(e == 0, m / 8 * 2.0 ** -6, (1 + m / 8) * np.exp2(e - 7.0))


E4M3_VALUES = _e4m3_grid()


# ------------------------------------------------------------------------------ byte layouts
def row_bytes(K: int, fmt: str, D: int = 128) -> int:
    """Bytes of a streamed row (quant.py:287-289): K for int8, else whole D-byte chunks."""
    return K if fmt == "int8" else -(-K // (2 * D)) * D


def scale_bytes(K: int, fmt: str, D: int = 128, rsc: bool = False) -> int:
    """Bytes of a scale row (quant.py:292-309)."""
    if K % D:
        raise ValueError(f"K={K} is not a multiple of D={D}")
    KB = K // D
    if rsc:
        return 4
    if fmt == "int8":
        return 4 + 4 * -(-KB // 4)
    if fmt in ("int4", "fp4"):
        return 8 + 8 * -(-KB // 2)
    if fmt == "nvfp4":
        return 16 + 16 * -(-KB // 2)
    raise ValueError(f"unknown format {fmt!r}")


def nibbles(b) -> np.ndarray:
    """bytes [..., n] -> codes [..., 2n], low nibble first (quant.py:275-278)."""
    b = np.asarray(b, np.uint8)
    return np.stack([b & 15, b >> 4], axis=-1).reshape(*b.shape[:-1], 2 * b.shape[-1])


def pack_nibbles(codes) -> np.ndarray:
    """codes [..., 2n] -> bytes [..., n] (quant.py:281-284)."""
    c = np.asarray(codes, np.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


def elements(rows, fmt: str, K: int) -> np.ndarray:
    """The integers MM multiplies, [N, K] (quant.py:452-457)."""
    rows = np.asarray(rows, np.uint8)
    if fmt == "int8":
        return rows[:, :K].view(np.int8)
    return NIBBLE[fmt][nibbles(rows[:, :K // 2])]


def pack_scale_rows(fmt: str, Sw, dw=None, m=None, e4=None) -> np.ndarray:
    """Scale rows from Sw [N], offsets dw [N, KB], multipliers m [N, KB, 4] or E4M3 bytes
    e4 [N, KB, 8] (quant.py:403-426)."""
    Sw = np.asarray(Sw, np.float32).reshape(-1)
    N = Sw.shape[0]
    KB = (e4 if fmt == "nvfp4" else dw).shape[1]
    out = np.zeros((N, scale_bytes(KB, fmt, 1)), np.uint8)
    out[:, :4] = Sw.view(np.uint8).reshape(N, 4)
    if fmt == "int8":
        out[:, 4:4 + KB] = dw
    elif fmt in ("int4", "fp4"):
        w = np.asarray(dw, np.uint32).copy()
        for b in range(SUB):
            w |= np.asarray(m[:, :, b], np.uint32) << np.uint32(8 + 6 * b)
        out[:, 8:8 + 4 * KB] = w.view(np.uint8).reshape(N, 4 * KB)
    elif fmt == "nvfp4":
        e4 = np.asarray(e4, np.uint8)
        if (e4 & 0x80).any():
            raise ValueError("an NVFP4 scale with the sign bit set")
        out[:, 16:16 + 8 * KB] = e4.reshape(N, 8 * KB)
    else:
        raise ValueError(fmt)
    return out


def read_scales(srows, fmt: str, KB: int, k0: int = 0, rsc: bool = False, unit: bool = False,
                N: int | None = None):
    """What MM reads from the scale rows (isasim.py:706-745; quant.py:428-449): Sw [N] fp32,
    dw [N, KB, G] and m [N, KB, G] (G = 8 for nvfp4, else 4), blocks k0 .. k0+KB-1. UNIT reads
    nothing (Sw 1, dw 0, m 1; srows may be None)."""
    G = NV_GROUPS if fmt == "nvfp4" else SUB
    if unit:
        return (np.ones(N, np.float32), np.zeros((N, KB, G), np.int64),
                np.ones((N, KB, G), np.int64))
    srows = np.ascontiguousarray(srows, np.uint8)
    N = srows.shape[0]
    zeros = np.zeros((N, KB, G), np.int64)
    ones = np.ones((N, KB, G), np.int64)
    Sw = srows[:, :4].copy().view(np.float32).reshape(N)
    if rsc:
        return Sw, zeros, ones
    blocks = k0 + np.arange(KB)
    if fmt == "int8":
        dw = srows[:, 4 + blocks].astype(np.int64)
        return Sw, np.repeat(dw[:, :, None], G, axis=2), ones
    if fmt in ("int4", "fp4"):
        words = srows[:, 8:].copy().view(np.uint32)[:, blocks].astype(np.int64)
        dw = np.repeat((words & 0xFF)[:, :, None], G, axis=2)
        m = np.stack([(words >> (8 + 6 * b)) & 63 for b in range(G)], axis=-1)
        return Sw, dw, m
    e4 = srows[:, 16:].reshape(N, -1, NV_GROUPS)[:, blocks].astype(np.int64)
    E, Mt = (e4 >> 3) & 15, e4 & 7
    return Sw, 15 - np.maximum(E, 1), np.where(E > 0, 8 + Mt, Mt)


def dequantize(rows, srows, fmt: str, K: int, D: int = 128, rsc: bool = False) -> np.ndarray:
    """w * m * 2^-dw * Sw as float64 [N, K]; a denormal Sw reads as 0 (quant.py:460-473)."""
    w = elements(rows, fmt, K).astype(np.float64)
    N, KB = w.shape[0], K // D
    Sw, dw, m = read_scales(srows, fmt, KB, rsc=rsc)
    G = dw.shape[2]
    sc = m * np.exp2(-dw.astype(np.float64))
    Sw = np.where(np.abs(Sw) < F.TINY, 0.0, Sw.astype(np.float64))
    return (w.reshape(N, KB, G, D // G) * sc[..., None]).reshape(N, K) * Sw[:, None]


def weight_offsets(srows, fmt: str, K: int, D: int = 128, rsc: bool = False) -> np.ndarray:
    """dw per group of D/8 elements [N, K/(D/8)] (quant.py:476-481)."""
    _, dw, _ = read_scales(srows, fmt, K // D, rsc=rsc)
    return np.repeat(dw, NV_GROUPS // dw.shape[2], axis=2).reshape(dw.shape[0], -1)


# ------------------------------------------------------------------------------ quantizers
def _e2m1_index(v) -> np.ndarray:
    """Nearest E2M1 magnitude index of |v|, ties to the even index, saturating
    (quant.py:104-110)."""
    a = np.abs(v)
    return ((a > 0.25).astype(np.int8) + (a >= 0.75) + (a > 1.25) + (a >= 1.75) + (a > 2.5)
            + (a >= 3.5) + (a > 5.0))


def _nearest_on_grid(v, grid) -> np.ndarray:
    """Index of the nearest value of an ascending grid to |v|, ties to the even index,
    saturating at the top (quant.py:50-60)."""
    a = np.abs(v)
    hi = np.clip(np.searchsorted(grid, a), 1, len(grid) - 1)
    lo = hi - 1
    below, above = a - grid[lo], grid[hi] - a
    idx = np.where(below < above, lo, np.where(above < below, hi, np.where(lo % 2 == 0, lo, hi)))
    return np.where(a >= grid[-1], len(grid) - 1, idx)


def _snap(values, grid_name: str) -> np.ndarray:
    """Scaled values onto the element grid (quant.py:113-122)."""
    if grid_name == "int4":
        return np.clip(np.rint(values), -7, 7)
    return np.sign(values) * E2M1_VALUES[_e2m1_index(values)]


def _quantize_int8x(W, D):
    q, Sw, dw = F.quantize_rows(W, D)
    return q.view(np.uint8), pack_scale_rows("int8", Sw, dw=dw)


def _quantize_4bit(W, fmt, D):
    """int4x / fp4x6 (quant.py:325-367): per row Sw = the largest ideal sub-block scale / 63
    (fp32), per block the power-of-two offset, per sub-block the 6-bit multiplier the
    13-point squared-error search picks."""
    N, K = W.shape
    KB, sub = K // D, D // SUB
    grid = "int4" if fmt == "int4" else "e2m1"
    qmax = 7.0 if grid == "int4" else E2M1_TOP
    x = np.asarray(W, np.float64).reshape(N, KB, SUB, sub)
    ideal = np.abs(x).max(-1) / qmax                          # [N, KB, SUB]
    top = ideal.max(axis=(1, 2))
    Sw = np.where(top == 0, 1.0, top / M_MAX).astype(np.float32).astype(np.float64)
    bmax = ideal.max(-1)
    with np.errstate(divide="ignore"):
        d = np.floor(np.log2(M_MAX * Sw[:, None] / bmax))
    d = np.where(bmax > 0, np.clip(d, 0, DW_MAX), 0)
    unit = (Sw[:, None] * np.exp2(-d))[..., None]
    m0 = ideal / unit
    best = None
    for f in SEARCH:
        m = np.clip(np.rint(m0 * f), 1, M_MAX)
        s = (unit * m)[..., None]
        qv = _snap(x / s, grid) * s
        err = ((qv - x) ** 2).sum(-1)
        if best is None:
            best = [m, qv, err]
        else:
            better = err < best[2]
            best = [np.where(better, m, best[0]), np.where(better[..., None], qv, best[1]),
                    np.where(better, err, best[2])]
    m, qv, _ = best
    grid_vals = qv / (unit * m)[..., None]
    if grid == "int4":
        code = np.rint(grid_vals).astype(np.int64) & 15
        sw = Sw
    else:
        mag = _e2m1_index(grid_vals)
        code = mag | np.where(np.signbit(grid_vals) & (mag != 0), 8, 0)
        sw = Sw * 0.5
    rows = np.zeros((N, row_bytes(K, fmt, D)), np.uint8)
    rows[:, :K // 2] = pack_nibbles(code.reshape(N, K).astype(np.uint8))
    return rows, pack_scale_rows(fmt, sw.astype(np.float32), dw=d.astype(np.uint8),
                                 m=m.astype(np.uint8))


def _quantize_nvfp4(W, D):
    """nvfp4 with a per-row fp32 scale (quant.py:370-401)."""
    N, K = W.shape
    g = D // NV_GROUPS
    a = np.asarray(W, np.float64)
    ts = np.abs(a).max(-1, keepdims=True) / (E4M3_TOP * E2M1_TOP)
    ts = np.where(ts == 0, 1.0, ts).astype(np.float32).astype(np.float64)
    x = a.reshape(N, K // g, g) / ts[..., None]
    amax = np.abs(x).max(-1)
    best = None
    for f in SEARCH:
        s = E4M3_VALUES[_nearest_on_grid(amax * f / E2M1_TOP, E4M3_VALUES)]
        s = np.where((amax == 0) | (s == 0), 1.0, s)
        qv = np.sign(x) * E2M1_VALUES[_e2m1_index(x / s[..., None])] * s[..., None]
        err = ((qv - x) ** 2).sum(-1)
        if best is None:
            best = [s, qv, err]
        else:
            better = err < best[2]
            best = [np.where(better, s, best[0]), np.where(better[..., None], qv, best[1]),
                    np.where(better, err, best[2])]
    s, qv, _ = best
    vals = qv / s[..., None]
    mag = _e2m1_index(vals)
    code = (mag | np.where(np.signbit(vals) & (mag != 0), 8, 0)).reshape(N, K)
    e4 = _nearest_on_grid(s, E4M3_VALUES).reshape(N, K // D, NV_GROUPS)
    rows = np.zeros((N, row_bytes(K, "nvfp4", D)), np.uint8)
    rows[:, :K // 2] = pack_nibbles(code.astype(np.uint8))
    return rows, pack_scale_rows("nvfp4", (16 * ts[:, 0]).astype(np.float32),
                                 e4=e4.astype(np.uint8))


def quantize_weights(W, fmt: str, D: int = 128):
    """quant.quantize_mxu (quant.py:484-524): (rows [N, row_bytes], scale rows [N, scale_bytes])."""
    W = np.asarray(W, np.float32)
    if W.shape[1] % D:
        raise ValueError(f"K={W.shape[1]} is not a multiple of D={D}")
    if fmt == "int8":
        return _quantize_int8x(W, D)
    if fmt in ("int4", "fp4"):
        return _quantize_4bit(W, fmt, D)
    if fmt == "nvfp4":
        return _quantize_nvfp4(W, D)
    raise ValueError(f"unknown format {fmt!r}")


def quantize_rows_rsc(W):
    """BASELINE's int8 per-row weights: runtime.quantize_rows(W, D, row=True)
    (runtime.py:66-76) -- int8 rows and a 4-byte scale row (Sw alone, MM RSC)."""
    q, S, _ = F.quantize_rows(W, np.asarray(W).shape[1], row_mode=True)
    return q.view(np.uint8), S.astype(np.float32).view(np.uint8).reshape(-1, 4)


# ------------------------------------------------------------------------------ MM
def mm(q, Sa, da, rows, srows, fmt: str, K: int, *, D: int = 128, k0: int = 0,
       unit: bool = False, rsc: bool = False, out=None, acc: bool = False, alpha=None):
    """MM over one QACT range (docs/isa.md "MM"; isasim.py:749-910), exact.

    q int8 [M, K], Sa fp32 [M], da uint8 [M, K/(D/4)] (QACT's); rows / srows the weight's
    element and scale rows. Per output: acc = sum over groups of (m << sh) * c with
    sh = W - dw - da (dropped where sh < 0), then y = (i2f(acc) * Sw) * (Sa * 2^-W); with
    acc=True, y = out + y; with alpha, y = out * alpha[j] + y (ASCALE). Returns (y fp32
    [M, N], the integer accumulators int64 [M, N]).
    """
    q = np.asarray(q, np.int8)
    M = q.shape[0]
    N = np.asarray(rows).shape[0]
    KB = K // D
    W = WINDOW[fmt]
    Sw, dw, m = read_scales(srows, fmt, KB, k0=k0, rsc=rsc, unit=unit, N=N)
    G = dw.shape[2]
    w = elements(rows, fmt, K).astype(np.float64).reshape(N, KB, G, D // G)
    a = q.astype(np.float64).reshape(M, KB, G, D // G)
    da = np.asarray(da, np.int64).reshape(M, KB, SUB)
    da = np.repeat(da, G // SUB, axis=2)                                     # [M, KB, G]
    total = np.zeros((M, N), np.int64)
    for k in range(KB):
        for gi in range(G):
            c = np.rint(a[:, k, gi] @ w[:, k, gi].T).astype(np.int64)      # exact: < 2^19
            sh = W - dw[None, :, k, gi] - da[:, None, k, gi]                 # [M, N]
            B = np.where(sh >= 0, m[None, :, k, gi] << np.maximum(sh, 0), 0)
            total += B * c
    y = F.fmul(F.fmul(F.i2f(total), Sw[None, :]),
               F.fmul(np.asarray(Sa, np.float32)[:, None], np.float32(2.0 ** -W)))
    if alpha is not None:
        y = F.fadd(F.fmul(out, np.asarray(alpha, np.float32)[:, None]), y)
    elif acc:
        y = F.fadd(out, y)
    return y, total


def mm_plain(q, Sa, da, rows, srows, fmt: str, K: int, *, unit: bool = False,
             out=None, acc: bool = False):
    """MM for weights whose multipliers are 1 and offsets 0 (RSC or UNIT rows, any format): the
    same results as `mm`, by one float64 matrix product. With m = 1 and dw = 0 a group's
    multiplier 2^(W - da) depends on the activation alone, so the activation bytes are scaled by
    it (0 where the group is dropped) and acc = A' @ w^T: every product and every partial sum
    is an integer below 2^53 (|acc| <= 2^16 * 127 * 127 * K), so the float64 product is exact
    in any summation order. Returns (y fp32 [M, N], acc int64 [M, N])."""
    q = np.asarray(q, np.int8)
    M = q.shape[0]
    W = WINDOW[fmt]
    N = np.asarray(rows).shape[0]
    if (1 << W) * 127 * 127 * K >= 2 ** 53:
        raise ValueError("mm_plain: K too large for an exact float64 product")
    da = np.asarray(da, np.int64).reshape(M, K // 32)
    sh = W - da
    mult = np.where(sh >= 0, np.exp2(np.maximum(sh, 0).astype(np.float64)), 0.0)
    a = (q.astype(np.float64).reshape(M, K // 32, 32) * mult[..., None]).reshape(M, K)
    w = elements(rows, fmt, K).astype(np.float64)
    total = np.rint(a @ w.T).astype(np.int64)
    Sw = np.ones(N, np.float32) if unit else \
        np.ascontiguousarray(np.asarray(srows, np.uint8)[:, :4]).view(np.float32).reshape(N)
    y = F.fmul(F.fmul(F.i2f(total), Sw[None, :]),
               F.fmul(np.asarray(Sa, np.float32)[:, None], np.float32(2.0 ** -W)))
    if acc:
        y = F.fadd(out, y)
    return y, total


def qlinear(x, rows, srows, fmt: str, *, D: int = 128, rsc: bool = False, row_mode: bool = False,
            k0: int = 0):
    """QACT over the whole row (one range) followed by one MM: y fp32 [M, N]."""
    x = np.atleast_2d(np.asarray(x, np.float32))
    q, S, d = F.quantize_rows(x, D // SUB, row_mode)
    if rsc:
        return mm_plain(q, S, d, rows, srows, fmt, x.shape[1])[0]
    return mm(q, S, d, rows, srows, fmt, x.shape[1], D=D, rsc=rsc, k0=k0)[0]


# ------------------------------------------------------------------------------ emulation
def fake_act(x, D: int = 128, row: bool = False):
    """QACT's values in float64 with the offsets per D/8 (quant.py:972-1023), one range per
    row; a value within 2^-31 of a rounding tie rounds as the fp32 quantizer does."""
    x = np.asarray(x, np.float64)
    shape, K = x.shape, x.shape[-1]
    g = D // SUB
    xr = x.reshape(-1, K)
    amax = np.abs(xr).max(-1, keepdims=True)
    xb = xr.reshape(len(xr), K // g, g)
    gmax = np.abs(xb).max(-1)
    if row:
        d = np.zeros(gmax.shape, np.int64)
    else:
        with np.errstate(divide="ignore", invalid="ignore"):
            fa, ea = np.frexp(gmax)
            fm, em = np.frexp(np.broadcast_to(amax, gmax.shape))
        d = np.where(gmax > 0, np.clip(em - ea - (fa > fm), 0, 31), 0)
    s = np.where(amax == 0, 1.0, amax / 127)
    unit = s * np.exp2(-d)
    r = xb / unit[..., None]
    qv = np.rint(r)
    tie = np.abs(r - qv) > 0.5 - 2.0 ** -31
    if tie.any():
        rows_t = tie.any(-1).any(-1)
        exact = F.quantize_rows(xr[rows_t].astype(np.float32), g, row)[0].astype(np.float64)
        qv[rows_t] = np.where(tie[rows_t], exact.reshape(qv[rows_t].shape), qv[rows_t])
    vals = (np.clip(qv, -127, 127) * unit[..., None]).reshape(shape)
    da = np.repeat(d, g * NV_GROUPS // D, axis=-1).reshape(*shape[:-1], K // (D // NV_GROUPS))
    return vals, da


def mx_matmul(h, da, w, dw, W: int, D: int = 128):
    """h @ w.T in float64 with the groups MM's window drops left out (quant.py:1042-1067):
    h [M, K] QACT values with offsets da [M, K/(D/8)]; w [N, K] weight values with offsets dw
    [N, K/(D/8)]."""
    h = np.asarray(h, np.float64).reshape(-1, np.asarray(w).shape[1])
    y = h @ np.asarray(w, np.float64).T
    da = np.asarray(da, np.int64).reshape(h.shape[0], -1)
    dw = np.asarray(dw, np.int64)
    G = D // NV_GROUPS
    for gi in np.nonzero(da.max(0) + dw.max(0) > W)[0]:
        drop = (da[:, gi][:, None] + dw[None, :, gi]) > W
        if drop.any():
            sl = slice(G * gi, G * (gi + 1))
            y -= (h[:, sl] @ np.asarray(w, np.float64)[:, sl].T) * drop
    return y
