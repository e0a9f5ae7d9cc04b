"""`opentpu.quant`'s call surface for the quantized linear layer, backed by this library.

The reference's LLM runtime and its CPU goldens reach the quantized linear layer through
`opentpu.quant` (reference opentpu/quant.py): the quantizers (`quantize` :208, `quantize_mxu`
:510, `quantize_mx` :484), the byte layouts (`row_bytes` :287, `scale_bytes` :292, `pack4` :281,
`unpack4` :275, `pack_scales` :403, `unpack_scales` :428, `elements` :452, `group_offsets` :476),
the decoder `dequantize_mxu` :460 and the float64 emulation of MM (`MXAct`/`MXW` :896-960,
`fake_w` :963, `fake_act` :972, `mx_matmul` :1042). This module has the same names, signatures,
return types (numpy in, numpy out) and ValueErrors, so `from opentpu_b200 import quant as Q`
stands in for `from opentpu import quant as Q` on this path.

Where the work is:
- the quantizers run on the GPU (otq_quantize_mxu, otq_pack_int8, otq_pack_g32,
  otq_quantize_rows): bytes identical to the reference's;
- `dequantize_mxu`, `fake_act` and `mx_matmul` evaluate the reference's float64 definitions on
  the GPU (torch float64 tensors on the current CUDA device; `fake_act`'s near-tie rows take the
  device QACT's bytes, as the reference takes fp32.quantize_mx's); float64 sums on the GPU
  add in another order than numpy's BLAS, so `mx_matmul` agrees with the reference to float64
  rounding, the rest bit for bit;
- the byte-layout helpers (`pack4`, `unpack4`, `pack_scales`, `unpack_scales`, `elements`,
  `row_bytes`, `scale_bytes`, `group_offsets`) are format definitions: numpy reshapes and
  bit operations of the reference's layout, used by callers to build or inspect images.

Formats `quantize` takes here: "int8" (an fp32 scale per g, g a multiple of 32), "int4" with
g = 32 and scale "fp16" (the 4-bit group-32 format of this path), and the MX formats "mx-int8",
"mx-int4", "mx-fp4", "mx-nvfp4". The reference's other survey formats (mxfp4, e2m1, int4 with
other scales, int4k, ...) are not on this path and raise ValueError. Every GPU entry point takes
D = 128 (the MXU's D). No CPU fallback: without a CUDA device the GPU-backed calls raise.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)
E2M1_MAX = 6.0
E4M3_MAX = 448.0


def _e4m3_table() -> np.ndarray:
    c = np.arange(127)
    e, m = c >> 3, c & 7
    return np.where(e == 0, m / 8 * 2.0 ** -6, (1 + m / 8) * np.exp2(e - 7.0)).astype(np.float64)


E4M3 = _e4m3_table()                   # the 127 finite non-negative E4M3 values by code
SCALE_BITS = {"fp32": 32, "fp16": 16, "bf16": 16, "e4m3": 8, "e8m0": 8}
QMAX = {"int4": 7.0, "e2m1": E2M1_MAX}
SEARCH = np.linspace(0.64, 1.12, 13)   # the MX quantizers' scale candidates (quant.py:125)
MX_NUMERICS = "mx1"
DEC_INT4 = np.array([0, 1, 2, 3, 4, 5, 6, 7, -8, -7, -6, -5, -4, -3, -2, -1], np.int8)
DEC_FP4 = np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], np.int8)
DEC = {"int4": DEC_INT4, "fp4": DEC_FP4, "nvfp4": DEC_FP4}
NSUB = 4                               # QACT offsets / 4-bit multipliers a K-block
NVG = 8                                # nvfp4 E4M3 groups a K-block
MXU_FORMATS = ("int8", "int4", "fp4", "nvfp4")
FOUR = ("int4", "fp4", "nvfp4")
MMAX = 63
DW_MAX = 255
MX_W = {"int8": 16, "int4": 11, "fp4": 11, "nvfp4": 13}   # MM's window (isa.py:28 MX_W)


class NotExact(ValueError):
    """A checkpoint's quantized weights that no MXU format holds exactly (quant.py:1071)."""


@dataclass
class Quantized:
    fmt: str
    deq: np.ndarray           # dequantized [N, K] fp32
    codes: np.ndarray         # element codes [N, K] (int8 values, or 4-bit codes)
    scales: np.ndarray        # block scales [N, K // g] (as values, fp64)
    g: int
    bits: float               # storage bits per weight (elements + block scales)


# ------------------------------------------------------------------------------ GPU plumbing
def _torch():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("opentpu_b200.quant: this call runs on the GPU and no CUDA device is "
                           "visible (there is no CPU implementation)")
    return torch


def _dev(a, dtype=None):
    torch = _torch()
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def _host(t) -> np.ndarray:
    return t.cpu().numpy()


def _need_d128(D: int, what: str):
    if D != 128:
        raise ValueError(f"{what}: this library's MX entry points take D = 128 (got {D})")


# ------------------------------------------------------------------------------ byte layouts
def unpack4(b: np.ndarray) -> np.ndarray:
    """Bytes [..., n] -> nibble codes [..., 2n], the low nibble first."""
    b = np.asarray(b, np.uint8)
    return np.stack([b & 15, b >> 4], -1).reshape(*b.shape[:-1], 2 * b.shape[-1])


def pack4(codes: np.ndarray) -> np.ndarray:
    """Nibble codes [..., 2n] (0..15) -> bytes [..., n]."""
    c = np.asarray(codes, np.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


def row_bytes(K: int, fmt: str, D: int = 128) -> int:
    """DRAM bytes of one streamed row of K elements (4-bit rows padded to whole D-byte chunks)."""
    return K if fmt == "int8" else -(-K // (2 * D)) * D


def scale_bytes(K: int, fmt: str, D: int = 128, rsc: bool = False) -> int:
    """Bytes of one weight row's scale row: Sw, then int8 a byte a block, int4 / fp4 a reserved
    word and a word a block, nvfp4 three reserved words and eight bytes a block, padded to 4, 8
    or 16 bytes. rsc: Sw alone."""
    if K % D:
        raise ValueError(f"inner dimension {K} is not a multiple of D={D}")
    KB = K // D
    if rsc:
        return 4
    if fmt == "int8":
        return 4 + 4 * -(-KB // 4)
    if fmt in ("int4", "fp4"):
        return 8 + 8 * -(-KB // 2)
    if fmt == "nvfp4":
        return 16 + 16 * -(-KB // 2)
    raise ValueError(f"unknown MXU format {fmt!r}")


def pack_scales(fmt: str, Sw, dw=None, m=None, e4=None) -> np.ndarray:
    """Scale rows [N, scale_bytes] (uint8) of Sw [N] and the blocks' offsets dw [N, KB],
    multipliers m [N, KB, NSUB] (int4, fp4) or E4M3 bytes e4 [N, KB, NVG] (nvfp4)."""
    Sw = np.asarray(Sw, np.float32).reshape(-1)
    N = len(Sw)
    KB = (e4 if fmt == "nvfp4" else dw).shape[1]
    out = np.zeros((N, scale_bytes(KB, fmt, 1)), np.uint8)
    out[:, :4] = Sw[:, None].view(np.uint8)
    if fmt == "int8":
        out[:, 4:4 + KB] = dw
    elif fmt in ("int4", "fp4"):
        word = np.asarray(dw, np.uint32)
        for b in range(NSUB):
            word = word | (np.asarray(m[..., b], np.uint32) << np.uint32(8 + 6 * b))
        out[:, 8:8 + 4 * KB] = word.astype(np.uint32).view(np.uint8).reshape(N, 4 * KB)
    elif fmt == "nvfp4":
        if np.any(np.asarray(e4) & 0x80):
            raise ValueError("an NVFP4 scale with the sign bit set")
        out[:, 16:16 + 8 * KB] = np.asarray(e4, np.uint8).reshape(N, 8 * KB)
    else:
        raise ValueError(f"unknown MXU format {fmt!r}")
    return out


def unpack_scales(srows: np.ndarray, fmt: str, KB: int, k0: int = 0, rsc: bool = False):
    """What MM reads from scale rows: Sw [N] fp32 and, per (row, block k0 .. k0 + KB - 1,
    group), the offset dw and multiplier m [N, KB, G] (G = NVG for nvfp4, else NSUB)."""
    srows = np.ascontiguousarray(srows, np.uint8)
    N = srows.shape[0]
    G = NVG if fmt == "nvfp4" else NSUB
    Sw = srows[:, :4].copy().view(np.float32)[:, 0]
    if rsc:
        return Sw, np.zeros((N, KB, G), np.int64), np.ones((N, KB, G), np.int64)
    kk = k0 + np.arange(KB)
    if fmt == "int8":
        dw = np.repeat(srows[:, 4 + kk].astype(np.int64)[:, :, None], G, axis=2)
        return Sw, dw, np.ones((N, KB, G), np.int64)
    if fmt in ("int4", "fp4"):
        word = srows[:, 8:].copy().view(np.uint32)[:, kk].astype(np.int64)
        dw = np.repeat((word & 0xFF)[:, :, None], G, axis=2)
        return Sw, dw, np.stack([(word >> (8 + 6 * b)) & 63 for b in range(G)], -1)
    if fmt != "nvfp4":
        raise ValueError(f"unknown MXU format {fmt!r}")
    e4 = srows[:, 16:].reshape(N, -1, NVG)[:, kk].astype(np.int64)
    E, M = (e4 >> 3) & 15, e4 & 7
    return Sw, 15 - np.maximum(E, 1), np.where(E > 0, 8 + M, M)


def elements(rows: np.ndarray, fmt: str, K: int) -> np.ndarray:
    """The integer elements w [N, K] MM multiplies (int8; 4-bit codes decoded)."""
    rows = np.asarray(rows, np.uint8)
    if fmt == "int8":
        return rows[:, :K].view(np.int8)
    if fmt not in DEC:
        raise ValueError(f"unknown MXU format {fmt!r}")
    return DEC[fmt][unpack4(rows[:, :K // 2])]


def group_offsets(srows: np.ndarray, fmt: str, K: int, D: int = 128,
                  rsc: bool = False) -> np.ndarray:
    """Each group of D/8 elements' weight offset dw [N, K / (D/8)] (MM's drop rule)."""
    _, dw, _ = unpack_scales(srows, fmt, K // D, rsc=rsc)
    return np.repeat(dw, NVG // dw.shape[2], axis=2).reshape(dw.shape[0], -1)


# ------------------------------------------------------------------------------ GPU decode
def dequantize_mxu(rows: np.ndarray, srows: np.ndarray | None, fmt: str, K: int,
                   D: int = 128, rsc: bool = False) -> np.ndarray:
    """The matrix [N, K] (float64) that MXU rows and their scale rows stand for, w m 2^-dw Sw
    (srows None: UNIT, the elements). A denormal Sw is 0. Evaluated on the GPU; every product
    is exact in float64, so the result is the reference's bit for bit."""
    torch = _torch()
    w = _dev(elements(rows, fmt, K), torch.float64)
    if srows is None:
        return _host(w)
    N, KB = w.shape[0], K // D
    Sw, dw, m = unpack_scales(srows, fmt, KB, rsc=rsc)
    G = dw.shape[2]
    sc = _dev(m, torch.float64) * torch.exp2(-_dev(dw, torch.float64))
    sw = np.where(np.abs(Sw) < np.float32(2.0 ** -126), 0.0, Sw.astype(np.float64))
    out = (w.reshape(N, KB, G, D // G) * sc[..., None]).reshape(N, K) * _dev(sw)[:, None]
    return _host(out)


# ------------------------------------------------------------------------------ quantizers
def _gpu_mx(W: np.ndarray, fmt: str):
    """quantize_mx of W on the GPU: (rows [N, row_bytes], scale rows [N, scale_bytes])."""
    torch = _torch()
    from . import linear
    W = np.asarray(W, np.float32)
    w = linear.PackedWeight.from_float(_dev(W), fmt)
    N, K = W.shape
    rows = _host(w.rows)[:, :row_bytes(K, fmt)]
    srows = _host(w.srows)[:, :scale_bytes(K, fmt)]
    torch.cuda.synchronize()
    return np.ascontiguousarray(rows), np.ascontiguousarray(srows)


def quantize_mx(W: np.ndarray, fmt: str, D: int = 128):
    """W [N, K] in an MXU format: (element bytes [N, row_bytes], scale rows [N, scale_bytes]),
    every row on its own, quantized on the GPU (the reference's bytes)."""
    W = np.asarray(W, np.float32)
    N, K = W.shape
    if K % D:
        raise ValueError(f"inner dimension {K} is not a multiple of D={D}")
    if fmt not in MXU_FORMATS:
        raise ValueError(f"unknown MXU format {fmt!r}")
    _need_d128(D, "quantize_mx")
    return _gpu_mx(W, fmt)


QUANT_ROWS = 1 << 14


def quantize_mxu(W: np.ndarray, fmt: str, D: int = 128) -> tuple[np.ndarray, np.ndarray]:
    """W [N, K] in an MXU weight format ("int8", "int4", "fp4" or "nvfp4"): the DRAM rows
    [N, row_bytes] (uint8) and the scale rows [N, scale_bytes] (uint8). Rows are quantized on
    their own, QUANT_ROWS at a time (bounded device temporaries)."""
    W = np.asarray(W, np.float32)
    N = W.shape[0]
    if N <= QUANT_ROWS:
        return quantize_mx(W, fmt, D)
    parts = [quantize_mx(W[i:i + QUANT_ROWS], fmt, D) for i in range(0, N, QUANT_ROWS)]
    return np.concatenate([p[0] for p in parts]), np.concatenate([p[1] for p in parts])


def quantize(W: np.ndarray, fmt: str, g: int | None = None, scale: str | None = None,
             search: bool = False, rule: str = "rtn") -> Quantized:
    """Quantize-dequantize W [N, K] (quant.py:208): "int8" with an fp32 scale per g (default
    128; g = K is the int8 per-row format), "int4" with g = 32 and an fp16 scale (the 4-bit
    group-32 format), or an MX format "mx-int8" / "mx-int4" / "mx-fp4" / "mx-nvfp4". The codes
    and scales come from the GPU quantizers, bit-identical to the reference's."""
    torch = None
    W = np.asarray(W, np.float32)
    if fmt.startswith("mx-"):
        f, K = fmt[3:], W.shape[1]
        rows, srows = quantize_mxu(W, f)
        deq = dequantize_mxu(rows, srows, f, K).astype(np.float32)
        return Quantized(fmt, deq, elements(rows, f, K), srows, 128,
                         8 * (row_bytes(K, f) + scale_bytes(K, f)) / K)
    if fmt == "int8":
        g = g or 128
        N, K = W.shape
        if K % g:
            raise ValueError(f"inner dimension {K} is not a multiple of the block size {g}")
        if g % 32 or g > 32768:
            raise ValueError(f"int8 groups of {g}: this library quantizes groups of a multiple "
                             f"of 32 elements up to 32768")
        torch = _torch()
        from . import linear
        x = _dev(W).reshape(-1, g)
        q, S, _ = linear.quantize_act(x, row_mode=True, group=g)
        deq = (q.float() * S[:, None]).reshape(N, K)
        return Quantized(fmt, _host(deq), _host(q).reshape(N, K),
                         _host(S).reshape(N, K // g).astype(np.float64), g, 8 + 32 / g)
    if fmt == "int4":
        g, scale = g or 32, scale or "fp16"
        if g != 32 or scale != "fp16" or search:
            raise ValueError("int4: this library implements the group-32 fp16-scale format "
                             "(g=32, scale='fp16', search=False)")
        N, K = W.shape
        if K % g:
            raise ValueError(f"inner dimension {K} is not a multiple of the block size {g}")
        torch = _torch()
        from . import linear
        w = linear.PackedWeight.from_float(_dev(W), "int4-g32")
        b = w.rows.to(torch.int16)
        lo, hi = b & 15, b >> 4
        codes = torch.stack([lo, hi], -1).reshape(N, K)
        codes = torch.where(codes >= 8, codes - 16, codes).to(torch.float64)
        s = w.srows.to(torch.float64)
        deq = (codes.reshape(N, K // 32, 32) * s[..., None]).reshape(N, K)
        # an element that rounds to 0 keeps the sign of rint(x / s), i.e. of x (the reference's
        # clip(rint(x / s)) * s in float64)
        deq = torch.where(codes == 0, torch.copysign(torch.zeros_like(deq),
                                                     _dev(W).to(torch.float64)), deq).float()
        return Quantized(fmt, _host(deq), np.zeros(0), _host(s), g, 4 + SCALE_BITS[scale] / g)
    raise ValueError(f"unknown format {fmt!r}" if fmt not in ("mxfp4", "nvfp4", "e2m1", "int4k",
                                                              "e2m1k")
                     else f"format {fmt!r} is not on this library's path (int8, int4 g32 fp16, "
                          f"mx-*)")


# ------------------------------------------------------------------------------ emulation
class MXAct(np.ndarray):
    """Activations as QACT leaves them (float64 values) with `da`, each group of D/8 elements'
    power-of-two offset [..., K / (D/8)] (MM's drop rule; mx_matmul). Arrays derived from one
    are plain arrays (da None)."""

    def __array_finalize__(self, obj):
        self.da = None

    @staticmethod
    def of(values, da) -> "MXAct":
        a = np.asarray(values).view(MXAct)
        a.da = None if da is None else np.asarray(da)
        return a

    def rows(self, sl) -> "MXAct":
        return MXAct.of(np.asarray(self).view(np.ndarray)[sl],
                        None if self.da is None else self.da[sl])


class MXW(np.ndarray):
    """A weight as the MXU holds it: values [N, K] with the groups' offsets dw and the window W;
    w @ h (h [K]) and h @ w.T sum as MM does (mx_matmul, on the GPU). Anything else derived
    from it is a plain array."""

    def __array_finalize__(self, obj):
        self.mx = None                  # (dw, W, D, transposed)

    @staticmethod
    def of(values, dw, W: int, D: int = 128) -> "MXW":
        v = np.asarray(values)
        w = (v if v.dtype in (np.float32, np.float64) else v.astype(np.float64)).view(MXW)
        w.mx = (np.asarray(dw), W, D, False)
        return w

    def astype(self, dtype, *a, **kw):
        if self.mx is not None and not self.mx[3]:
            return MXW.of(np.asarray(self).view(np.ndarray).astype(dtype, *a, **kw), self.mx[0],
                          self.mx[1], self.mx[2])
        return np.asarray(self).view(np.ndarray).astype(dtype, *a, **kw)

    @property
    def T(self):
        t = np.ndarray.transpose(self).view(MXW)
        if self.mx is not None:
            dw, W, D, tr = self.mx
            t.mx = (dw, W, D, not tr)
        return t

    def __array_ufunc__(self, ufunc, method, *inputs, **kw):
        if ufunc is np.matmul and method == "__call__" and not kw and len(inputs) == 2:
            a, b = inputs
            if isinstance(b, MXW) and b.mx is not None and b.mx[3]:          # h @ w.T
                dw, W, D, _ = b.mx
                return mx_matmul(a, np.asarray(b).view(np.ndarray).T, dw, W, D)
            if isinstance(a, MXW) and a.mx is not None and not a.mx[3] and np.ndim(b) == 1:
                dw, W, D, _ = a.mx                                             # w @ h
                return mx_matmul(b, np.asarray(a).view(np.ndarray), dw, W, D)
        args = [np.asarray(x).view(np.ndarray) if isinstance(x, np.ndarray) else x
                for x in inputs]
        if "out" in kw:
            kw["out"] = tuple(np.asarray(o).view(np.ndarray) for o in kw["out"])
        return getattr(ufunc, method)(*args, **kw)


def fake_w(W: np.ndarray, fmt: str, D: int = 128, quantized: tuple | None = None) -> MXW:
    """W [N, K] as the MXU holds it in format fmt (quantize_mxu on the GPU, dequantized;
    `quantized`: its (rows, scale rows) already): an MXW."""
    rows, srows = quantize_mxu(W, fmt, D) if quantized is None else quantized
    K = np.asarray(W).shape[1]
    return MXW.of(dequantize_mxu(rows, srows, fmt, K, D), group_offsets(srows, fmt, K, D),
                  MX_W[fmt], D)


def fake_act(x, D: int = 128, n: int | None = None, row: bool = False,
             g: int | None = None):
    """x [..., K] quantized as QACT / QST quantize it, in float64 (quant.py:972-1023): per range
    of n columns (default the whole row; a sequence: the ranges' widths) S = amax / 127, per
    group of g (default D/4) the offset d (0 with row), values rint(x 127 / amax 2^d) S 2^-d
    clipped to 127; a value within 2^-31 of a rounding tie takes the device QACT's byte (the
    fp32 quantizer). Evaluated on the GPU in float64. Returns an MXAct (da per D/8)."""
    torch = _torch()
    from . import linear
    x = np.asarray(x, np.float64)
    sh = x.shape
    K = sh[-1]
    if n is not None and not isinstance(n, (int, np.integer)):        # ranges of their own
        if sum(n) != K:
            raise ValueError(f"fake_act: ranges {list(n)} over {K} columns")
        c, parts = 0, []
        for w in n:
            parts.append(fake_act(x[..., c:c + w], D, None, row, g))
            c += w
        out = np.concatenate([np.asarray(p).view(np.ndarray) for p in parts], -1).view(MXAct)
        out.da = np.concatenate([p.da for p in parts], -1)
        return out
    n = K if n is None else n
    g = D // NSUB if g is None else g
    if K % n or n % g:
        raise ValueError(f"fake_act: ranges of {n} over {K} columns, groups of {g}")
    xr = _dev(x.reshape(-1, n))
    amax = xr.abs().amax(-1, keepdim=True)
    xb = xr.reshape(xr.shape[0], n // g, g)
    ag = xb.abs().amax(-1)
    if row:
        d = torch.zeros(ag.shape, dtype=torch.int64, device=ag.device)
    else:
        fa, ea = torch.frexp(ag)
        fm, em = torch.frexp(amax.expand_as(ag))
        d = torch.where(ag > 0, torch.clamp(em.long() - ea.long() - (fa > fm).long(), 0, 31),
                        torch.zeros((), dtype=torch.int64, device=ag.device))
    # a tensor divisor: PyTorch turns division by a Python scalar into a multiplication by its
    # reciprocal, which is not the reference's correctly rounded amax / 127
    s = torch.where(amax == 0, torch.ones_like(amax), amax / torch.full_like(amax, 127.0))
    unit = s * torch.exp2(-d.to(torch.float64))
    r = xb / unit[..., None]
    q = torch.round(r)                                   # half to even, as numpy's rint
    tie = (r - q).abs() > 0.5 - 2.0 ** -31
    if bool(tie.any()):
        b = tie.any(-1).any(-1)
        if n % 32 or g % 32 or n > 32768:
            raise ValueError(f"fake_act: a near-tie row in ranges of {n}, groups of {g}: the "
                             f"device quantizer takes multiples of 32 up to 32768")
        qd, _, _ = linear.quantize_act(xr[b].float(), row_mode=row, group=g)
        qd = qd.to(torch.float64).reshape(q[b].shape)
        q[b] = torch.where(tie[b], qd, q[b])
    vals = (torch.clamp(q, -127, 127) * unit[..., None]).reshape(sh)
    da = d.repeat_interleave(g * NVG // D, dim=-1).reshape(*sh[:-1], K // (D // NVG))
    # the reference's offsets are frexp's int32 exponents (row mode: an int64 zero array)
    return MXAct.of(_host(vals), _host(da).astype(np.int64 if row else np.int32))


def mx_matmul(h, w: np.ndarray, dw: np.ndarray | None = None, W: int = 16,
              D: int = 128) -> np.ndarray:
    """h @ w.T (float64, on the GPU) as MM sums it: w [N, K] the streamed matrix's values with
    its groups' offsets dw [N or 1, K / (D/8)] (None: 0) and the window W; h an MXAct (a plain
    array: nothing dropped), the groups whose two offsets add up to more than W left out."""
    torch = _torch()
    hv = np.asarray(h).view(np.ndarray)
    wt = _dev(np.asarray(w), torch.float64)
    hd = _dev(hv, torch.float64)
    y = hd @ wt.T
    da = getattr(h, "da", None)
    if da is None:
        return _host(y)
    K = wt.shape[1]
    dwn = np.zeros((1, K // (D // NVG)), np.int64) if dw is None else np.asarray(dw, np.int64)
    hr = hd.reshape(-1, K)
    dg = np.asarray(da).reshape(-1, dwn.shape[1])
    yf = y.reshape(-1, wt.shape[0])
    G = D // NVG
    dwmax = dwn.max(0)
    dwt = _dev(dwn)
    for gi in np.nonzero(dg.max(0) + dwmax > W)[0]:
        rows = np.nonzero(dg[:, gi] + dwmax[gi] > W)[0]
        rt = _dev(rows)
        m = (_dev(dg[rows, gi])[:, None] + dwt[None, :, gi]) > W
        if not bool(m.any()):
            continue
        sl = slice(G * int(gi), G * (int(gi) + 1))
        yf[rt] -= (hr[rt, sl] @ wt[:, sl].T) * m
    return _host(y)
