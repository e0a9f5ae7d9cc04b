"""openTPU fp32 arithmetic restated in numpy (oracle; test infrastructure only).

Rules (reference `docs/isa.md` "Arithmetic (fp32)", implemented in `opentpu/fp32.py:1-101`):
- binary32 values, every add / sub / mul rounds to nearest even;
- denormal operands are read as signed zeros and a denormal result becomes a signed zero,
  where "denormal result" means IEEE rounding onto the subnormal grid gave a denormal (a
  product that rounds up to 2^-126 is kept: `tests/test_fp.py:214`);
- every NaN an operation produces is the canonical 0x7FC00000.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
U32 = np.uint32
TINY = F32(2.0 ** -126)          # smallest normal
QNAN = U32(0x7FC00000)
ONE_OVER_127 = F32(1.0 / 127.0)   # the reference's INV127 (fp32.py:28)
RECIP_SEED = 0x7EF311C3           # fp32.py:29; docs/isa.md recip
OFFSET_MAX = 31                   # fp32.py:310 MX_DMAX


def as_f32(x) -> np.ndarray:
    return np.asarray(x, dtype=F32)


def to_bits(x) -> np.ndarray:
    return as_f32(x).view(U32)


def of_bits(b) -> np.ndarray:
    return np.asarray(b, dtype=U32).view(F32)


def flush(x) -> np.ndarray:
    """Denormals -> zero of the same sign; NaN bits kept (fp32.py:45-54)."""
    b = to_bits(x)
    den = ((b & U32(0x7F800000)) == 0) & ((b & U32(0x7FFFFFFF)) != 0)
    if not den.any():
        return as_f32(x)
    return of_bits(np.where(den, b & U32(0x80000000), b)).copy()


def _canonical(x) -> np.ndarray:
    x = as_f32(x)
    nan = np.isnan(x)
    if nan.any():
        return np.where(nan, of_bits(QNAN), x).astype(F32)
    return x


def _op(f, a, b) -> np.ndarray:
    with np.errstate(all="ignore"):
        return _canonical(flush(f(flush(a), flush(b)).astype(F32)))


def fmul(a, b):
    """mul (fp32.py:100-101): flushed operands, IEEE product, flushed result."""
    return _op(np.multiply, a, b)


def fadd(a, b):
    """add (fp32.py:92-93)."""
    return _op(np.add, a, b)


def fsub(a, b):
    """sub (fp32.py:96-97)."""
    return _op(np.subtract, a, b)


def magnitude_bits(x) -> np.ndarray:
    """|flush(x)| as its bit pattern (the quantizer's unsigned compare of x[30:0])."""
    return to_bits(flush(x)) & U32(0x7FFFFFFF)


def i2f(acc) -> np.ndarray:
    """int64 -> fp32, round to nearest even (fp32.py:162-164)."""
    return np.asarray(acc, dtype=np.int64).astype(F32)


def _bump_exponent(y, k) -> np.ndarray:
    """y * 2^k by adding k to the exponent field (fp32.py:227-229)."""
    return of_bits((to_bits(y).astype(np.int64) + (np.asarray(k, np.int64) << 23)).astype(U32))


def recip(x) -> np.ndarray:
    """openTPU's reciprocal (docs/isa.md "recip"; fp32.py:242-261).

    The significand a in [1, 2) gets the magic seed, two Newton steps y*(2 - a*y), then the
    correction step y*(1 - a*y) + y, every op a flushed RNE op; the exponent is put back by
    adding 127 - field(x) to y's exponent field and x's sign is or-ed in. Zero gives +0 and
    |x| >= 2^126 (infinities and NaNs included) a zero with x's sign.
    """
    xb = to_bits(flush(x))
    mag = xb & U32(0x7FFFFFFF)
    sign = xb & U32(0x80000000)
    a = of_bits(U32(0x3F800000) | (mag & U32(0x007FFFFF)))
    y = of_bits(U32(RECIP_SEED) - to_bits(a)).copy()
    two, one = F32(2.0), F32(1.0)
    y = fmul(y, fsub(two, fmul(a, y)))
    y = fmul(y, fsub(two, fmul(a, y)))
    y = fadd(fmul(y, fsub(one, fmul(a, y))), y)
    too_big = mag >= U32(0x7E800000)
    is_zero = mag == 0
    k = np.where(too_big | is_zero, 0, 127 - (mag >> U32(23)).astype(np.int64))
    r = np.where(too_big, F32(0.0), _bump_exponent(y, k)).astype(F32)
    r = of_bits(to_bits(r) | sign)
    return np.where(is_zero, F32(0.0), r).astype(F32)


def q8(p) -> np.ndarray:
    """Round half to even, clip to [-127, 127], NaN -> 0 (fp32.py:167-172)."""
    p = flush(p)
    r = np.rint(np.where(np.isnan(p), F32(0.0), p).astype(np.float64))
    return np.clip(r, -127, 127).astype(np.int8)


def group_offset(gmax_bits, amax_bits) -> np.ndarray:
    """The largest d <= 31 with a * 2^d <= amax, from the two bit patterns (fp32.py:313-318):
    the exponent difference, less one when a's fraction exceeds amax's; 0 where a == 0."""
    a = np.asarray(gmax_bits, np.int64)
    m = np.asarray(amax_bits, np.int64)
    d = (m >> 23) - (a >> 23) - ((a & 0x7FFFFF) > (m & 0x7FFFFF)).astype(np.int64)
    return np.where(a == 0, 0, np.clip(d, 0, OFFSET_MAX)).astype(np.uint8)


def quantize_rows(x, g: int, row_mode: bool = False):
    """QACT / QST of the rows of x [R, n] in groups of g (docs/isa.md "Quantization";
    fp32.py:321-343).

    Per row: amax = the largest |x| by bit pattern, S = amax * f32(1/127),
    inv = 127 * recip(amax) (both 0 for an all-zero row); per group the offset d (0 in row mode)
    and q = q8(x * (inv * 2^d)). Returns (q int8 [R, n], S fp32 [R], d uint8 [R, n/g]).
    """
    x = flush(as_f32(x))
    R, n = x.shape
    if n % g:
        raise ValueError(f"row of {n} is not whole groups of {g}")
    mb = magnitude_bits(x)
    amax_b = mb.max(axis=1)
    amax = of_bits(amax_b)
    zero = amax_b == 0
    S = np.where(zero, F32(0.0), fmul(amax, ONE_OVER_127)).astype(F32)
    inv = np.where(zero, F32(0.0), fmul(F32(127.0), recip(amax))).astype(F32)
    if row_mode:
        d = np.zeros((R, n // g), np.uint8)
    else:
        gmax_b = mb.reshape(R, n // g, g).max(axis=2)
        d = group_offset(gmax_b, amax_b[:, None])
    pow2 = np.ldexp(F32(1.0), d.astype(np.int32)).astype(F32)
    scale = fmul(inv[:, None], pow2)                                  # [R, n/g]
    p = fmul(x.reshape(R, n // g, g), scale[:, :, None])
    return q8(p).reshape(R, n), S, d


def quantize_whole_rows(x):
    """fp32.quantize along the last axis (fp32.py:295-307): one scale per row, no offsets;
    the same bytes as quantize_rows(x, n, row_mode=True)."""
    q, S, _ = quantize_rows(x, as_f32(x).shape[1], row_mode=True)
    return q, S
