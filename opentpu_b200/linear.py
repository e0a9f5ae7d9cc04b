"""The quantized linear layer as torch-level operators over libotq.

Reference surface this mirrors:
- `runtime.Weight(array, shard, fmt)` (opentpu/runtime.py:38-51) and the quantizers
  `quant.quantize_mxu` (quant.py:510-524), `runtime.quantize_rows` (runtime.py:66-76) and
  `quant.quantize(W, "int4", g=32, scale="fp16")` (quant.py:225-227) -> `PackedWeight`;
- `fp32.quantize_mx` / QACT (fp32.py:321-343) -> `quantize_act`;
- MM (isasim.py:749-910) -> `mm`; `ol.dot` of an fp32 tile (language.py:150-162, one QACT
  over the row then one MM) -> `qlinear`.

Formats: the MX formats "int8" (int8x), "int4" (int4x), "fp4" (fp4x6), "nvfp4", plus
"int8-row" (int8 per output row with an fp32 scale: MM RSC) and "int4-g32" (4-bit, group 32,
fp16 scale; weight-only: fp32 activations, not bit-exact by construction).

Every tensor lives on a CUDA device; every call runs on torch's current stream. Nothing here
computes on the CPU.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib as L

D = 128
MX_FORMATS = ("int8", "int4", "fp4", "nvfp4")
FORMATS = MX_FORMATS + ("int8-row", "int4-g32")
WINDOW = {"int8": 16, "int4": 11, "fp4": 11, "nvfp4": 13}     # opentpu/isa.py:28 MX_W


def row_bytes(K: int, fmt: str) -> int:
    """Streamed bytes of one weight row (quant.py:287-289; int4-g32: K/2)."""
    if fmt in ("int8", "int8-row"):
        return K
    if fmt == "int4-g32":
        return K // 2
    return -(-K // (2 * D)) * D


def scale_bytes(K: int, fmt: str) -> int:
    """Bytes of one scale row (quant.py:292-309; int8-row: Sw alone; int4-g32: fp16 a group)."""
    if K % D and fmt != "int4-g32":
        raise ValueError(f"inner dimension {K} is not a multiple of D={D}")
    KB = K // D
    if fmt == "int8-row":
        return 4
    if fmt == "int8":
        return 4 + 4 * -(-KB // 4)
    if fmt in ("int4", "fp4"):
        return 8 + 8 * -(-KB // 2)
    if fmt == "nvfp4":
        return 16 + 16 * -(-KB // 2)
    if fmt == "int4-g32":
        return 2 * (K // 32)
    raise ValueError(f"unknown format {fmt!r}")


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _cuda(t: torch.Tensor, what: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{what} must be a CUDA tensor")
    return t


@dataclass
class PackedWeight:
    """A weight matrix [N, K] resident in HBM in one format.

    MX formats: `rows` uint8 [N, rs] (rs a multiple of 16) and `srows` uint8 [N, srs] -- the
    reference's byte layout (or srows None: UNIT, no scales); `k0` the first scale block (a
    column part, quant.part_scales). int4-g32: `rows` the nibble codes [N, K/2] and `srows` the
    fp16 scales [N, K/32] (torch.float16)."""
    fmt: str
    N: int
    K: int
    rows: torch.Tensor
    srows: torch.Tensor | None
    k0: int = 0
    rsc: bool = False

    def __post_init__(self):
        if self.fmt == "int8-row":
            self.rsc = True
        if self.rsc and self.fmt in ("nvfp4", "int4-g32"):
            raise ValueError("RSC (row scales only) does not take nvfp4 (isa.py:527)")

    @property
    def mx_fmt(self) -> str:
        return "int8" if self.fmt == "int8-row" else self.fmt

    @property
    def flags(self) -> int:
        f = 0
        if self.srows is None:
            f |= L.MM_UNIT
        if self.rsc:
            f |= L.MM_RSC
        return f

    @property
    def stream_bytes(self) -> int:
        """HBM bytes one pass over the weight reads (elements and scales actually used)."""
        if self.srows is None:
            s = 0
        elif self.rsc:
            s = 4 * self.N
        else:
            s = self.N * scale_bytes(self.K, self.fmt)
        return self.N * row_bytes(self.K, self.fmt) + s

    @staticmethod
    def from_float(W: torch.Tensor, fmt: str, shard: int | None = None, world: int = 1,
                   rank: int = 0) -> "PackedWeight":
        """Quantize fp32 W [N, K] on the GPU into `fmt` (the reference quantizer's bytes).

        shard (runtime.Weight(array, shard, fmt), runtime.py:38-51,138-142): None keeps the
        whole matrix; 0 keeps rank `rank`'s contiguous block of N / world rows (the row shard a
        row-sharded projection runs: every output's exact sum stays on one rank); 1 keeps its
        block of K / world columns, quantized on its own as the reference quantizes a slice's
        part (per-row scales of the part). ValueError for a bad shard, a world that does not
        divide the sharded dimension, or a column block that is not whole quantization
        blocks, as for a bad format or shape."""
        if fmt not in FORMATS:
            raise ValueError(f"Weight fmt must be one of {FORMATS}")
        if shard not in (None, 0, 1):
            raise ValueError("Weight shard must be None, 0 (rows) or 1 (columns)")
        W = _cuda(W, "W")
        if W.ndim != 2:
            raise ValueError("Weight must be 2-D [N, K]")
        if world < 1 or not 0 <= rank < world:
            raise ValueError(f"rank {rank} of world {world}")
        if shard is not None and world > 1:
            n = W.shape[shard]
            if n % world:
                raise ValueError(f"{n} {'rows' if shard == 0 else 'columns'} do not split over "
                                 f"{world} ranks")
            part = n // world
            if shard == 1 and part % (32 if fmt == "int4-g32" else D):
                raise ValueError(f"a column shard of {part} is not whole blocks of "
                                 f"{32 if fmt == 'int4-g32' else D}")
            W = W[rank * part:(rank + 1) * part] if shard == 0 else \
                W[:, rank * part:(rank + 1) * part]
        W = W.to(torch.float32).contiguous()
        N, K = W.shape
        dev = W.device
        if fmt == "int8-row":
            rows = torch.empty((N, -(-K // 16) * 16), dtype=torch.uint8, device=dev)
            srows = torch.empty((N, 4), dtype=torch.uint8, device=dev)
            L.call("otq_pack_int8", W.data_ptr(), N, K, K, 1, rows.data_ptr(), rows.shape[1],
                   srows.data_ptr(), 4, _stream())
            return PackedWeight(fmt, N, K, rows, srows)
        if fmt == "int4-g32":
            codes = torch.empty((N, K // 2), dtype=torch.uint8, device=dev)
            scales = torch.empty((N, K // 32), dtype=torch.float16, device=dev)
            L.call("otq_pack_g32", W.data_ptr(), N, K, K, codes.data_ptr(), scales.data_ptr(),
                   _stream())
            return PackedWeight(fmt, N, K, codes, scales)
        rows = torch.empty((N, -(-row_bytes(K, fmt) // 16) * 16), dtype=torch.uint8, device=dev)
        srows = torch.empty((N, scale_bytes(K, fmt)), dtype=torch.uint8, device=dev)
        L.call("otq_quantize_mxu", L.FMT[fmt], W.data_ptr(), N, K, K, rows.data_ptr(),
               rows.shape[1], srows.data_ptr(), srows.shape[1], _stream())
        return PackedWeight(fmt, N, K, rows, srows)

    @staticmethod
    def from_packed(rows, srows, fmt: str, K: int, device="cuda", k0: int = 0,
                    rsc: bool = False) -> "PackedWeight":
        """Wrap packed bytes (e.g. the reference's quant.quantize_mxu output) without
        re-quantizing: copied to `device` once, padded to 16-byte row strides. rsc: the scale
        rows are Sw alone (MM RSC)."""
        if fmt not in FORMATS:
            raise ValueError(f"Weight fmt must be one of {FORMATS}")
        r = torch.as_tensor(rows).to(device)
        N = r.shape[0]
        if fmt != "int4-g32":
            r = r.to(torch.uint8)
            rs = -(-r.shape[1] // 16) * 16
            if rs != r.shape[1]:
                r = torch.nn.functional.pad(r, (0, rs - r.shape[1]))
            s = None if srows is None else torch.as_tensor(srows).to(device).to(torch.uint8)
        else:
            r = r.to(torch.uint8)
            s = torch.as_tensor(srows)
            if s.dtype != torch.float16:
                s = s.to(torch.float16)
            s = s.to(device)
        return PackedWeight(fmt, N, K, r.contiguous(), None if s is None else s.contiguous(), k0,
                            rsc)

    def row_slice(self, n0: int, n1: int) -> "PackedWeight":
        """Rows n0..n1 (a row shard: runtime.Weight(shard=0), runtime.py:138-142); a view."""
        return PackedWeight(self.fmt, n1 - n0, self.K, self.rows[n0:n1],
                            None if self.srows is None else self.srows[n0:n1], self.k0,
                            self.rsc)


def _as_rows(x: torch.Tensor, K: int) -> tuple[torch.Tensor, bool]:
    _cuda(x, "x")
    if x.dtype != torch.float32:
        raise ValueError("x must be float32")
    vec = x.ndim == 1
    x2 = x.reshape(1, -1) if vec else x
    if x2.ndim != 2 or x2.shape[1] != K:
        raise ValueError(f"x must be [M, {K}] (or [{K}])")
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    return x2, vec


def quantize_act(x: torch.Tensor, row_mode: bool = False, group: int = 32):
    """QACT of the rows of x [M, K] (fp32.quantize_mx): (q int8 [M, K], S fp32 [M],
    d uint8 [M, K/group])."""
    x2, _ = _as_rows(x, x.shape[-1])
    M, K = x2.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    S = torch.empty((M,), dtype=torch.float32, device=x.device)
    d = torch.empty((M, K // group), dtype=torch.uint8, device=x.device)
    L.call("otq_quantize_rows", x2.data_ptr(), M, K, x2.stride(0), group, int(row_mode),
           q.data_ptr(), K, S.data_ptr(), d.data_ptr(), K // group, _stream())
    return q, S, d


def _out(y, M, N, dev, need_old: bool):
    if y is None:
        if need_old:
            raise ValueError("acc / alpha need `out` holding the old values")
        return torch.empty((M, N), dtype=torch.float32, device=dev)
    _cuda(y, "out")
    if y.dtype != torch.float32 or y.shape[-1] != N or y.stride(-1) != 1:
        raise ValueError(f"out must be float32 [M, {N}] with unit column stride")
    return y.reshape(M, N) if y.ndim == 1 else y


def mm(q, S, d, w: PackedWeight, *, out=None, acc: bool = False, alpha=None):
    """MM of pre-quantized activations (quantize_act's) against w: y [M, N] fp32, bit-exact
    with the reference's MM. acc: y = out + MM; alpha: y = out * alpha + MM (ASCALE: w UNIT)."""
    if w.fmt == "int4-g32":
        raise ValueError("int4-g32 is weight-only: use qlinear on fp32 activations")
    M, K = q.shape
    if K != w.K:
        raise ValueError(f"activations have K={K}, the weight {w.K}")
    y = _out(out, M, w.N, q.device, acc or alpha is not None)
    flags = w.flags | (L.MM_ACC if acc or alpha is not None else 0) | \
        (L.MM_ASCALE if alpha is not None else 0)
    L.call("otq_mm", L.FMT[w.mx_fmt], flags, w.rows.data_ptr(), w.rows.stride(0),
           _ptr(w.srows), 0 if w.srows is None else w.srows.stride(0), w.k0, w.N, w.K,
           q.data_ptr(), q.stride(0), S.data_ptr(), d.data_ptr(), d.stride(0), M,
           _ptr(alpha), y.data_ptr(), y.stride(0), _stream())
    return y


def qlinear(x: torch.Tensor, w: PackedWeight, *, out=None, acc: bool = False, alpha=None,
            row_mode: bool = False, k_split: int = 0, pdl: bool = False):
    """y = x @ W^T through the quantized weight (ol.dot on an fp32 tile).

    MX formats: QACT of each row of x (offsets per 32, or ROW mode) fused with MM in one kernel,
    bit-exact with the reference. int4-g32: weight-only, fp32 accumulation (tolerance).
    x [M, K] or [K]; returns [M, N] (or [N]); out / acc / alpha as in `mm`. k_split (warps
    sharing a row's K range; 0 picks) and pdl tune the launch: results are identical for every
    value."""
    x2, vec = _as_rows(x, w.K)
    M = x2.shape[0]
    y = _out(out, M, w.N, x.device, acc or alpha is not None)
    if w.fmt == "int4-g32":
        if alpha is not None:
            raise ValueError("int4-g32 takes no alpha")
        L.call("otq_linear_g32", w.rows.data_ptr(), w.srows.data_ptr(), w.N, w.K, x2.data_ptr(),
               x2.stride(0), M, int(acc), y.data_ptr(), y.stride(0), _stream())
    else:
        flags = w.flags | (L.MM_ACC if acc or alpha is not None else 0) | \
            (L.MM_ASCALE if alpha is not None else 0)
        L.call("otq_qmm_ex", L.FMT[w.mx_fmt], flags, w.rows.data_ptr(), w.rows.stride(0),
               _ptr(w.srows), 0 if w.srows is None else w.srows.stride(0), w.k0, w.N, w.K,
               x2.data_ptr(), x2.stride(0), int(row_mode), M, _ptr(alpha), y.data_ptr(),
               y.stride(0), k_split, int(pdl), _stream())
    return y.reshape(-1) if vec and out is None else y


def _gemm_proj(x: torch.Tensor, w: PackedWeight, y: torch.Tensor | None, acc: bool):
    """Checked operands of one prefill GEMM projection: (GemmProj, y)."""
    if w.fmt != "int8-row" and not (w.fmt == "int8" and w.srows is None):
        raise ValueError("the prefill GEMM takes int8-row weights (or UNIT int8)")
    _cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.ndim != 2 or x.shape[1] != w.K:
        raise ValueError(f"x must be bfloat16 [M, {w.K}]")
    if x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    M = x.shape[0]
    y = _out(y, M, w.N, x.device, acc)
    p = L.GemmProj()
    p.flags = w.flags | (L.MM_ACC if acc else 0)
    p.rows, p.rs = w.rows.data_ptr(), w.rows.stride(0)
    p.srows, p.srs = _ptr(w.srows), 0 if w.srows is None else w.srows.stride(0)
    p.N, p.K, p.x, p.ldx, p.M = w.N, w.K, x.data_ptr(), x.stride(0), M
    p.y, p.ldy = y.data_ptr(), y.stride(0)
    return p, y, x


def gemm_w8a16(x: torch.Tensor, w: PackedWeight, *, out=None, acc: bool = False) -> torch.Tensor:
    """Prefill linear layer: y [M, N] fp32 = x [M, K] bf16 @ (q * Sw)^T on the tensor cores
    (tcgen05), w an int8-row weight -- the reference's `deq @ x` with bf16 activations
    (opentpu/reference.py:14-17 on quant.quantize(W, "int8", g=K), quant.py:218-224). fp32
    accumulation: within a relative tolerance of float64, not bit-exact. acc: y = out + ."""
    p, y, x = _gemm_proj(x, w, out, acc)
    L.call("otq_gemm_w8a16", p.flags, p.rows, p.rs, p.srows, p.srs, p.N, p.K, p.x, p.ldx, p.M,
           p.y, p.ldy, _stream())
    return y


def gemm_w8a16_group(items) -> list:
    """Several independent prefill projections in one launch: items is a list of (x, w, out,
    acc) as gemm_w8a16 takes them (at most 8). Returns the outputs in order."""
    import ctypes
    arr = (L.GemmProj * len(items))()
    outs, keep = [], []
    for i, (x, w, out, acc) in enumerate(items):
        arr[i], y, xx = _gemm_proj(x, w, out, acc)
        outs.append(y)
        keep.append(xx)
    L.call("otq_gemm_w8a16_group", ctypes.addressof(arr), len(items), _stream())
    return outs


class QActPlanes:
    """QACT'd activations laid out for the tensor-core MM (otq_qact_planes): a device buffer
    for up to `rows` rows of K; `fill(x)` quantizes x [M, K] (M <= rows) into it. One buffer
    serves every projection that reads the same x (a layer's q / k / v, gate / up)."""

    def __init__(self, rows: int, K: int, device=None):
        n = L.load().otq_qact_planes_bytes(int(rows), int(K))
        if n < 0:
            raise ValueError(f"planes of {rows} x {K}: {L.load().otq_status_string(n).decode()}")
        self.buf = torch.empty(n, dtype=torch.uint8, device=device or "cuda")
        self.K, self.M = int(K), 0

    def fill(self, x: torch.Tensor, row_mode: bool = False) -> "QActPlanes":
        x2, _ = _as_rows(x, self.K)
        L.call("otq_qact_planes", x2.data_ptr(), x2.stride(0), x2.shape[0], self.K,
               int(row_mode), self.buf.data_ptr(), self.buf.numel(), _stream())
        self.M = x2.shape[0]
        return self


def _tc_weight(w: PackedWeight):
    if w.fmt != "int8-row" and not (w.fmt == "int8" and w.srows is None):
        raise ValueError("the tensor-core MM takes int8-row weights (or UNIT int8)")


def qlinear_tc(x: torch.Tensor, w: PackedWeight, *, out=None, acc: bool = False,
               row_mode: bool = False, planes: QActPlanes | None = None) -> torch.Tensor:
    """y = MM(QACT(x), w) on the tcgen05 tensor cores (kind::i8, otq_qmm_tc): the same bits as
    `qlinear` for int8-row (or UNIT int8) weights, at any M (prefill, batched decode). x [M, K]
    or [K] fp32; planes: a QActPlanes of at least M rows to reuse as the scratch buffer."""
    _tc_weight(w)
    x2, vec = _as_rows(x, w.K)
    M = x2.shape[0]
    y = _out(out, M, w.N, x.device, acc)
    if planes is None:
        planes = QActPlanes(M, w.K, x.device)
    elif planes.K != w.K:
        raise ValueError(f"planes hold K = {planes.K}, the weight has K = {w.K}")
    L.call("otq_qmm_tc", w.flags | (L.MM_ACC if acc else 0), w.rows.data_ptr(), w.rows.stride(0),
           _ptr(w.srows), 0 if w.srows is None else w.srows.stride(0), w.N, w.K, x2.data_ptr(),
           x2.stride(0), int(row_mode), M, planes.buf.data_ptr(), planes.buf.numel(),
           y.data_ptr(), y.stride(0), _stream())
    planes.M = M
    return y.reshape(-1) if vec and out is None else y


def gemm_w8a8_group(items) -> list:
    """Up to 8 independent tensor-core MMs in one launch (otq_gemm_w8a8_group): items is a list
    of (planes, w, out, acc), planes a filled QActPlanes. Returns the outputs in order."""
    import ctypes
    arr = (L.Gemm8Proj * len(items))()
    outs = []
    for i, (planes, w, out, acc) in enumerate(items):
        _tc_weight(w)
        if planes.K != w.K or planes.M < 1:
            raise ValueError("planes must be filled with rows of the weight's K")
        y = _out(out, planes.M, w.N, planes.buf.device, acc)
        p = arr[i]
        p.flags = w.flags | (L.MM_ACC if acc else 0)
        p.rows, p.rs = w.rows.data_ptr(), w.rows.stride(0)
        p.srows = _ptr(w.srows)
        p.srs = 0 if w.srows is None else w.srows.stride(0)
        p.N, p.K = w.N, w.K
        p.planes, p.M = planes.buf.data_ptr(), planes.M
        p.y, p.ldy = y.data_ptr(), y.stride(0)
        outs.append(y)
    L.call("otq_gemm_w8a8_group", ctypes.addressof(arr), len(items), _stream())
    return outs


def qlinear_peer(x: torch.Tensor, w: PackedWeight, y: torch.Tensor, peer, *,
                 row_mode: bool = False, pdl: bool = False) -> torch.Tensor:
    """QACT + MM of one activation row against this rank's rows of a row-sharded projection,
    the output all-gather fused in (otq_qmm_peer). y is this rank's slice of its symmetric copy
    of the output row as tagged words: a contiguous float32 tensor [N, 2] (value, tag bits).
    x is plain fp32 [K] (peer.wait == 0) or the previous projection's tagged row [K, 2]
    (peer.wait != 0). Every rank must make the same sequence of calls."""
    if w.fmt == "int4-g32":
        raise ValueError("int4-g32 is not an MM format; it has no fused gather")
    _cuda(x, "x")
    _cuda(y, "y")
    if peer.wait:
        if x.dtype != torch.float32 or x.numel() != 2 * w.K or not x.is_contiguous():
            raise ValueError(f"a tagged x must be a contiguous float32 [{w.K}, 2] view")
        xp, ldx = x.data_ptr(), w.K
    else:
        x2, _ = _as_rows(x, w.K)
        if x2.shape[0] != 1:
            raise ValueError("the fused gather takes one activation row")
        xp, ldx = x2.data_ptr(), x2.stride(0)
    if y.dtype != torch.float32 or y.numel() != 2 * w.N or not y.is_contiguous():
        raise ValueError(f"y must be a contiguous float32 [{w.N}, 2] view")
    import ctypes
    L.call("otq_qmm_peer", L.FMT[w.mx_fmt], w.flags, w.rows.data_ptr(), w.rows.stride(0),
           _ptr(w.srows), 0 if w.srows is None else w.srows.stride(0), w.k0, w.N, w.K,
           xp, ldx, int(row_mode), y.data_ptr(), ctypes.addressof(peer), int(pdl), _stream())
    return y


def argmax(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """The index of the first maximum of the logit row x (a 1-D or [1, N] float32 view with any
    element stride): the reference's greedy sink (llm/generate.py:252-280; numpy argmax, ties to
    the lowest id), on the device. Returns an int64 tensor of 2 words whose first is the index
    (`out`, if given, is reused)."""
    _cuda(x, "x")
    if x.dtype != torch.float32:
        raise ValueError("x must be float32")
    v = x.reshape(-1) if x.dim() > 1 and x.shape[0] == 1 else x
    if v.dim() != 1:
        raise ValueError("x must be one row")
    if out is None:
        out = torch.empty(2, dtype=torch.int64, device=x.device)
    L.call("otq_argmax", v.data_ptr(), v.numel(), v.stride(0), out.data_ptr(), _stream())
    return out


def chain_table(steps) -> "ctypes.Array":
    """The otq_proj array of a chain: steps is a list of (x [K] or [1, K], w, out [N] or [1, N],
    acc, row_mode) with MX / int8-row weights. Kept by the caller to call qlinear_chain again."""
    import ctypes
    arr = (L.Proj * len(steps))()
    for i, (x, w, y, acc, row_mode) in enumerate(steps):
        if w.fmt == "int4-g32":
            raise ValueError("int4-g32 is not an MM format; it has no chain launch")
        if x.numel() != w.K or y.numel() != w.N:
            raise ValueError(f"projection {i}: x has {x.numel()} elements for K = {w.K}, "
                             f"out {y.numel()} for N = {w.N}")
        if not (x.is_contiguous() and y.is_contiguous()):
            raise ValueError(f"projection {i}: x and out must be contiguous")
        p = arr[i]
        p.fmt, p.flags = L.FMT[w.mx_fmt], w.flags | (L.MM_ACC if acc else 0)
        p.rows, p.rs = w.rows.data_ptr(), w.rows.stride(0)
        p.srows, p.srs = _ptr(w.srows), 0 if w.srows is None else w.srows.stride(0)
        p.k0, p.N, p.K = w.k0, w.N, w.K
        p.x, p.row_mode, p.y = x.data_ptr(), int(row_mode), y.data_ptr()
    return arr


def qlinear_chain(table) -> None:
    """Run a chain table (chain_table) on the current stream: the projections in order, one
    activation row each, each possibly reading an earlier one's output -- the same results as
    qlinear called per projection, in one persistent launch per run of one weight format."""
    import ctypes
    L.call("otq_qmm_chain", ctypes.addressof(table), len(table), _stream())
