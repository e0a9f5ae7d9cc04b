"""Generate the golden vectors of tests/golden/ by running the REFERENCE itself.

Run in a container where the reference project is importable (its path is the first argument,
or the REF_ROOT environment variable). Nothing at test time imports the reference: the tests
read the .npz files this script writes.

    python tests/golden/make_golden.py /path/to/reference

What it records (each array's producer is the reference's own code):
- fp32:  recip and mul bit patterns (opentpu/fp32.py recip, mul);
- qact:  fp32.quantize_mx of rows with wide exponent spreads and edge rows, groups of 32 and
         128, offset and ROW mode;
- fmt_*: quant.quantize_mxu rows and scale rows of every MX format, and
         runtime.quantize_rows(row=True);
- mm_*:  ISA-simulator programs LD, QACT, MM (opentpu/isasim.py) at D = 128 (and D = 32, the
         reference's own test geometry) for every format with UNIT, RSC, k0, ACC and ASCALE:
         the simulator's ACT RAM bytes, scales, offsets and the MM outputs;
- dot_*: runtime.launch of the reference's k_dot kernel (tests/test_quant.py:202-204), the
         whole QACT + quantize_mxu + MM pipeline;
- cfg1:  configuration 1 (W 1024x1024 N(0, 0.02), x N(0, 1), seed 0) through MM RSC and
         through k_dot (int8x), outputs and a digest of the packed weights;
- g32:   quant.quantize(W, "int4", g=32, scale="fp16") dequantized values and scales.
"""
from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))          # the repo (opentpu_b200.workloads)


def _ref_root() -> str:
    if len(sys.argv) > 1:
        return sys.argv[1]
    if os.environ.get("REF_ROOT"):
        return os.environ["REF_ROOT"]
    raise SystemExit("usage: make_golden.py <reference project root>")


sys.path.insert(0, _ref_root())
from opentpu import Config, fp32 as RF, isa as I, quant as RQ       # noqa: E402
from opentpu import language as ol                                     # noqa: E402
from opentpu.isasim import Machine                                     # noqa: E402
from opentpu.runtime import Input, Output, Weight, launch, quantize_rows   # noqa: E402

from opentpu_b200 import workloads as WL                              # noqa: E402


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


# ------------------------------------------------------------------------------ fp32
def gen_fp32(out):
    rng = np.random.default_rng(11)
    mant = np.concatenate([[0, 1, 0x7FFFFF, 0x400000, 0x7311C3], rng.integers(0, 1 << 23, 40)])
    xs = np.array([(e << 23) | int(m) for e in range(0, 256) for m in mant], np.uint32)
    xs = np.concatenate([xs, xs | np.uint32(0x80000000)])
    x = xs.view(np.float32)
    out["fp32_recip_in"] = xs
    out["fp32_recip_out"] = RF.bits(RF.recip(x)).astype(np.uint32)
    a = np.concatenate([rng.integers(0, 1 << 32, 4000, dtype=np.uint64).astype(np.uint32),
                        np.array([0x3F000000, 0xBF000000, 0x3F000000, 0x7F800000, 0],
                                 np.uint32)])
    b = np.concatenate([rng.integers(0, 1 << 32, 4000, dtype=np.uint64).astype(np.uint32),
                        np.array([0x00FFFFFF, 0x00FFFFFF, 0x00FFFFFE, 0, 0x7F800000],
                                 np.uint32)])
    # bias the random pairs towards products near the flush boundary and overflow
    e = rng.integers(0, 255, a.shape[0]).astype(np.uint32)
    a = np.where(rng.random(a.shape[0]) < 0.5, (a & np.uint32(0x807FFFFF)) | (e << 23), a)
    out["fp32_mul_a"], out["fp32_mul_b"] = a.astype(np.uint32), b.astype(np.uint32)
    out["fp32_mul_out"] = RF.bits(RF.mul(a.view(np.float32), b.view(np.float32))).astype(np.uint32)


# ------------------------------------------------------------------------------ QACT
def qact_inputs():
    rng = np.random.default_rng(12)
    K = 1024
    rows = [WL.spread_acts(rng, 6, K, 3.0, 32), WL.spread_acts(rng, 4, K, 8.0, 8),
            rng.standard_normal((4, K)).astype(np.float32)]
    edge = np.zeros((8, K), np.float32)
    edge[1, 5] = np.uint32(0x01000000).view(np.float32)        # amax so small inv is +inf
    edge[2] = rng.standard_normal(K).astype(np.float32)
    edge[2, 64:96] = 0                                          # a zero group
    edge[3] = rng.standard_normal(K).astype(np.float32) * 1e-38  # denormal inputs flush
    with np.errstate(over="ignore"):                            # amax >= 2^126: recip is 0,
        edge[4] = rng.standard_normal(K).astype(np.float32) * np.float32(3e38)   # some inf
    edge[5] = -0.0
    edge[6] = np.where(rng.random(K) < 0.5, 1.0, -1.0) * np.exp2(rng.integers(-40, 40, K))
    edge[7, ::3] = 0.5                                          # exact ties of q8's rounding
    edge[7, 1] = 127.0
    return np.concatenate(rows + [edge]).astype(np.float32)


def gen_qact(out):
    x = qact_inputs()
    out["qact_x"] = x
    for g in (32, 128):
        for row in (0, 1):
            q, S, d = RF.quantize_mx(x, g, bool(row))
            out[f"qact_g{g}_r{row}_q"] = q
            out[f"qact_g{g}_r{row}_S"] = RF.bits(S).astype(np.uint32)
            out[f"qact_g{g}_r{row}_d"] = d


# ------------------------------------------------------------------------------ formats
def gen_formats(out):
    rng = np.random.default_rng(13)
    W = WL.spread_rows(rng, 24, 1024, 3.0, 32)
    W[3, 100:132] = 0
    W[5, :128] = 0
    out["fmt_W"] = W
    for fmt in RQ.MXU_FORMATS:
        rows, srows = RQ.quantize_mxu(W, fmt)
        out[f"fmt_{fmt}_rows"], out[f"fmt_{fmt}_srows"] = rows, srows
    q, s = quantize_rows(W, 128, row=True)
    out["fmt_rsc_q"], out["fmt_rsc_s"] = q, s


# ------------------------------------------------------------------------------ MM programs
def scale_rows(rng, wf, N, KBr, rsc, big):
    """Random scale rows as tests/test_mx.py:_scale_rows draws them (bytes [N, srs])."""
    G = 8 if wf == I.WNV else 4
    sw = (rng.standard_normal(N) * 0.01).astype(np.float32)
    hi = 20 if big else 4
    if rsc:
        return sw[:, None].view(np.uint8).copy()
    if wf == I.W8:
        dw = rng.integers(0, hi, (N, KBr))
        rows = np.zeros((N, 4 + 4 * -(-KBr // 4)), np.uint8)
        rows[:, :4] = sw[:, None].view(np.uint8)
        rows[:, 4:4 + KBr] = dw
        return rows
    if wf in (I.W4I, I.W4F):
        dw = rng.integers(0, hi, (N, KBr))
        m = rng.integers(0, 64, (N, KBr, G))
        word = (dw | sum(m[:, :, b] << (8 + 6 * b) for b in range(G))).astype(np.uint32)
        rows = np.zeros((N, 8 + 8 * -(-KBr // 2)), np.uint8)
        rows[:, :4] = sw[:, None].view(np.uint8)
        rows[:, 8:8 + 4 * KBr] = word.view(np.uint8).reshape(N, -1)
        return rows
    e4 = rng.integers(0, 0x7F, (N, KBr, G))
    if big:
        e4[rng.random(e4.shape) < 0.3] &= 0x0F
    rows = np.zeros((N, 16 + 16 * -(-KBr // 2)), np.uint8)
    rows[:, :4] = sw[:, None].view(np.uint8)
    rows[:, 16:16 + 8 * KBr] = e4.astype(np.uint8).reshape(N, -1)
    return rows


def run_mm(D, x, data, srows, wf, M, N, KB, *, unit=False, rsc=False, k0=0, row_mode=False,
           old=None, alpha=None):
    """LD x, QACT, MM on the ISA simulator; returns (act q, Sa, da, y)."""
    K = KB * D
    rs = data.shape[1]
    x_bytes = -(-x.nbytes // D) * D
    WA = x_bytes
    SA = -(-(WA + N * rs) // 64) * 64
    dram_bytes = 1 << max(20, int(np.ceil(np.log2(SA + srows.size + 64))))
    OUT = -(-x.size // 64) * 64
    AS = OUT + M * N
    tmem = 1 << max(16, int(np.ceil(np.log2(AS + M + 64))))
    cfg = Config(S=1, D=D, MCOLS=max(4, M), ACT_BLOCKS=max(64, 1 + KB), TMEM_WORDS=tmem,
                 DRAM_BYTES=dram_bytes)
    img = np.zeros(dram_bytes, np.uint8)
    img[:x.nbytes] = x.view(np.uint8).reshape(-1)
    img[WA:WA + data.size] = data.reshape(-1)
    img[SA:SA + srows.size] = srows.reshape(-1)
    mm_kw = dict(unit=unit, wf=wf, k0=k0, rsc=rsc)
    if alpha is not None:
        mm_kw.update(acc=True, ascale=AS)
        ssa = 0
    else:
        mm_kw.update(acc=old is not None)
        ssa = SA
    prog = [I.ld(0, 0, x.size), I.qact(0, M, 1, KB, K, row=row_mode),
            I.mm(WA, ssa, OUT, N, KB, rs, N, M, 1, srows.shape[1], **mm_kw), I.halt()]
    mach = Machine(cfg, [prog], [img])
    sl = mach.slices[0]
    if old is not None:
        sl.tput(OUT + np.arange(M * N), old.reshape(-1))
    if alpha is not None:
        sl.tput(AS + np.arange(M), alpha)
    mach.run()
    y = sl.tget(OUT + np.arange(M * N)).reshape(M, N).astype(np.float32)
    return (sl.act[:M, D:(1 + KB) * D].copy(), sl.ascale[:M, 1].copy(),
            sl.adoff[:M, 1:1 + KB].copy(), y)


# test_mx.py:154-161's cases without PAIR (a timing mode of the MXU that changes no bit)
MM_CASES = [  # wf, unit, rsc, k0, big offsets
    (I.W8, False, False, 0, False), (I.W8, False, False, 3, True), (I.W8, False, True, 0, False),
    (I.W8, True, False, 0, False), (I.W4F, False, False, 1, False), (I.W4F, False, False, 2, True),
    (I.W4I, False, False, 0, False), (I.W4I, False, False, 1, True), (I.W4F, True, False, 0, False),
    (I.W4F, False, True, 0, False), (I.W4I, False, True, 0, False), (I.WNV, False, False, 1, True),
    (I.WNV, False, False, 2, False), (I.WNV, True, False, 0, False),
]


def gen_mm(out, D, tag, shapes):
    cases = []
    for ci, (wf, unit, rsc, k0, big) in enumerate(MM_CASES):
        for KB, M in shapes:
            if True:
                N = 24
                rng = np.random.default_rng(1000 * wf + 10 * KB + k0 + 3 * unit + rsc + 97 * M)
                x = (rng.standard_normal((M, KB * D))
                     * np.exp(rng.uniform(-8 if big else -2, 2, (M, KB * 4, 1)))
                     .repeat(D // 4, axis=2).reshape(M, -1)).astype(np.float32)
                if wf == I.W8:
                    data = rng.integers(-127, 128, (N, KB * D)).astype(np.int8).view(np.uint8)
                else:
                    codes = rng.integers(0, 16, (N, KB * D))
                    data = np.zeros((N, -(-KB * D // (2 * D)) * D), np.uint8)
                    data[:, :KB * D // 2] = RQ.pack4(codes)
                srows = scale_rows(rng, wf, N, k0 + KB, rsc, big)
                row_mode = bool((ci + KB) % 3 == 0)
                act, Sa, da, y = run_mm(D, x, data, srows, wf, M, N, KB, unit=unit, rsc=rsc,
                                        k0=k0, row_mode=row_mode)
                key = f"{tag}_{len(cases)}"
                out[key + "_x"], out[key + "_data"], out[key + "_srows"] = x, data, srows
                out[key + "_q"], out[key + "_Sa"] = act, RF.bits(Sa).astype(np.uint32)
                out[key + "_da"], out[key + "_y"] = da, RF.bits(y).astype(np.uint32)
                out[key + "_meta"] = np.array([wf, unit, rsc, k0, KB, M, N, row_mode], np.int64)
                cases.append(key)
    # ACC and ASCALE (tests/test_mx.py:226-254) on int8 rows
    rng = np.random.default_rng(6 + D)
    M, N, KB = 4, 24, 2
    x = rng.standard_normal((M, KB * D)).astype(np.float32)
    data = rng.integers(-127, 128, (N, KB * D)).astype(np.int8).view(np.uint8)
    srows = scale_rows(rng, I.W8, N, KB, False, False)
    old = rng.standard_normal((M, N)).astype(np.float32)
    alpha = rng.standard_normal(M).astype(np.float32)
    *_, y_acc = run_mm(D, x, data, srows, I.W8, M, N, KB, old=old)
    *_, y_asc = run_mm(D, x, data, np.zeros((N, 4), np.uint8), I.W8, M, N, KB, unit=True,
                       old=old, alpha=alpha)
    key = f"{tag}_acc"
    out[key + "_x"], out[key + "_data"], out[key + "_srows"] = x, data, srows
    out[key + "_old"], out[key + "_alpha"] = old, alpha
    out[key + "_y_acc"] = RF.bits(y_acc).astype(np.uint32)
    out[key + "_y_ascale"] = RF.bits(y_asc).astype(np.uint32)
    out[f"{tag}_cases"] = np.array(cases)


# ------------------------------------------------------------------------------ k_dot
@ol.jit
def k_dot(x, w, out):
    ol.store(out, ol.dot(ol.load(x), w))


def gen_dot(out):
    D = 128
    for fmt in RQ.MXU_FORMATS:
        rng = np.random.default_rng(D + RQ.MXU_FORMATS.index(fmt))
        M, N, K = 3, 24, 8 * D
        x = WL.spread_acts(rng, M, K, 6.0, 8)
        W = WL.spread_rows(rng, N, K, 6.0, 8)
        cfg = Config(S=1, D=D, MCOLS=4)
        y = launch(k_dot, cfg, x=Input(x), w=Weight(W, fmt=fmt), out=Output((M, N))).outputs["out"]
        out[f"dot_{fmt}_x"], out[f"dot_{fmt}_W"] = x, W
        out[f"dot_{fmt}_y"] = RF.bits(np.asarray(y, np.float32)).astype(np.uint32)


def gen_config1(out):
    W, x = WL.gemv_config1(0)
    D = 128
    q, s = quantize_rows(W, D, row=True)
    _, _, _, y = run_mm(D, x[None, :], q.view(np.uint8), s, I.W8, 1, 1024, 8, rsc=True)
    out["cfg1_rsc_y"] = RF.bits(y[0]).astype(np.uint32)
    out["cfg1_rsc_digest"] = np.array(digest(q.view(np.uint8), s))
    cfg = Config(S=1, D=D, MCOLS=4, DRAM_BYTES=1 << 22)
    y2 = launch(k_dot, cfg, x=Input(x[None, :]), w=Weight(W, fmt="int8"),
                out=Output((1, 1024))).outputs["out"]
    out["cfg1_int8x_y"] = RF.bits(np.asarray(y2, np.float32)[0]).astype(np.uint32)
    rows, srows = RQ.quantize_mxu(W, "int8")
    out["cfg1_int8x_digest"] = np.array(digest(rows, srows))
    out["cfg1_weightonly_y"] = (RQ.quantize(W, "int8", g=1024).deq.astype(np.float64)
                                @ x.astype(np.float64))


# ------------------------------------------------------------------------------ g32 fp16
def gen_g32(out):
    rng = np.random.default_rng(14)
    W = WL.spread_rows(rng, 40, 512, 1.0, 32)
    W[2, 32:64] = 0
    W[7, :] *= 1e-7                                   # fp16 subnormal scales
    W[9, :] *= 3e4                                    # scales past fp16's top clip at 65504
    qz = RQ.quantize(W, "int4", g=32, scale="fp16")
    x = rng.standard_normal((4, 512)).astype(np.float32)
    out["g32_W"], out["g32_deq"], out["g32_scales"] = W, qz.deq, qz.scales
    out["g32_x"] = x
    out["g32_y"] = x.astype(np.float64) @ qz.deq.astype(np.float64).T


def main():
    out: dict = {}
    gen_fp32(out)
    gen_qact(out)
    gen_formats(out)
    gen_mm(out, 128, "mm128", ((1, 3), (3, 1), (8, 8)))
    gen_mm(out, 32, "mm32", ((1, 3), (3, 3)))
    gen_dot(out)
    gen_config1(out)
    gen_g32(out)
    np.savez_compressed(HERE / "reference_vectors.npz", **out)
    size = (HERE / "reference_vectors.npz").stat().st_size
    print(f"wrote {len(out)} arrays, {size / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
