"""Golden vectors and signatures of the reference's numerics call surface (opentpu.quant,
opentpu.reference), produced by running the REFERENCE itself; read by tests/test_api_surface.py
(signatures, byte layouts, on the CPU) and tests/test_gpu_api.py (the GPU-backed calls).

    python tests/golden/make_api_golden.py /path/to/reference

Writes api_signatures.json (inspect.signature of every function this library mirrors) and
api_vectors.npz (seeded inputs and the reference's outputs of quantize, quantize_mxu,
dequantize_mxu, the byte-layout helpers, fake_w, fake_act, mx_matmul and reference.rmsnorm /
silu / mlp / attention / rope / attention_layer).
"""
from __future__ import annotations

import inspect
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

QUANT_FUNCS = ["quantize", "row_bytes", "scale_bytes", "pack4", "unpack4", "pack_scales",
               "unpack_scales", "elements", "group_offsets", "dequantize_mxu", "quantize_mx",
               "quantize_mxu", "fake_w", "fake_act", "mx_matmul"]
REFERENCE_FUNCS = ["rmsnorm", "silu", "mlp", "attention", "rope", "attention_layer"]


def _ref_root() -> str:
    if len(sys.argv) > 1:
        return sys.argv[1]
    if os.environ.get("REF_ROOT"):
        return os.environ["REF_ROOT"]
    raise SystemExit("usage: make_api_golden.py <reference project root>")


def main():
    sys.path.insert(0, _ref_root())
    from opentpu import quant as Q
    from opentpu import reference as R
    sig = {f"quant.{n}": str(inspect.signature(getattr(Q, n))) for n in QUANT_FUNCS}
    sig.update({f"reference.{n}": str(inspect.signature(getattr(R, n))) for n in REFERENCE_FUNCS})
    sig["quant.MXAct.of"] = str(inspect.signature(Q.MXAct.of))
    sig["quant.MXW.of"] = str(inspect.signature(Q.MXW.of))
    sig["quant.Quantized"] = [f.name for f in Q.Quantized.__dataclass_fields__.values()]
    (HERE / "api_signatures.json").write_text(json.dumps(sig, indent=1, sort_keys=True) + "\n")

    rng = np.random.default_rng(7)
    out = {}
    N, K, M = 48, 512, 5
    W = (rng.standard_normal((N, K)) * np.exp(rng.standard_normal((N, K // 32, 1)))
         .repeat(32, 2).reshape(N, K) * 0.02).astype(np.float32)
    x = (rng.standard_normal((M, K)) * np.exp(1.5 * rng.standard_normal((M, K // 8, 1)))
         .repeat(8, 2).reshape(M, K)).astype(np.float32)
    x[0, 5] = x[0, 9] * 0       # a zero
    out["W"], out["x"] = W, x
    for g in (128, K):
        q = Q.quantize(W, "int8", g=g)
        out[f"q_int8_g{g}_deq"], out[f"q_int8_g{g}_codes"] = q.deq, q.codes
        out[f"q_int8_g{g}_scales"], out[f"q_int8_g{g}_bits"] = q.scales, np.float64(q.bits)
    q = Q.quantize(W, "int4", g=32, scale="fp16")
    out["q_int4_deq"], out["q_int4_scales"], out["q_int4_bits"] = q.deq, q.scales, np.float64(q.bits)
    for f in Q.MXU_FORMATS:
        q = Q.quantize(W, "mx-" + f)
        out[f"q_mx{f}_deq"], out[f"q_mx{f}_codes"] = q.deq, q.codes
        out[f"q_mx{f}_scales"], out[f"q_mx{f}_bits"] = q.scales, np.float64(q.bits)
        rows, srows = Q.quantize_mxu(W, f)
        out[f"mxu_{f}_rows"], out[f"mxu_{f}_srows"] = rows, srows
        out[f"deq_{f}"] = Q.dequantize_mxu(rows, srows, f, K)
        out[f"elements_{f}"] = Q.elements(rows, f, K)
        Sw, dw, m = Q.unpack_scales(srows, f, K // 128)
        out[f"unpack_{f}_Sw"], out[f"unpack_{f}_dw"], out[f"unpack_{f}_m"] = Sw, dw, m
        out[f"unpack_{f}_k1_dw"] = Q.unpack_scales(srows, f, 2, k0=1)[1]
        out[f"group_offsets_{f}"] = Q.group_offsets(srows, f, K)
        fw = Q.fake_w(W, f)
        out[f"fake_w_{f}"], out[f"fake_w_{f}_dw"] = np.asarray(fw), fw.mx[0]
        h = Q.fake_act(x)
        out[f"mx_matmul_{f}"] = Q.mx_matmul(h, np.asarray(fw), fw.mx[0], fw.mx[1])
        out[f"matmul_op_{f}"] = np.asarray(h @ fw.T)
        out[f"matvec_op_{f}"] = np.asarray(fw @ h.rows(0))
        out[f"row_bytes_{f}"] = np.int64(Q.row_bytes(K, f))
        out[f"scale_bytes_{f}"] = np.int64(Q.scale_bytes(K, f))
    out["rsc_unpack_dw"] = Q.unpack_scales(out["mxu_int8_srows"], "int8", 4, rsc=True)[1]
    out["scale_bytes_rsc"] = np.int64(Q.scale_bytes(K, "int8", rsc=True))
    codes = rng.integers(0, 16, (7, 64)).astype(np.uint8)
    out["pack4_in"], out["pack4_out"] = codes, Q.pack4(codes)
    out["unpack4_out"] = Q.unpack4(out["pack4_out"])
    Sw = rng.random(6).astype(np.float32)
    dw = rng.integers(0, 20, (6, 3)).astype(np.uint8)
    mm = rng.integers(1, 64, (6, 3, 4)).astype(np.uint8)
    e4 = rng.integers(0, 127, (6, 3, 8)).astype(np.uint8)
    out["ps_Sw"], out["ps_dw"], out["ps_m"], out["ps_e4"] = Sw, dw, mm, e4
    out["ps_int8"] = Q.pack_scales("int8", Sw, dw=dw)
    out["ps_int4"] = Q.pack_scales("int4", Sw, dw=dw, m=mm)
    out["ps_nvfp4"] = Q.pack_scales("nvfp4", Sw, e4=e4)
    a = Q.fake_act(x)
    out["fake_act"], out["fake_act_da"] = np.asarray(a), a.da
    a = Q.fake_act(x, row=True)
    out["fake_act_row"], out["fake_act_row_da"] = np.asarray(a), a.da
    a = Q.fake_act(x, n=128)
    out["fake_act_n128"], out["fake_act_n128_da"] = np.asarray(a), a.da
    a = Q.fake_act(x, n=[128, 384])
    out["fake_act_ranges"], out["fake_act_ranges_da"] = np.asarray(a), a.da
    a = Q.fake_act(x, g=128)
    out["fake_act_g128"], out["fake_act_g128_da"] = np.asarray(a), a.da
    # exact rounding ties (values with exact ratios): the fp32 quantizer's rounding
    t = np.zeros((2, 256), np.float32)
    t[0, :4] = [127.0, 0.5, 1.5, -2.5]
    t[1, :3] = [63.5, 31.75, 3.0]
    a = Q.fake_act(t)
    out["tie_x"], out["fake_act_tie"], out["fake_act_tie_da"] = t, np.asarray(a), a.da

    # reference.py (float64 math)
    H, F, d, nq, nkv, T = 64, 96, 16, 4, 2, 6
    h = rng.standard_normal((1, H))
    gam = rng.random(H) + 0.5
    wg, wu, wd = (rng.standard_normal(s) * 0.1 for s in ((F, H), (F, H), (H, F)))
    out["ref_h"], out["ref_gamma"] = h, gam
    out["ref_wg"], out["ref_wu"], out["ref_wd"] = wg, wu, wd
    out["ref_rmsnorm"] = R.rmsnorm(h, gam, 1e-6)
    out["ref_silu"] = R.silu(h)
    out["ref_mlp"] = R.mlp(h, gam, wg, wu, wd, 1e-6)
    q = rng.standard_normal((nq, d))
    kc, vc = rng.standard_normal((nkv, T, d)), rng.standard_normal((nkv, T, d))
    out["ref_q"], out["ref_k"], out["ref_v"] = q, kc, vc
    out["ref_attention"] = R.attention(q, kc, vc, nkv)
    cos, sin = rng.standard_normal(d // 2), rng.standard_normal(d // 2)
    out["ref_cos"], out["ref_sin"] = cos, sin
    out["ref_rope"] = R.rope(q, cos, sin)
    wq, wk, wv = (rng.standard_normal(s) * 0.1 for s in ((nq * d, H), (nkv * d, H), (nkv * d, H)))
    wo = rng.standard_normal((H, nq * d)) * 0.1
    out["ref_wq"], out["ref_wk"], out["ref_wv"], out["ref_wo"] = wq, wk, wv, wo
    o, k, v = R.attention_layer(h, gam, wq, wk, wv, wo, cos, sin, kc, vc, nq, nkv, 4, 1e-6)
    out["ref_attn_layer_h"], out["ref_attn_layer_k"], out["ref_attn_layer_v"] = o, k, v
    np.savez_compressed(HERE / "api_vectors.npz", **out)
    print(f"wrote {len(out)} arrays, {len(sig)} signatures")


if __name__ == "__main__":
    main()
