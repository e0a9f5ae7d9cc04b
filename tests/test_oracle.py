"""The CPU oracle against vectors produced by running the reference itself
(tests/golden/make_golden.py): bit for bit on every integer, byte and fp32 result."""
import hashlib

import numpy as np
import pytest

from conftest import bits
from oracle import fp32 as F
from oracle import mx as X
from oracle import survey as SV
from opentpu_b200 import workloads as WL

FMT_OF_WF = {0: "int8", 1: "int4", 2: "fp4", 3: "nvfp4"}


def test_recip_bits(golden):
    x = golden["fp32_recip_in"].view(np.float32)
    assert np.array_equal(bits(F.recip(x)), golden["fp32_recip_out"])


def test_mul_bits(golden):
    a, b = golden["fp32_mul_a"].view(np.float32), golden["fp32_mul_b"].view(np.float32)
    assert np.array_equal(bits(F.fmul(a, b)), golden["fp32_mul_out"])


def test_mul_subnormal_grid_rule():
    # tests/test_fp.py:214: a product rounding up to 2^-126 is kept, one below it flushes
    half = np.float32(0.5)
    assert bits(F.fmul(half, np.uint32(0x00FFFFFF).view(np.float32))) == 0x00800000
    assert bits(F.fmul(-half, np.uint32(0x00FFFFFF).view(np.float32))) == 0x80800000
    assert bits(F.fmul(half, np.uint32(0x00FFFFFE).view(np.float32))) == 0


@pytest.mark.parametrize("g", [32, 128])
@pytest.mark.parametrize("row", [0, 1])
def test_qact_bytes(golden, g, row):
    q, S, d = F.quantize_rows(golden["qact_x"], g, bool(row))
    assert np.array_equal(q, golden[f"qact_g{g}_r{row}_q"])
    assert np.array_equal(bits(S), golden[f"qact_g{g}_r{row}_S"])
    assert np.array_equal(d, golden[f"qact_g{g}_r{row}_d"])


@pytest.mark.parametrize("fmt", X.FORMATS)
def test_weight_quantizers(golden, fmt):
    rows, srows = X.quantize_weights(golden["fmt_W"], fmt)
    assert np.array_equal(rows, golden[f"fmt_{fmt}_rows"])
    assert np.array_equal(srows, golden[f"fmt_{fmt}_srows"])


def test_rsc_rows(golden):
    q, s = X.quantize_rows_rsc(golden["fmt_W"])
    assert np.array_equal(q.view(np.int8), golden["fmt_rsc_q"])
    assert np.array_equal(s, golden["fmt_rsc_s"])


def _mm_cases(golden, tag):
    return [str(k) for k in golden[f"{tag}_cases"]]


@pytest.mark.parametrize("tag,D", [("mm128", 128), ("mm32", 32)])
def test_mm_programs(golden, tag, D):
    """The reference ISA simulator's QACT + MM for every format / UNIT / RSC / k0 case."""
    for key in _mm_cases(golden, tag):
        wf, unit, rsc, k0, KB, M, N, row_mode = (int(v) for v in golden[key + "_meta"])
        fmt = FMT_OF_WF[wf]
        K = KB * D
        q, S, d = F.quantize_rows(golden[key + "_x"], D // 4, bool(row_mode))
        assert np.array_equal(q, golden[key + "_q"]), key
        assert np.array_equal(bits(S), golden[key + "_Sa"]), key
        assert np.array_equal(d.reshape(M, KB, 4), golden[key + "_da"]), key
        y, acc = X.mm(q, S, d, golden[key + "_data"], golden[key + "_srows"], fmt, K, D=D, k0=k0,
                      unit=bool(unit), rsc=bool(rsc))
        assert np.abs(acc).max() < 2 ** 47
        assert np.array_equal(bits(y), golden[key + "_y"]), key


@pytest.mark.parametrize("tag,D", [("mm128", 128), ("mm32", 32)])
def test_mm_acc_and_ascale(golden, tag, D):
    k = f"{tag}_acc"
    x, data, srows = golden[k + "_x"], golden[k + "_data"], golden[k + "_srows"]
    old, alpha = golden[k + "_old"], golden[k + "_alpha"]
    q, S, d = F.quantize_rows(x, D // 4)
    y, _ = X.mm(q, S, d, data, srows, "int8", x.shape[1], D=D, out=old, acc=True)
    assert np.array_equal(bits(y), golden[k + "_y_acc"])
    y, _ = X.mm(q, S, d, data, None, "int8", x.shape[1], D=D, unit=True, out=old, alpha=alpha)
    assert np.array_equal(bits(y), golden[k + "_y_ascale"])


@pytest.mark.parametrize("fmt", X.FORMATS)
def test_whole_pipeline_k_dot(golden, fmt):
    """runtime.launch(k_dot) (QACT + quantize_mxu + MM) of the reference, bit for bit."""
    x, W = golden[f"dot_{fmt}_x"], golden[f"dot_{fmt}_W"]
    rows, srows = X.quantize_weights(W, fmt)
    y = X.qlinear(x, rows, srows, fmt)
    assert np.array_equal(bits(y), golden[f"dot_{fmt}_y"])


def test_config1(golden):
    W, x = WL.gemv_config1(0)
    q, s = X.quantize_rows_rsc(W)
    h = hashlib.sha256(q.tobytes() + s.tobytes()).hexdigest()
    assert h == str(golden["cfg1_rsc_digest"])
    y = X.qlinear(x, q, s, "int8", rsc=True)
    assert np.array_equal(bits(y[0]), golden["cfg1_rsc_y"])
    rows, srows = X.quantize_weights(W, "int8")
    assert hashlib.sha256(rows.tobytes() + srows.tobytes()).hexdigest() == \
        str(golden["cfg1_int8x_digest"])
    assert np.array_equal(bits(X.qlinear(x, rows, srows, "int8")[0]), golden["cfg1_int8x_y"])


def test_g32_fp16_quantizer(golden):
    codes, scales, deq = SV.quantize_g32(golden["g32_W"])
    assert np.array_equal(deq, golden["g32_deq"])
    assert np.array_equal(scales.astype(np.float64), golden["g32_scales"])
    assert np.array_equal(SV.unpack_g32(SV.pack_g32(codes), codes.shape[1]), codes)
    y = SV.linear_g32(golden["g32_x"], codes, scales)
    assert np.abs(y - golden["g32_y"]).max() <= 1e-12 * np.abs(golden["g32_y"]).max()


def test_emulation_matches_exact_mm(golden):
    """fake_act + dequantize + mx_matmul (the reference's float64 emulation) agree with the
    exact MM to fp32 rounding, as tests/test_quant.py:216-240 asserts for the simulator."""
    for fmt in X.FORMATS:
        x, W = golden[f"dot_{fmt}_x"], golden[f"dot_{fmt}_W"]
        rows, srows = X.quantize_weights(W, fmt)
        h, da = X.fake_act(x)
        want = X.mx_matmul(h, da, X.dequantize(rows, srows, fmt, W.shape[1]),
                           X.weight_offsets(srows, fmt, W.shape[1]), X.WINDOW[fmt])
        got = golden[f"dot_{fmt}_y"].view(np.float32)
        assert np.abs(got - want).max() < 1e-6 * np.abs(want).max(), fmt


def test_prefill_oracle_bf16_and_deq(golden):
    """oracle/prefill: bf16 rounding (ties to even) as torch rounds, and q * Sw as the MX
    dequantizer gives it for RSC rows."""
    import torch
    from oracle import prefill as PF
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.normal(size=4096).astype(np.float32),
                        np.array([1.00390625, 1.01171875, -3.0078125, 0.0, -0.0], np.float32)])
    want = torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()
    assert np.array_equal(bits(PF.bf16_round(x)), bits(want))
    rows, srows = golden["fmt_rsc_q"].view(np.uint8), golden["fmt_rsc_s"]
    K = rows.shape[1]
    d = PF.deq_rows(rows, srows, K)
    assert np.array_equal(d, X.dequantize(rows, srows, "int8", K, rsc=True))
    y, bound = PF.gemm_w8a16(want[:K][None], rows, srows, K)
    assert y.shape == (1, rows.shape[0]) and np.all(bound >= np.abs(y))
