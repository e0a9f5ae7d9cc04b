"""The drop-in numerics surface on the GPU: opentpu_b200.quant's quantizers, decoder and
emulation and opentpu_b200.reference's layer math against the reference's own outputs
(tests/golden/api_vectors.npz, made by running the reference). Bytes, codes, scales, decoded
matrices and QACT values bit for bit; float64 sums (mx_matmul, the reference's float layers) to
float64 rounding (their GPU sums add in another order than numpy's BLAS)."""
import numpy as np
import pytest

from conftest import ROOT

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

F64_TOL = 1e-12


@pytest.fixture(scope="module")
def api():
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA device")
    with np.load(ROOT / "tests" / "golden" / "api_vectors.npz", allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape and a.dtype == b.dtype, (a.shape, b.shape, a.dtype, b.dtype)
    assert np.array_equal(a.view(np.uint8), b.view(np.uint8))


def close(a, b, tol=F64_TOL):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    assert a.shape == b.shape
    assert np.abs(a - b).max() <= tol * max(np.abs(b).max(), 1e-300)


def test_quantize_int8_and_int4_match_reference(api):
    from opentpu_b200 import quant as Q
    W = api["W"]
    for g in (128, W.shape[1]):
        q = Q.quantize(W, "int8", g=g)
        same(q.deq, api[f"q_int8_g{g}_deq"])
        same(q.codes, api[f"q_int8_g{g}_codes"])
        same(q.scales, api[f"q_int8_g{g}_scales"])
        assert q.bits == float(api[f"q_int8_g{g}_bits"]) and q.g == g and q.fmt == "int8"
    q = Q.quantize(W, "int4", g=32, scale="fp16")
    same(q.deq, api["q_int4_deq"])
    same(q.scales, api["q_int4_scales"])
    assert q.codes.size == 0 and q.bits == float(api["q_int4_bits"])


@pytest.mark.parametrize("fmt", ["int8", "int4", "fp4", "nvfp4"])
def test_mx_quantizers_decoder_and_emulation_match_reference(api, fmt):
    from opentpu_b200 import quant as Q
    W, x = api["W"], api["x"]
    K = W.shape[1]
    rows, srows = Q.quantize_mxu(W, fmt)
    same(rows, api[f"mxu_{fmt}_rows"])
    same(srows, api[f"mxu_{fmt}_srows"])
    same(Q.dequantize_mxu(rows, srows, fmt, K), api[f"deq_{fmt}"])
    q = Q.quantize(W, "mx-" + fmt)
    same(q.deq, api[f"q_mx{fmt}_deq"])
    same(q.codes, api[f"q_mx{fmt}_codes"])
    same(q.scales, api[f"q_mx{fmt}_scales"])
    fw = Q.fake_w(W, fmt)
    same(np.asarray(fw), api[f"fake_w_{fmt}"])
    same(fw.mx[0], api[f"fake_w_{fmt}_dw"])
    h = Q.fake_act(x)
    close(Q.mx_matmul(h, np.asarray(fw), fw.mx[0], fw.mx[1]), api[f"mx_matmul_{fmt}"])
    close(h @ fw.T, api[f"matmul_op_{fmt}"])            # MXW's operator: mx_matmul on the GPU
    close(fw @ h.rows(0), api[f"matvec_op_{fmt}"])


def test_fake_act_matches_reference(api):
    from opentpu_b200 import quant as Q
    x = api["x"]
    for key, kw in (("fake_act", {}), ("fake_act_row", {"row": True}),
                    ("fake_act_n128", {"n": 128}), ("fake_act_ranges", {"n": [128, 384]}),
                    ("fake_act_g128", {"g": 128})):
        a = Q.fake_act(x, **kw)
        same(np.asarray(a), api[key])
        same(a.da, api[key + "_da"])
    a = Q.fake_act(api["tie_x"])                         # exact ties: the device quantizer's bytes
    same(np.asarray(a), api["fake_act_tie"])
    same(a.da, api["fake_act_tie_da"])


def test_reference_layer_math_matches_reference(api):
    from opentpu_b200 import reference as R
    h, g = api["ref_h"], api["ref_gamma"]
    close(R.rmsnorm(h, g, 1e-6), api["ref_rmsnorm"])
    close(R.silu(h), api["ref_silu"])
    close(R.mlp(h, g, api["ref_wg"], api["ref_wu"], api["ref_wd"], 1e-6), api["ref_mlp"])
    close(R.attention(api["ref_q"], api["ref_k"], api["ref_v"], 2), api["ref_attention"])
    close(R.rope(api["ref_q"], api["ref_cos"], api["ref_sin"]), api["ref_rope"])
    o, k, v = R.attention_layer(h, g, api["ref_wq"], api["ref_wk"], api["ref_wv"], api["ref_wo"],
                                api["ref_cos"], api["ref_sin"], api["ref_k"], api["ref_v"], 4, 2,
                                4, 1e-6)
    close(o, api["ref_attn_layer_h"])
    close(k, api["ref_attn_layer_k"])
    close(v, api["ref_attn_layer_v"])


def test_reference_mlp_on_the_quantized_layer():
    """reference.mlp with packed int8-row weights runs the quantized linear layer: each
    projection bit-exact with the oracle's QACT + MM on the same fp32 input."""
    from opentpu_b200 import linear
    from opentpu_b200 import reference as R
    from oracle import mx as X
    rng = np.random.default_rng(3)
    H, F = 256, 384
    h = rng.standard_normal((1, H))
    g = rng.random(H) + 0.5
    Ws = [(rng.standard_normal(s) * 0.02).astype(np.float32) for s in ((F, H), (F, H), (H, F))]
    P = [linear.PackedWeight.from_float(torch.from_numpy(w).cuda(), "int8-row") for w in Ws]
    got = R.mlp(h, g, *P, 1e-6)

    def lin(x, w):
        rows, srows = X.quantize_rows_rsc(w)
        return X.qlinear(np.asarray(x, np.float32).reshape(1, -1), rows, srows, "int8",
                         rsc=True)[0].astype(np.float64)
    xn = h / np.sqrt(np.mean(h * h, -1, keepdims=True) + 1e-6) * g
    gg, uu = lin(xn, Ws[0]), lin(xn, Ws[1])
    a = gg / (1 + np.exp(-gg)) * uu
    want = h + lin(a, Ws[2])
    close(got, want, 1e-9)   # the float64 norm / SiLU on the GPU vs numpy: float64 rounding


@pytest.mark.parametrize("fmt", ["int8", "int8-row", "int4", "nvfp4", "int4-g32"])
def test_packed_weight_shards(fmt):
    """PackedWeight.from_float(shard=0): rank r's block of rows, the same bytes as those rows of
    the whole matrix's quantization (every format quantizes a row on its own); shard=1: the
    column block quantized on its own (runtime.Weight(shard=1)); ValueError as the reference's
    Weight raises it."""
    from opentpu_b200 import linear
    rng = np.random.default_rng(9)
    W = torch.from_numpy((rng.standard_normal((64, 1024)) * 0.02).astype(np.float32)).cuda()
    full = linear.PackedWeight.from_float(W, fmt)
    for rank in range(4):
        part = linear.PackedWeight.from_float(W, fmt, shard=0, world=4, rank=rank)
        assert part.N == 16 and part.K == 1024
        assert torch.equal(part.rows, full.rows[16 * rank:16 * (rank + 1)])
        assert torch.equal(part.srows, full.srows[16 * rank:16 * (rank + 1)])
        col = linear.PackedWeight.from_float(W, fmt, shard=1, world=4, rank=rank)
        alone = linear.PackedWeight.from_float(W[:, 256 * rank:256 * (rank + 1)].contiguous(), fmt)
        assert col.N == 64 and col.K == 256
        assert torch.equal(col.rows, alone.rows) and torch.equal(col.srows, alone.srows)
    bad_cols = {"shard": 1, "world": 64 if fmt == "int4-g32" else 16}   # part not whole blocks
    for bad in ({"shard": 2}, {"shard": 0, "world": 3}, {"shard": 1, "world": 3}, bad_cols,
                {"shard": 0, "world": 2, "rank": 2}):
        with pytest.raises(ValueError):
            linear.PackedWeight.from_float(W, fmt, **bad)
