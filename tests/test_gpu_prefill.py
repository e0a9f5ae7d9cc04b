"""GPU parity of the prefill GEMM (tcgen05, bf16 activations x int8-row weights) against the
float64 oracle (oracle/prefill.py), through the C ABI.

Tolerance: every product of a bf16 and an int8 is exact in fp32, so the only error is the
fp32 accumulation and the final scale product; each output must satisfy
|y - y64| <= TOL * (|x| @ |deq|^T)[m, n]  (elementwise), TOL stated below."""
import numpy as np
import pytest

from oracle import mx as X
from oracle import prefill as PF
from opentpu_b200 import workloads as WL

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

# fp32 accumulation over K terms, measured against the sum of the terms' magnitudes
TOL = 2.0 ** -19


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA device")
    from opentpu_b200 import linear
    return linear


def _weights(ops, rng, N, K):
    W = rng.normal(0.0, 0.02, size=(N, K)).astype(np.float32)
    rows, srows = X.quantize_rows_rsc(W)
    return rows, srows, ops.PackedWeight.from_packed(rows, srows, "int8-row", K)


def _acts(rng, M, K):
    x = PF.bf16_round(rng.normal(0.0, 1.0, size=(M, K)).astype(np.float32))
    return x, torch.from_numpy(x).cuda().to(torch.bfloat16)


def _check(y, x, rows, srows, K, unit=False):
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    want, bound = PF.gemm_w8a16(x, rows, srows, K, unit)
    err = np.abs(got - want)
    ratio = float((err / np.maximum(bound, 1e-30)).max())
    assert ratio <= TOL, f"max |y - y64| / (|x| @ |deq|^T) = {ratio:.3g} > {TOL:.3g}"
    return ratio


def _status_clean(ops):
    import ctypes
    from opentpu_b200 import _lib as L
    v = ctypes.c_int(0)
    L.call("otq_status_word", ctypes.addressof(v), 0)
    return v.value == 0


@pytest.mark.parametrize("M,N,K", [(1, 8, 64), (37, 300, 200), (256, 256, 64), (300, 520, 1032),
                                   (512, 256, 2048), (777, 129, 128)])
def test_gemm_matches_float64(ops, M, N, K):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    rows, srows, w = _weights(ops, rng, N, K)
    x, xd = _acts(rng, M, K)
    _check(ops.gemm_w8a16(xd, w), x, rows, srows, K)
    assert _status_clean(ops)


def test_gemm_reference_rsc_bytes(ops, golden):
    """The reference's own int8-row bytes (quant.quantize_rows via runtime.py:66-76)."""
    rows, srows = golden["fmt_rsc_q"].view(np.uint8), golden["fmt_rsc_s"]
    K = rows.shape[1]
    w = ops.PackedWeight.from_packed(rows, srows, "int8-row", K)
    x, xd = _acts(np.random.default_rng(5), 384, K)
    _check(ops.gemm_w8a16(xd, w), x, rows, srows, K)


@pytest.mark.parametrize("K", [256, 1024])   # one K slice a tile / several (added into y)
def test_gemm_acc_and_unit(ops, K):
    rng = np.random.default_rng(11 + K)
    M, N = 300, 384
    rows, srows, w = _weights(ops, rng, N, K)
    x, xd = _acts(rng, M, K)
    old_np = rng.normal(size=(M, N)).astype(np.float32)
    acc = ops.gemm_w8a16(xd, w, out=torch.from_numpy(old_np).cuda(), acc=True)
    torch.cuda.synchronize()
    want, bound = PF.gemm_w8a16(x, rows, srows, K)
    err = np.abs(acc.cpu().numpy().astype(np.float64) - (old_np + want))
    # the product's tolerance plus the rounding of the sums with the old value
    assert np.all(err <= TOL * bound + 2.0 ** -22 * (np.abs(old_np) + np.abs(want)))
    wu = ops.PackedWeight.from_packed(rows, None, "int8", K)
    _check(ops.gemm_w8a16(xd, wu), x, rows, None, K, unit=True)


def test_unsplit_tiles_are_reproducible(ops):
    """K = 256 is four chunks: never sliced, so every tile is one unit and the result is the
    same bits on every run (and the same in a group launch)."""
    rng = np.random.default_rng(2)
    rows, srows, w = _weights(ops, rng, 1000, 256)
    x, xd = _acts(rng, 700, 256)
    y0 = ops.gemm_w8a16(xd, w)
    y1 = ops.gemm_w8a16(xd, w)
    _, _, w2 = _weights(ops, rng, 300, 256)
    y2 = ops.gemm_w8a16_group([(xd, w, None, False), (xd, w2, None, False)])[0]
    torch.cuda.synchronize()
    assert torch.equal(y0, y1) and torch.equal(y0, y2)
    _check(y0, x, rows, srows, 256)


def test_group_launch_matches_float64(ops):
    """A SmolLM3-3B layer's seven projections at 512 tokens in one
    launch, and one launch a projection: both within TOL of float64."""
    rng = np.random.default_rng(3)
    items, host_side = [], []
    for name, N, K in WL.SMOLLM3_3B.projections():
        rows, srows, w = _weights(ops, rng, N, K)
        x, xd = _acts(rng, 512, K)
        items.append((xd, w, None, False))
        host_side.append((x, rows, srows, K))
    outs = ops.gemm_w8a16_group(items)
    for (xd, w, _, _), y, (x, rows, srows, K) in zip(items, outs, host_side):
        _check(y, x, rows, srows, K)
        _check(ops.gemm_w8a16(xd, w), x, rows, srows, K)
    assert _status_clean(ops)


def test_gemm_rejects_bad_operands(ops):
    rng = np.random.default_rng(0)
    _, _, w = _weights(ops, rng, 64, 128)
    with pytest.raises(ValueError):
        ops.gemm_w8a16(torch.zeros(4, 128, device="cuda"), w)          # fp32 x
    with pytest.raises(ValueError):
        ops.gemm_w8a16(torch.zeros(4, 64, device="cuda", dtype=torch.bfloat16), w)   # K
    w4 = ops.PackedWeight.from_float(torch.randn(64, 128, device="cuda"), "int4")
    with pytest.raises(ValueError):
        ops.gemm_w8a16(torch.zeros(4, 128, device="cuda", dtype=torch.bfloat16), w4)
