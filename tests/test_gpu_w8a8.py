"""GPU parity of the exact W8A8 MM on the tensor cores (tcgen05 kind::i8: QACT activations x
int8-row weights, otq_qact_planes + otq_gemm_w8a8_group / otq_qmm_tc) against the CPU oracle's
MM (oracle/mx.py mm_plain, the reference's opentpu/isasim.py:749-910 for RSC / UNIT rows), bit
for bit: the integer accumulation is exact and the fp32 epilogue the reference's.

Cases: M from 1 to 777 (token tiles of 16 .. 128, ragged), K from 32 (one group, a partial
chunk) to 8192, rows whose offsets need one, two or three planes, dropped groups (d > 16),
all-zero rows and groups, QACT ROW mode, UNIT weights, ACC, several projections in one launch
(different K, shared planes), and a CUDA-graph replay."""
import numpy as np
import pytest

from oracle import fp32 as F
from oracle import mx as X

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


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


def _want(x, rows, srows, K, *, row_mode=False, unit=False, old=None):
    q, S, d = F.quantize_rows(x, 32, row_mode)
    return X.mm_plain(q, S, d, rows, srows, "int8", K, unit=unit, out=old,
                      acc=old is not None)[0]


def _same_bits(got, want, what=""):
    torch.cuda.synchronize()
    g = got.cpu().numpy().view(np.uint32)
    w = np.ascontiguousarray(want, np.float32).view(np.uint32)
    bad = np.argwhere(g != w)
    assert bad.size == 0, f"{what}: {len(bad)} of {g.size} outputs differ, first at {bad[0]}"


def _status_clean():
    from opentpu_b200 import _lib as L
    return L.status_word(reset=False) == 0


def _plane_counts(planes, M):
    """The per-row plane counts the QACT kernel wrote (bytes [8 Mp, 8 Mp + M) of the buffer)."""
    Mp = -(-M // 128) * 128
    return planes.buf[8 * Mp: 8 * Mp + M].cpu().numpy()


@pytest.mark.parametrize("M,N,K", [(1, 8, 32), (2, 200, 96), (16, 128, 128), (17, 130, 160),
                                   (37, 300, 1024), (64, 1000, 3072), (130, 256, 256),
                                   (512, 384, 2048), (777, 129, 128), (8, 2048, 8192)])
def test_tc_matches_oracle(ops, M, N, K):
    rng = np.random.default_rng(M * 1000 + K)
    rows, srows, w = _weights(ops, rng, N, K)
    x = rng.normal(0.0, 1.0, size=(M, K)).astype(np.float32)
    y = ops.qlinear_tc(torch.from_numpy(x).cuda(), w)
    _same_bits(y, _want(x, rows, srows, K), f"M={M} N={N} K={K}")
    assert _status_clean()


def test_tc_equals_gemv(ops):
    """The tensor-core MM and the CUDA-core GEMV (otq_qmm) give the same bits: both are the
    reference's exact MM."""
    rng = np.random.default_rng(5)
    M, N, K = 64, 4096, 3072
    _, _, w = _weights(ops, rng, N, K)
    x = torch.randn((M, K), device="cuda", generator=torch.Generator("cuda").manual_seed(5))
    a = ops.qlinear_tc(x, w)
    b = ops.qlinear(x, w)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))


def _wide_rows(rng, M, K):
    """Rows whose 32-element groups span many binades: offsets 0 .. 20 (three planes, and
    groups past the MM window, d > 16, which MM drops), an all-zero group and an all-zero row."""
    x = rng.normal(0.0, 1.0, size=(M, K)).astype(np.float32)
    g = K // 32
    scale = np.exp2(-rng.integers(0, 21, size=(M, g))).astype(np.float32)
    scale[:, 0] = 1.0
    x = (x.reshape(M, g, 32) * scale[..., None]).reshape(M, K)
    x[0, 32:64] = 0.0
    x[M // 2] = 0.0
    return x


@pytest.mark.parametrize("M,K", [(5, 256), (128, 1024), (200, 640)])
def test_three_planes_and_dropped_groups(ops, M, K):
    rng = np.random.default_rng(7 + M)
    N = 384
    rows, srows, w = _weights(ops, rng, N, K)
    x = _wide_rows(rng, M, K)
    planes = ops.QActPlanes(M, K)
    y = ops.qlinear_tc(torch.from_numpy(x).cuda(), w, planes=planes)
    _same_bits(y, _want(x, rows, srows, K), f"wide M={M} K={K}")
    counts = _plane_counts(planes, M)
    assert counts.max() == 3 and counts[M // 2] == 1   # the zero row needs one plane


def test_two_planes_typical_and_row_mode(ops):
    rng = np.random.default_rng(9)
    M, N, K = 96, 256, 1024
    rows, srows, w = _weights(ops, rng, N, K)
    x = rng.normal(0.0, 1.0, size=(M, K)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    planes = ops.QActPlanes(M, K)
    _same_bits(ops.qlinear_tc(xd, w, planes=planes), _want(x, rows, srows, K), "typical")
    assert set(_plane_counts(planes, M).tolist()) <= {1, 2, 3}
    y = ops.qlinear_tc(xd, w, row_mode=True, planes=planes)
    _same_bits(y, _want(x, rows, srows, K, row_mode=True), "row mode")
    assert set(_plane_counts(planes, M).tolist()) == {1}


def test_unit_and_acc(ops):
    rng = np.random.default_rng(13)
    M, N, K = 70, 300, 512
    rows, srows, w = _weights(ops, rng, N, K)
    x = rng.normal(0.0, 1.0, size=(M, K)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    wu = ops.PackedWeight.from_packed(rows, None, "int8", K)
    _same_bits(ops.qlinear_tc(xd, wu), _want(x, rows, None, K, unit=True), "UNIT")
    old = rng.normal(size=(M, N)).astype(np.float32)
    out = torch.from_numpy(old.copy()).cuda()
    ops.qlinear_tc(xd, w, out=out, acc=True)
    _same_bits(out, _want(x, rows, srows, K, old=old), "ACC")


def test_group_launch(ops):
    """A layer's worth in one launch: q / k share one planes buffer, down another K."""
    rng = np.random.default_rng(17)
    M = 300
    shapes = [(512, 1024), (256, 1024), (1024, 3072)]
    ws = [_weights(ops, rng, N, K) for N, K in shapes]
    xa = rng.normal(0.0, 1.0, size=(M, 1024)).astype(np.float32)
    xb = _wide_rows(rng, M, 3072)
    pa = ops.QActPlanes(M, 1024).fill(torch.from_numpy(xa).cuda())
    pb = ops.QActPlanes(M, 3072).fill(torch.from_numpy(xb).cuda())
    outs = ops.gemm_w8a8_group([(pa, ws[0][2], None, False), (pa, ws[1][2], None, False),
                                (pb, ws[2][2], None, False)])
    for (rows, srows, _), (N, K), y, x in zip(ws, shapes, outs, (xa, xa, xb)):
        _same_bits(y, _want(x, rows, srows, K), f"group N={N} K={K}")
    assert _status_clean()


def test_graph_replay(ops):
    rng = np.random.default_rng(19)
    M, N, K = 64, 640, 2048
    rows, srows, w = _weights(ops, rng, N, K)
    x = torch.from_numpy(rng.normal(size=(M, K)).astype(np.float32)).cuda()
    planes = ops.QActPlanes(M, K)
    y = torch.empty((M, N), device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ops.qlinear_tc(x, w, out=y, planes=planes)   # first call: kernel attributes set
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            ops.qlinear_tc(x, w, out=y, planes=planes)
    y.zero_()
    g.replay()
    _same_bits(y, _want(x.cpu().numpy(), rows, srows, K), "graph")
    x.copy_(torch.from_numpy(rng.normal(size=(M, K)).astype(np.float32)))
    g.replay()
    _same_bits(y, _want(x.cpu().numpy(), rows, srows, K), "graph, new x")
    del g


def test_rejects_bad_operands(ops):
    from opentpu_b200 import _lib as L
    rng = np.random.default_rng(23)
    _, _, w = _weights(ops, rng, 64, 64)
    with pytest.raises(ValueError):   # K not whole 32-element groups
        ops.QActPlanes(4, 48)
    x = torch.zeros((200, 64), device="cuda")
    planes = ops.QActPlanes(2, 64)   # one 128-row block: too small for 200 rows
    with pytest.raises(Exception):
        ops.qlinear_tc(x, w, planes=planes)
    with pytest.raises(ValueError):
        ops.qlinear_tc(x, ops.PackedWeight.from_float(torch.randn(64, 64, device="cuda"), "int8"))
    assert L.load().otq_qact_planes_bytes(4, 48) < 0
