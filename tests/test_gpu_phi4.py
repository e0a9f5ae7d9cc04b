"""BASELINE configuration 5 on the GPU: the Phi-4-mini-shaped quantized linears (hidden 3072, MLP
8192, vocab 200064) at batches of 1, 8 and 64 activation rows, in int8 per-row (QACT + MM,
bit-exact against the oracle) and 4-bit group-32 fp16 (weight-only, against float64 `deq @ x`
within the 4-bit tolerance), the 200064 x 3072 LM head included, the int8 ones also through the
exact tensor-core MM (qlinear_tc, the same bits), and their row shards over
2 / 4 / 8 ranks (runtime.Weight(shard=0)): the ranks' outputs, gathered in rank order, are the
unsharded output bit for bit."""
import numpy as np
import pytest

from conftest import bits
from opentpu_b200 import workloads as WL

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

G32_TOL = 2e-6
SHAPES = [(n, N, K) for n, N, K in WL.PHI4_MINI.projections() if n in ("q_proj", "k_proj",
                                                                      "up_proj", "down_proj")]


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA device")
    from opentpu_b200 import linear
    return linear


def _oracle_rsc(x, rows, srows, K, chunk=16384):
    from oracle import fp32 as F
    from oracle import mx as X
    q, S, d = F.quantize_rows(x, 32)
    parts = [X.mm_plain(q, S, d, rows[i:i + chunk], srows[i:i + chunk], "int8", K)[0]
             for i in range(0, rows.shape[0], chunk)]
    return np.concatenate(parts, axis=1)


@pytest.mark.parametrize("M", [1, 8, 64])
@pytest.mark.parametrize("name,N,K", SHAPES)
def test_phi4_layer_int8_row(ops, name, N, K, M):
    rng = np.random.default_rng(N + K + M)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = ops.PackedWeight.from_float(torch.from_numpy(W).cuda(), "int8-row")
    y = ops.qlinear(torch.from_numpy(x).cuda(), w).cpu().numpy()
    rows = w.rows.cpu().numpy()[:, :K]
    srows = w.srows.cpu().numpy()
    assert np.array_equal(bits(y), bits(_oracle_rsc(x, rows, srows, K)))
    # the exact tensor-core path (QACT planes + tcgen05 kind::i8): the same bits
    ytc = ops.qlinear_tc(torch.from_numpy(x).cuda(), w).cpu().numpy()
    assert np.array_equal(bits(ytc), bits(y))
    for G in (2, 4, 8):   # row shards, gathered in rank order
        n = N // G
        parts = [ops.qlinear(torch.from_numpy(x).cuda(), w.row_slice(r * n, (r + 1) * n))
                 for r in range(G)]
        assert np.array_equal(bits(torch.cat(parts, dim=1).cpu().numpy()), bits(y))


@pytest.mark.parametrize("M", [1, 8, 64])
@pytest.mark.parametrize("name,N,K", SHAPES)
def test_phi4_layer_int4_g32(ops, name, N, K, M):
    from oracle import survey as SV
    rng = np.random.default_rng(N * 3 + K + M)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = ops.PackedWeight.from_float(torch.from_numpy(W).cuda(), "int4-g32")
    y = ops.qlinear(torch.from_numpy(x).cuda(), w).cpu().numpy()
    codes, scales, _ = SV.quantize_g32(W)
    ref = SV.linear_g32(x, codes, scales)
    assert np.abs(y - ref).max() <= G32_TOL * np.abs(ref).max()


@pytest.mark.slow
@pytest.mark.parametrize("M", [1, 8, 64])
def test_phi4_head_int8_row(ops, M):
    """The 200064 x 3072 LM head (614.6 MB of int8 rows), bit-exact at every batch, and its
    8-way row shards."""
    shape = WL.PHI4_MINI
    gen = torch.Generator(device="cuda").manual_seed(5)
    W = torch.randn((shape.vocab, shape.hidden), device="cuda", generator=gen) * 0.02
    w = ops.PackedWeight.from_float(W, "int8-row")
    del W
    rng = np.random.default_rng(M)
    x = rng.standard_normal((M, shape.hidden)).astype(np.float32)
    y = ops.qlinear(torch.from_numpy(x).cuda(), w).cpu().numpy()
    rows = w.rows.cpu().numpy()[:, :shape.hidden]
    srows = w.srows.cpu().numpy()
    assert np.array_equal(bits(y), bits(_oracle_rsc(x, rows, srows, shape.hidden)))
    ytc = ops.qlinear_tc(torch.from_numpy(x).cuda(), w).cpu().numpy()
    assert np.array_equal(bits(ytc), bits(y))
    n = shape.vocab // 8
    parts = [ops.qlinear(torch.from_numpy(x).cuda(), w.row_slice(r * n, (r + 1) * n))
             for r in range(8)]
    assert np.array_equal(bits(torch.cat(parts, dim=1).cpu().numpy()), bits(y))
