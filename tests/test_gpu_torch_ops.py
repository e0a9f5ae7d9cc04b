"""torch.ops.otq.* on the GPU: the registered operators against the reference's golden vectors
(QACT bytes, configuration 1's MM outputs, k_dot), inside a captured CUDA graph too, and the
prefill / int4-g32 operators against the oracle within the tolerances of their own tests."""
import numpy as np
import pytest

from conftest import bits
from opentpu_b200 import workloads as WL

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def otq():
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA device")
    from opentpu_b200 import ops
    ops.load()
    return torch.ops.otq


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("g", [32, 128])
@pytest.mark.parametrize("row", [0, 1])
def test_quantize_act_matches_reference(otq, golden, g, row):
    q, S, d = otq.quantize_act(dev(golden["qact_x"]), bool(row), g)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), golden[f"qact_g{g}_r{row}_q"])
    assert np.array_equal(bits(S.cpu().numpy()), golden[f"qact_g{g}_r{row}_S"])
    if not row:
        assert np.array_equal(d.cpu().numpy(), golden[f"qact_g{g}_r{row}_d"])


def test_qlinear_mm_and_argmax_in_a_captured_graph(otq, golden):
    """Configuration 1 (W 1024x1024 int8 per row, x N(0,1)) through qlinear, through
    quantize_act + mm, and its greedy index through argmax, captured as one CUDA graph and
    replayed: the outputs are the reference's MM outputs bit for bit."""
    from opentpu_b200 import _lib as L
    from opentpu_b200 import linear
    W, x = WL.gemv_config1(0)
    w = linear.PackedWeight.from_float(dev(W), "int8-row")
    xd = dev(x)
    fmt, flags = L.FMT[w.mx_fmt], w.flags
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):   # first calls outside capture (shared-memory limits, allocator)
        otq.qlinear(xd, w.rows, w.srows, fmt, flags, w.K)
        q, S, d = otq.quantize_act(xd)
        otq.mm(q, S, d, w.rows, w.srows, fmt, flags, w.K)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        y1 = otq.qlinear(xd, w.rows, w.srows, fmt, flags, w.K)
        q, S, d = otq.quantize_act(xd)
        y2 = otq.mm(q, S, d, w.rows, w.srows, fmt, flags, w.K)
        idx = otq.argmax(y1)
    g.replay()
    torch.cuda.synchronize()
    want = golden["cfg1_rsc_y"]
    assert np.array_equal(bits(y1.cpu().numpy()), want)
    assert np.array_equal(bits(y2.cpu().numpy().reshape(-1)), want)
    assert int(idx[0]) == int(np.argmax(want.view(np.float32)))


@pytest.mark.parametrize("fmt", ["int8", "int4", "fp4", "nvfp4"])
def test_qlinear_matches_reference_k_dot(otq, golden, fmt):
    from opentpu_b200 import _lib as L
    from opentpu_b200 import linear
    w = linear.PackedWeight.from_float(dev(golden[f"dot_{fmt}_W"]), fmt)
    y = otq.qlinear(dev(golden[f"dot_{fmt}_x"]), w.rows, w.srows, L.FMT[fmt], w.flags, w.K)
    torch.cuda.synchronize()
    # the golden output is stored as its fp32 bit patterns
    assert np.array_equal(bits(y.cpu().numpy()).reshape(-1), np.asarray(golden[f"dot_{fmt}_y"]).reshape(-1))


def test_gemm_and_g32_operators_within_tolerance(otq):
    from opentpu_b200 import linear
    from oracle import prefill as PF
    from oracle import survey as SV
    rng = np.random.default_rng(4)
    N, K, M = 384, 1024, 200
    rows = rng.integers(-127, 128, (N, K), dtype=np.int8).view(np.uint8)
    sw = (rng.random(N) * 1e-3 + 1e-4).astype(np.float32)
    srows = sw.view(np.uint8).reshape(N, 4)
    x = PF.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    y = otq.gemm_w8a16(dev(x).to(torch.bfloat16), dev(rows), dev(srows), 0x80)
    want, bound = PF.gemm_w8a16(x, rows, srows, K)
    assert (np.abs(y.cpu().numpy() - want) <= 2.0 ** -19 * bound + 1e-30).all()
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    wq = linear.PackedWeight.from_float(dev(W), "int4-g32")
    xs = rng.standard_normal((3, K)).astype(np.float32)
    yg = otq.linear_g32(dev(xs), wq.rows, wq.srows).cpu().numpy()
    codes, scales, _ = SV.quantize_g32(W)
    ref = SV.linear_g32(xs, codes, scales)
    assert np.abs(yg - ref).max() <= 2e-6 * np.abs(ref).max()


def test_value_error_from_the_library(otq):
    x = torch.zeros(100, device="cuda")          # K not a multiple of 32 for QACT groups
    with pytest.raises(ValueError):
        otq.quantize_act(x)
