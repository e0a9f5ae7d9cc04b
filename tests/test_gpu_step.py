"""The decode step as one persistent launch (otq_decode_step, decode.DecodeStep) against the
launch-per-projection chain (otq_qmm per projection, decode.DecodeChain) on the same seeded
weights: every projection's output bit for bit and the same greedy token, over several graph
replays (the step count in the tags advances once a launch); the general path (a group offset
of 16) against otq_qmm; and a bounded wait that runs out when a rank never writes its words."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA device")
    from opentpu_b200 import _lib as L
    L.load()
    return L


def _status(L, reset=False):
    v = ctypes.c_int(0)
    L.call("otq_status_word", ctypes.addressof(v), int(reset))
    return v.value


def _bits(t):
    torch.cuda.synchronize()
    return t.float().contiguous().cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("shape_name", ["TINY", "QWEN3_0_6B"])
def test_step_equals_chain(lib, shape_name):
    from opentpu_b200 import workloads as WL
    from opentpu_b200.decode import DecodeChain, DecodeStep
    shape = getattr(WL, shape_name)
    _status(lib, reset=True)
    step = DecodeStep(shape, seed=13)
    chain = DecodeChain(shape, seed=13)
    step.capture()
    chain.capture()
    for replays in (1, 3):
        step.replay(replays)
        chain.replay(replays)
        torch.cuda.synchronize()
        for i in range(len(step.plan)):
            assert np.array_equal(_bits(step.full_out(i)), _bits(chain.full_out(i))), i
        assert int(step.token[0]) == int(chain.token[0])
        assert int(step.token[0]) == int(torch.argmax(chain.logits()))
    steps, done, k0, k1 = step.counters.tolist()
    assert steps == 3 + 1 + 3 and done == 0 and k0 == 0 and k1 == 0
    assert _status(lib) == 0
    step.release()
    chain.release()


def test_step_general_path_and_host_input(lib):
    """A first input whose groups include one at offset 16 (multiplier 1, no class row): the
    step takes the general path for that projection; every projection still equals otq_qmm
    (QACT + MM) applied in order. The input is then replaced from the host (run_host)."""
    from opentpu_b200 import linear
    from opentpu_b200 import workloads as WL
    from opentpu_b200.decode import DecodeStep
    shape = WL.TINY
    step = DecodeStep(shape, seed=5)
    x = torch.randn(shape.hidden, device="cuda")
    x[0] = 1000.0
    x[32:64] = x[32:64].sign() * 1000.0 * 2.0 ** -16 * 0.75    # group max = amax 2^-16.4
    step.x0.copy_(x.reshape(1, -1))
    step.capture(warmup=1)
    step.replay(1)
    torch.cuda.synchronize()
    prev = step.x0
    for i, w in enumerate(step.weights):
        want = linear.qlinear(prev.reshape(1, -1)[:, :w.K].contiguous(), w)
        assert np.array_equal(_bits(step.full_out(i)), _bits(want)), i
        prev = want.reshape(-1)
    tok = torch.zeros(1, dtype=torch.int64).pin_memory()
    host = {shape.hidden: torch.randn(1, shape.hidden).pin_memory()}
    step.run_host(host, tok)
    torch.cuda.synchronize()
    assert int(tok[0]) == int(torch.argmax(step.logits()))
    assert _status(lib) == 0


def test_step_wait_runs_out_when_a_rank_never_writes(lib):
    """World 2 on one GPU, the other rank's copy a buffer nobody writes: every wait for that
    rank's words runs out (a short limit), the status word records it, the launch ends; cleared,
    the device runs a world-1 step correctly afterwards."""
    from opentpu_b200 import _lib as L
    from opentpu_b200 import workloads as WL
    from opentpu_b200.decode import DecodeStep
    shape = WL.TINY
    one = DecodeStep(shape, seed=2)
    n = len(one.plan)
    projs = (L.StepProj * n)()
    for i, w in enumerate(one.weights):
        p = projs[i]
        p.rows, p.rs, p.srows, p.srs = w.rows.data_ptr(), w.rows.stride(0), w.srows.data_ptr(), \
            w.srows.stride(0)
        p.N, p.K, p.src, p.fmt = w.N // 2, w.K, i - 1, L.STEP_RSC   # this rank's half
    total = ctypes.c_int64(0)
    L.call("otq_step_layout", ctypes.addressof(projs), n, 2, None, ctypes.byref(total))
    mine = torch.zeros(2 * total.value, device="cuda")
    other = torch.zeros(2 * total.value, device="cuda")
    counters = torch.zeros(4, dtype=torch.int32, device="cuda")
    token = torch.zeros(2, dtype=torch.int64, device="cuda")
    st = L.Step()
    st.projs, st.count, st.rank, st.world = ctypes.addressof(projs), n, 0, 2
    st.delta[0], st.delta[1] = 0, other.data_ptr() - mine.data_ptr()
    st.x0, st.out, st.counters, st.token = one.x0.data_ptr(), mine.data_ptr(), \
        counters.data_ptr(), token.data_ptr()
    nb = ctypes.c_int64(0)
    L.call("otq_step_table_bytes", ctypes.byref(nb))
    table = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
    L.call("otq_step_prepare", ctypes.addressof(st), table.data_ptr())
    _status(lib, reset=True)
    L.call("otq_set_wait_limit", 64)
    try:
        L.call("otq_decode_step", ctypes.addressof(st), table.data_ptr(),
               torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
    finally:
        L.call("otq_set_wait_limit", 0)
    assert _status(lib) & 1
    assert counters.tolist()[:2] == [1, 0]     # the launch completed and counted its step
    assert _status(lib, reset=True) & 1 and _status(lib) == 0
    one.step_eager()
    torch.cuda.synchronize()
    assert _status(lib) == 0
    assert int(one.token[0]) == int(torch.argmax(one.logits()))


def test_step_4bit_layers_within_tolerance(lib):
    """int4-g32 layers and an int8-row head in the one-launch step: each projection's output
    against the weight-only GEMV (otq_linear_g32) applied to the step's own input row, within
    the 4-bit tolerance (fp32 sums in another order), the head bit-exact (QACT + MM of the same
    row), the greedy token the head's first maximum."""
    from opentpu_b200 import linear
    from opentpu_b200 import workloads as WL
    from opentpu_b200.decode import DecodeStep
    for shape in (WL.TINY, WL.QWEN3_0_6B):
        step = DecodeStep(shape, fmt="int4-g32", seed=21)
        step.capture(warmup=2)
        step.replay(2)
        torch.cuda.synchronize()
        prev = step.x0.reshape(1, -1)
        for i, w in enumerate(step.weights):
            x = prev[:, :w.K].contiguous()
            want = linear.qlinear(x, w)
            got = step.full_out(i)
            if w.fmt == "int4-g32":
                err = (got - want).abs().max().item()
                assert err <= 2e-6 * want.abs().max().item() + 1e-30, (i, err)
            else:
                assert np.array_equal(_bits(got), _bits(want)), i
            prev = got
        assert int(step.token[0]) == int(torch.argmax(step.logits()))
        assert _status(lib) == 0
        step.release()
