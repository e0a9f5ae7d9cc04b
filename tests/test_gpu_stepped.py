"""Stepped tags on one GPU (otq_qmm_peer with tags = OTQ_TAGS_STEPPED, world 1; DecodeChain
gather="tagged"), the tags row-sharded steps use on several GPUs: every projection writes its
output as tagged words and the next launch reads them until the tags show this step's output,
instead of waiting for the launch before it to end. The outputs must equal, bit for bit, the
chain with plain outputs and stream-ordered launches, over several graph-replayed steps (the
step count in the tags advances once a step), and no bounded wait may run out."""
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


def _status(L):
    v = ctypes.c_int(0)
    L.call("otq_status_word", ctypes.addressof(v), 0)
    return v.value


def _bits(t):
    torch.cuda.synchronize()
    return t.float().cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("shape_name", ["TINY", "QWEN3_0_6B"])
def test_stepped_chain_equals_plain_chain(lib, shape_name):
    from opentpu_b200 import workloads as WL
    from opentpu_b200.decode import DecodeChain
    shape = getattr(WL, shape_name)
    tagged = DecodeChain(shape, seed=11, gather="tagged")
    plain = DecodeChain(shape, seed=11)   # world 1: plain outputs
    assert tagged.fused and not plain.fused
    tagged.capture()   # 3 eager steps, then the graph
    plain.capture()
    for replays in (1, 4):
        tagged.replay(replays)
        plain.replay(replays)
        torch.cuda.synchronize()
        for i in range(len(tagged.plan)):
            assert np.array_equal(_bits(tagged.full_out(i)), _bits(plain.full_out(i))), i
        assert int(tagged.token[0]) == int(plain.token[0])
    steps, done = tagged.counters.tolist()
    assert steps == 3 + 1 + 4 and done == 0   # one advance a step; the CTA count re-armed
    assert _status(lib) == 0
    tagged.release()
    plain.release()


def test_stepped_tags_validated(lib):
    from opentpu_b200 import linear
    w = linear.PackedWeight.from_float(torch.randn(64, 128, device="cuda") * 0.02, "int8-row")
    x = torch.randn(128, device="cuda")
    y = torch.zeros(64, 2, device="cuda")
    counters = torch.zeros(2, dtype=torch.int32, device="cuda")
    pr = lib.Peer()
    pr.rank, pr.world, pr.wait = 0, 1, 0
    pr.seq, pr.done = counters.data_ptr(), counters.data_ptr() + 4
    for tags, pos in ((2, 0), (lib.TAGS_STEPPED, 1023), (lib.TAGS_STEPPED, -1)):
        pr.tags, pr.step_pos = tags, pos
        with pytest.raises(ValueError):   # refused on the host: nothing is launched
            linear.qlinear_peer(x, w, y, pr)
    pr.tags, pr.step_pos, pr.step_last = lib.TAGS_STEPPED, 5, 1
    linear.qlinear_peer(x, w, y, pr)
    torch.cuda.synchronize()
    tags = y[:, 1].contiguous().view(torch.int32).cpu()
    assert (tags == 5 + 1).all()                     # step 0, position 5
    assert counters.tolist() == [1, 0]               # the step's last launch advanced the count
    ref = linear.qlinear(x.unsqueeze(0), w)
    assert np.array_equal(_bits(y[:, 0]), _bits(ref.reshape(-1)))
