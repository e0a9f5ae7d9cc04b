"""A bounded device wait that runs out, on purpose and without a fault: failure detection for the
fused NVLink gather, in the form that leaves the GPU context usable.

A launch of otq_qmm_peer with a tagged input (wait != 0) reads its input words until their tags
reach the rank's count. Here nobody ever writes those words (their tags stay 0 while the count
is 7), so every read comes back behind. With a short limit (otq_set_wait_limit) the wait gives
up, sets bit 0 of the device status word and the launch ends normally. The host then reads the
status, clears it, restores the default limit, delivers the input words with the expected tag,
and the next launch must be bit-exact with the plain QACT + MM of the same row and leave the
status clear."""
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


def _tagged(x, tag):
    """The fp32 row x as tagged words [K, 2] (value bits, tag)."""
    w = torch.empty((x.numel(), 2), dtype=torch.int32, device="cuda")
    w[:, 0] = x.view(torch.int32)
    w[:, 1] = tag
    return w.view(torch.float32)


def test_tagged_wait_runs_out_and_the_next_launch_is_exact(lib):
    from opentpu_b200 import linear
    torch.manual_seed(3)
    N, K = 256, 1024
    w = linear.PackedWeight.from_float(torch.randn(N, K, device="cuda") * 0.02, "int8-row")
    x = torch.randn(K, device="cuda")
    want = linear.qlinear(x.unsqueeze(0), w).reshape(-1)
    y = torch.zeros((N, 2), device="cuda")
    counters = torch.tensor([7, 0], dtype=torch.int32, device="cuda")   # count 7, no CTA done
    pr = lib.Peer()
    pr.rank, pr.world, pr.wait, pr.tags = 0, 1, 1, lib.TAGS_COUNTED
    pr.seq, pr.done = counters.data_ptr(), counters.data_ptr() + 4
    torch.cuda.synchronize()
    assert _status(lib, reset=True) in (0, 1)   # start from a clear word

    never = torch.zeros((K, 2), device="cuda")   # tags 0 < 7: the words never arrive
    lib.call("otq_set_wait_limit", 256)
    try:
        linear.qlinear_peer(never, w, y, pr)
        torch.cuda.synchronize()                 # the launch ends: the wait was bounded
    finally:
        lib.call("otq_set_wait_limit", 0)
    assert _status(lib) & 1, "the wait on tags that never arrive did not record its timeout"
    assert counters.tolist() == [8, 0]           # the launch still completed and counted
    assert _status(lib, reset=True) & 1
    assert _status(lib) == 0

    xt = _tagged(x, 8)                           # now the input arrives with the expected tag
    linear.qlinear_peer(xt, w, y, pr)
    torch.cuda.synchronize()
    assert _status(lib) == 0
    got = y[:, 0].contiguous()
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.cpu().numpy().view(np.uint32))
    assert (y[:, 1].contiguous().view(torch.int32) == 9).all().item()   # tag = count + 1
    assert counters.tolist() == [9, 0]
