"""The greedy token on the device (otq_argmax) against numpy's argmax, the reference's greedy
sink (llm/generate.py:252-280: the first index of the maximum)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA device")
    from opentpu_b200 import linear
    return linear


@pytest.mark.parametrize("n", [1, 7, 1000, 151936, 200064])
def test_argmax_is_the_first_maximum(ops, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    if n > 10:
        x[n // 3] = x[n // 2] = x.max() + 1.0    # a tie: the lower index wins
        x[:5] = -np.inf
    got = ops.argmax(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert int(got[0]) == int(np.argmax(x))
    assert int(got[1]) == 0


def test_argmax_edge_rows(ops):
    for x in (np.zeros(4096, np.float32), np.full(33, -np.inf, np.float32),
              np.array([-0.0, 0.0, -1.0], np.float32), np.array([-5.0, -3.0, -3.0], np.float32),
              np.array([1.0, np.nan, 3.0, -np.nan, np.inf], np.float32)):
        got = ops.argmax(torch.from_numpy(x).cuda())
        torch.cuda.synchronize()
        assert int(got[0]) == int(np.argmax(x)), x


def test_argmax_strided_tagged_row(ops):
    rng = np.random.default_rng(1)
    words = torch.from_numpy(rng.standard_normal((5000, 2)).astype(np.float32)).cuda()
    got = ops.argmax(words[:, 0])
    torch.cuda.synchronize()
    assert int(got[0]) == int(np.argmax(words[:, 0].cpu().numpy()))


def test_decode_chain_token_is_argmax_of_logits(ops):
    from opentpu_b200 import workloads as WL
    from opentpu_b200.decode import DecodeChain
    ch = DecodeChain(WL.TINY, seed=5)
    ch.capture()
    ch.replay(3)
    torch.cuda.synchronize()
    assert int(ch.token[0]) == int(np.argmax(ch.logits().cpu().numpy().reshape(-1)))
    ch.release()
