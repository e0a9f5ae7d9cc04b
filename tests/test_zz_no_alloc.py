"""otq_argmax_noalloc: the greedy-token argmax for callers that cannot allocate device memory
(a plugin that is handed its inputs and outputs by a host framework that owns every buffer, or
a loop in which a cudaMalloc is not allowed). It keeps the reduction's scratch in the library's
own device array and writes only the index; here it must give the same index as otq_argmax,
which takes that scratch from the caller, on two calls in a row (the second call's row has a
smaller maximum than the first's, so scratch left over from the first call would show).

Collected last on purpose (the file name), so that a run stopping at its first failure has run
every other test before this one; it also passes alone in a fresh process."""
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


def _argmax_with_scratch(L, x):
    out = torch.zeros(2, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    L.call("otq_argmax", x.data_ptr(), x.numel(), 1, out.data_ptr(), stream)
    torch.cuda.synchronize()
    return int(out[0])


def _argmax_no_alloc(L, x, index):
    stream = torch.cuda.current_stream().cuda_stream
    L.call("otq_argmax_noalloc", x.data_ptr(), x.numel(), 1, index.data_ptr(), stream)
    torch.cuda.synchronize()
    return int(index[0])


def test_no_alloc_argmax_matches_the_entry_point_with_scratch(lib):
    rng = np.random.default_rng(17)
    first = rng.standard_normal(151936).astype(np.float32)
    first[123456] = 50.0                       # a large maximum late in the row
    second = rng.standard_normal(151936).astype(np.float32)
    second[77] = second[4000] = 9.0            # a smaller maximum, tied: the lower index wins
    index = torch.full((1,), -1, dtype=torch.int64, device="cuda")
    for row in (first, second):
        x = torch.from_numpy(row).cuda()
        want = _argmax_with_scratch(lib, x)
        got = _argmax_no_alloc(lib, x, index)
        assert got == want == int(np.argmax(row))


def test_no_alloc_argmax_strided_rows_nan_and_signed_zeros(lib):
    """A tagged row read with stride 2 (the values of (value, tag) words), a row whose maximum
    is -0 tied with +0 (the lower index wins: numpy compares them equal) and a row with a NaN
    (numpy's argmax stops at the first NaN), each against otq_argmax and numpy."""
    rng = np.random.default_rng(5)
    tagged = np.zeros((4096, 2), np.float32)
    tagged[:, 0] = rng.standard_normal(4096)
    tagged[:, 1] = 1e30                        # tags larger than every value: must be skipped
    tagged[3001, 0] = 12.0
    zeros = -np.abs(rng.standard_normal(1000)).astype(np.float32) - 1.0
    zeros[10], zeros[20] = -0.0, 0.0
    nan = rng.standard_normal(1000).astype(np.float32)
    nan[500], nan[700] = np.nan, 99.0
    index = torch.full((1,), -1, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for row, stride, want in ((tagged, 2, int(np.argmax(tagged[:, 0]))), (zeros, 1, 10),
                              (nan, 1, int(np.argmax(nan)))):
        x = torch.from_numpy(np.ascontiguousarray(row)).cuda().reshape(-1)
        n = x.numel() // stride
        out = torch.zeros(2, dtype=torch.int64, device="cuda")
        lib.call("otq_argmax", x.data_ptr(), n, stride, out.data_ptr(), stream)
        lib.call("otq_argmax_noalloc", x.data_ptr(), n, stride, index.data_ptr(), stream)
        torch.cuda.synchronize()
        assert int(index[0]) == int(out[0]) == want


def test_no_alloc_argmax_rejects_rows_past_its_limit(lib):
    x = torch.zeros(16, device="cuda")
    index = torch.zeros(1, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError):   # refused on the host: nothing is launched
        lib.call("otq_argmax_noalloc", x.data_ptr(), 1 << 32, 1, index.data_ptr(),
                 torch.cuda.current_stream().cuda_stream)
