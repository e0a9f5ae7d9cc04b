"""torch.ops.otq.* without a GPU: the extension loads (it links the same libotq.so the ctypes
binding loads), registers the six operators with their schemas, and has no CPU kernel (a CPU
tensor raises instead of computing anything on the host)."""
import pytest

torch = pytest.importorskip("torch")

SCHEMAS = {
    "quantize_act": "otq::quantize_act(Tensor x, bool row_mode=False, int group=32) -> "
                    "(Tensor, Tensor, Tensor)",
    "mm": "otq::mm(Tensor q, Tensor S, Tensor d, Tensor rows, Tensor? srows, int fmt, int flags, "
          "int K, int k0=0) -> Tensor",
    "qlinear": "otq::qlinear(Tensor x, Tensor rows, Tensor? srows, int fmt, int flags, int K, "
               "int k0=0, bool row_mode=False) -> Tensor",
    "gemm_w8a16": "otq::gemm_w8a16(Tensor x, Tensor rows, Tensor? srows, int flags) -> Tensor",
    "linear_g32": "otq::linear_g32(Tensor x, Tensor codes, Tensor scales) -> Tensor",
    "argmax": "otq::argmax(Tensor x) -> Tensor",
}


def test_ops_registered_with_their_schemas():
    from opentpu_b200 import ops  # noqa: F401
    for name, schema in SCHEMAS.items():
        assert str(getattr(torch.ops.otq, name).default._schema) == schema


def test_no_cpu_kernel():
    from opentpu_b200 import ops  # noqa: F401
    x = torch.zeros(4, 128)
    with pytest.raises(NotImplementedError):
        torch.ops.otq.quantize_act(x)
    with pytest.raises(NotImplementedError):
        torch.ops.otq.argmax(x[0])
