"""The drop-in numerics surface on the CPU: opentpu_b200.quant and opentpu_b200.reference have
the reference's function names and signatures (tests/golden/api_signatures.json, written by
running the reference: tests/golden/make_api_golden.py), and the byte-layout helpers give the
reference's arrays bit for bit (tests/golden/api_vectors.npz). The GPU-backed calls are
tests/test_gpu_api.py."""
import inspect
import json

import numpy as np
import pytest

from conftest import ROOT
from opentpu_b200 import quant as Q
from opentpu_b200 import reference as R

SIG = json.loads((ROOT / "tests" / "golden" / "api_signatures.json").read_text())


@pytest.fixture(scope="module")
def api():
    with np.load(ROOT / "tests" / "golden" / "api_vectors.npz", allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def _params(fn):
    return [(p.name, p.kind, repr(p.default)) for p in inspect.signature(fn).parameters.values()]


def _ref_params(text):
    """Parameter (name, kind, default) of a signature string written by inspect."""
    import ast
    args = ast.parse(f"def f{text.split(' -> ')[0]}: pass").body[0].args
    out = []
    pos = args.posonlyargs + args.args
    defaults = [None] * (len(pos) - len(args.defaults)) + list(args.defaults)
    for a, d in zip(pos, defaults):
        out.append((a.arg, inspect.Parameter.POSITIONAL_OR_KEYWORD,
                    repr(inspect.Parameter.empty) if d is None else repr(ast.literal_eval(d))))
    return out


@pytest.mark.parametrize("name", sorted(k for k in SIG if isinstance(SIG[k], str)))
def test_signature_is_the_references(name):
    mod, *attr = name.split(".")
    obj = {"quant": Q, "reference": R}[mod]
    for a in attr:
        obj = getattr(obj, a)
    assert _params(obj) == _ref_params(SIG[name]), name


def test_quantized_fields_are_the_references():
    assert list(Q.Quantized.__dataclass_fields__) == SIG["quant.Quantized"]


@pytest.mark.parametrize("fmt", Q.MXU_FORMATS)
def test_byte_layouts_match_reference(api, fmt):
    K = api["W"].shape[1]
    rows, srows = api[f"mxu_{fmt}_rows"], api[f"mxu_{fmt}_srows"]
    assert Q.row_bytes(K, fmt) == int(api[f"row_bytes_{fmt}"])
    assert Q.scale_bytes(K, fmt) == int(api[f"scale_bytes_{fmt}"])
    assert np.array_equal(Q.elements(rows, fmt, K), api[f"elements_{fmt}"])
    Sw, dw, m = Q.unpack_scales(srows, fmt, K // 128)
    assert np.array_equal(Sw.view(np.uint32), api[f"unpack_{fmt}_Sw"].view(np.uint32))
    assert np.array_equal(dw, api[f"unpack_{fmt}_dw"]) and np.array_equal(m, api[f"unpack_{fmt}_m"])
    assert np.array_equal(Q.unpack_scales(srows, fmt, 2, k0=1)[1], api[f"unpack_{fmt}_k1_dw"])
    assert np.array_equal(Q.group_offsets(srows, fmt, K), api[f"group_offsets_{fmt}"])


def test_pack_helpers_match_reference(api):
    assert np.array_equal(Q.pack4(api["pack4_in"]), api["pack4_out"])
    assert np.array_equal(Q.unpack4(api["pack4_out"]), api["unpack4_out"])
    Sw, dw, m, e4 = api["ps_Sw"], api["ps_dw"], api["ps_m"], api["ps_e4"]
    assert np.array_equal(Q.pack_scales("int8", Sw, dw=dw), api["ps_int8"])
    assert np.array_equal(Q.pack_scales("int4", Sw, dw=dw, m=m), api["ps_int4"])
    assert np.array_equal(Q.pack_scales("nvfp4", Sw, e4=e4), api["ps_nvfp4"])
    assert Q.scale_bytes(512, "int8", rsc=True) == int(api["scale_bytes_rsc"])
    assert np.array_equal(Q.unpack_scales(api["mxu_int8_srows"], "int8", 4, rsc=True)[1],
                          api["rsc_unpack_dw"])


def test_value_errors_where_the_reference_raises():
    with pytest.raises(ValueError):
        Q.scale_bytes(100, "int8")
    with pytest.raises(ValueError):
        Q.scale_bytes(128, "int5")
    with pytest.raises(ValueError):
        Q.pack_scales("nvfp4", np.ones(1, np.float32), e4=np.full((1, 1, 8), 0x80, np.uint8))
    with pytest.raises(ValueError):
        Q.quantize(np.zeros((4, 128), np.float32), "nonsense")
    with pytest.raises(ValueError):          # a survey format that is not on this path
        Q.quantize(np.zeros((4, 128), np.float32), "mxfp4")
    assert issubclass(Q.NotExact, ValueError)
