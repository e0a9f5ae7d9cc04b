"""The model oracle (oracle/model.py) pinned to the reference's own model code, on the CPU.

tests/golden/model_vectors.npz holds the reference's logits for the tiny Qwen3 shape
(tests/golden/make_model_golden.py runs qwen3.reference_logits and qwen3.emulated_logits):
- float form (every projection the fp32 `h @ W.T`): the oracle's logits are reference_logits'
  bit for bit (the same numpy float32 operations in the same order);
- int4-g32 layers (configuration 3's weight-only format): reference_logits on the survey
  quantizer's dequantized layer weights, bit for bit;
- MX int8 / int4 (QACT + exact MM, the down projection's input in the reference MLP's QACT
  ranges): emulated_logits is the reference's float64 decode with the same quantization points
  plus int8 K / V / P attention (which this oracle keeps in fp32); the oracle agrees to a
  cosine of 0.9995 at every position and sits closer to it than the fp32 model does."""
import sys

import numpy as np
import pytest

from conftest import ROOT
from oracle.model import Qwen3Oracle, clear_steps, noise_floor, reference_down_chunk
from opentpu_b200 import workloads as WL

sys.path.insert(0, str(ROOT / "tests" / "golden"))
from make_model_golden import tiny_weights  # noqa: E402


@pytest.fixture(scope="module")
def model():
    with np.load(ROOT / "tests" / "golden" / "model_vectors.npz", allow_pickle=False) as z:
        g = {k: z[k] for k in z.files}
    return g, tiny_weights(), [int(t) for t in g["tokens"]]


def _oracle(W, fmt, head_fmt, **kw):
    s = WL.TINY
    return Qwen3Oracle(s, W, fmt=fmt, head_fmt=head_fmt, rope=lambda p: WL.rope_tables(s, p), **kw)


def _cos(a, b):
    return float(min((x * y).sum() / np.linalg.norm(x) / np.linalg.norm(y) for x, y in zip(a, b)))


def test_float_oracle_is_reference_logits(model):
    g, W, toks = model
    got = _oracle(W, None, None).forward(toks)
    assert np.array_equal(got.view(np.uint32), g["reference_logits"].astype(np.float32).view(np.uint32))


def test_g32_oracle_is_reference_logits_on_the_g32_weights(model):
    g, W, toks = model
    got = _oracle(W, "int4-g32", None).forward(toks)
    assert np.array_equal(got.view(np.uint32),
                          g["reference_logits_g32"].astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("fmt", ["int8", "int4"])
def test_mx_oracle_follows_emulated_logits(model, fmt):
    g, W, toks = model
    emu = g[f"emulated_{fmt}"]
    got = _oracle(W, fmt, fmt).forward(toks).astype(np.float64)
    f32 = g["reference_logits"].astype(np.float64)
    assert _cos(got, emu) >= 0.9995
    assert np.abs(got - emu).max() < np.abs(f32 - emu).max()


def test_forced_and_noise_floor(model):
    """Teacher forcing picks the rows that chose each token; the noise floor is positive and
    tiny in the float model (1-ulp input noise), and clear_steps keeps steps above it."""
    g, W, toks = model
    o = _oracle(W, None, None)
    full = o.forward(toks[:23])
    forced = o.forced(toks[:10], toks[10:])
    assert np.array_equal(forced, full[9:23])
    fl = noise_floor(o, toks[:10], toks[10:], forced)
    assert 0 < fl < 1e-4
    assert clear_steps(forced, fl).sum() >= 12


def test_reference_down_chunks():
    # kernels/mlp.py _chunk: about F/8, whole D (2D for 4-bit), at least 2D
    assert reference_down_chunk(3072, "int8-row") == 384
    assert reference_down_chunk(3072, "int4") == 256
    assert reference_down_chunk(512, "int8") == 256
    assert reference_down_chunk(8192, "int8") == 1024
    assert reference_down_chunk(11008, "int8") == 256
    assert reference_down_chunk(3072, "int4-g32") is None
