"""Golden logits of the reference's own model code for the tiny Qwen3 shape (the reference's
test model geometry: hidden 256, 2 layers, 4 q / 2 kv heads of 128, F 512, vocab 1000), read by
tests/test_model_oracle.py to pin oracle/model.py at model level.

    python tests/golden/make_model_golden.py /path/to/reference

Runs, on seeded weights (opentpu_b200.workloads.decoder_weights(TINY, 1), norm gains 1 + 0.1 N)
and 24 random token ids:
- qwen3.reference_logits (opentpu/llm/qwen3.py:701-743): the fp32 model;
- reference_logits on the layers' survey-format 4-bit weights (quant.quantize(W, "int4", g=32,
  scale="fp16").deq, configuration 3's layers), the embedding / tied head in fp32;
- qwen3.emulated_logits (qwen3.py:830-901) with wformat "int8" and "int4" (the MX formats):
  the float64 decode with openTPU's quantization points (QACT inputs, MX weights, the down
  projection's QACT ranges, int8 K and V, P per attention block).
Writes model_vectors.npz.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))          # the repo (opentpu_b200.workloads)


def _ref_root() -> str:
    if len(sys.argv) > 1:
        return sys.argv[1]
    if os.environ.get("REF_ROOT"):
        return os.environ["REF_ROOT"]
    raise SystemExit("usage: make_model_golden.py <reference project root>")


def tiny_weights():
    from opentpu_b200 import workloads as WL
    W = WL.decoder_weights(WL.TINY, seed=1)
    rng = np.random.default_rng(11)
    for k in W:
        if "norm" in k:
            W[k] = (1 + 0.1 * rng.standard_normal(W[k].shape)).astype(np.float32)
    return W


def main():
    sys.path.insert(0, _ref_root())
    from opentpu import quant as Q
    from opentpu.llm.qwen3 import Spec, emulated_logits, reference_logits
    from opentpu_b200 import workloads as WL
    s = WL.TINY
    spec = Spec(s.hidden, s.layers, s.n_q, s.n_kv, s.head_dim, s.ffn, s.vocab, eps=s.eps,
                theta=s.theta, qk_smooth=False)
    W = tiny_weights()
    tokens = [int(t) for t in np.random.default_rng(12).integers(0, s.vocab, 24)]
    out = {"tokens": np.array(tokens, np.int64)}
    out["reference_logits"] = reference_logits(spec, W, tokens)
    Wg = dict(W)
    for k in W:
        if k.startswith("model.layers.") and k.endswith("_proj.weight"):
            Wg[k] = Q.quantize(W[k], "int4", g=32, scale="fp16").deq
    out["reference_logits_g32"] = reference_logits(spec, Wg, tokens)
    for f in ("int8", "int4"):
        out[f"emulated_{f}"] = emulated_logits(spec, W, tokens, wformat=f)
    np.savez_compressed(HERE / "model_vectors.npz", **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
