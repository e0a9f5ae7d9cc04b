"""CPU restatement of the decoder of opentpu_b200/model.py (oracle; test infrastructure only).

The float math is the reference's fp32 model (opentpu/llm/qwen3.py:701-743 reference_logits):
rmsnorm (v / sqrt(mean(v^2) + eps) * g), per-head q / k norms, rotate-half RoPE from float64
tables (qwen3.py:335-346), causal softmax attention with GQA, SwiGLU, the tied LM head -- one
token at a time with a KV cache, in numpy float32. Every projection is the oracle's restatement
of the reference's quantized linear layer in the same format: MX formats through QACT + MM
(oracle/mx.py, bit-exact with the reference's ISA simulator), int8-row through the reference's
per-row quantizer with MM RSC, int4-g32 through the survey quantizer and the reference's float32
`deq @ x` (oracle/survey.py, opentpu/reference.py:14-17). Greedy decoding takes the first maximal logit (opentpu/llm/generate.py:
252-280).
"""
from __future__ import annotations

import numpy as np

from . import mx as X
from . import survey as SV

F32 = np.float32


class Linear:
    """One projection in format fmt, quantized from float32 W [N, K] by the oracle."""

    def __init__(self, W, fmt: str):
        self.fmt = fmt
        W = np.asarray(W, F32)
        self.N, self.K = W.shape
        if fmt == "int4-g32":
            _, _, self.deq = SV.quantize_g32(W)   # float32, as the reference holds it
        elif fmt == "int8-row":
            self.rows, self.srows = X.quantize_rows_rsc(W)
        else:
            self.rows, self.srows = X.quantize_weights(W, fmt)

    def __call__(self, x):
        x = np.asarray(x, F32)
        if self.fmt == "int4-g32":
            return self.deq @ x   # the reference's `deq @ x` on float32 arrays (reference.py:14-17)
        mfmt = "int8" if self.fmt == "int8-row" else self.fmt
        return X.qlinear(x[None, :], self.rows, self.srows, mfmt, rsc=self.fmt == "int8-row")[0]


class Qwen3Oracle:
    def __init__(self, shape, weights: dict, fmt: str = "int8-row", head_fmt: str = "int8-row",
                 rope=None):
        self.shape, self.W = shape, weights
        self.rope = rope          # rope(pos) -> (cos, sin) float32 [head_dim / 2]
        self.head = Linear(weights["model.embed_tokens.weight"], head_fmt)
        self.layers = []
        for i in range(shape.layers):
            p = f"model.layers.{i}."
            self.layers.append({
                "qkv": Linear(np.concatenate([weights[p + "self_attn.q_proj.weight"],
                                              weights[p + "self_attn.k_proj.weight"],
                                              weights[p + "self_attn.v_proj.weight"]]), fmt),
                "o": Linear(weights[p + "self_attn.o_proj.weight"], fmt),
                "gateup": Linear(np.concatenate([weights[p + "mlp.gate_proj.weight"],
                                                 weights[p + "mlp.up_proj.weight"]]), fmt),
                "down": Linear(weights[p + "mlp.down_proj.weight"], fmt),
            })
        self.reset()

    def reset(self):
        self.K = [[] for _ in range(self.shape.layers)]
        self.V = [[] for _ in range(self.shape.layers)]
        self.pos = 0

    def _norm(self, v, g):
        return (v / np.sqrt(np.mean(v * v, axis=-1, keepdims=True) + F32(self.shape.eps))) * g

    def _rot(self, v, c, s):
        h = v.shape[-1] // 2
        v1, v2 = v[..., :h], v[..., h:]
        return np.concatenate([v1 * c - v2 * s, v2 * c + v1 * s], axis=-1)

    def step(self, token: int, head: bool = True):
        """One token at the next position: the logits [vocab], or None with head=False (a
        prompt token whose logits nobody reads)."""
        sh, W, pos = self.shape, self.W, self.pos
        d, G = sh.head_dim, sh.n_q // sh.n_kv
        c, s = self.rope(pos)
        x = W["model.embed_tokens.weight"][token].astype(F32)
        for i, L in enumerate(self.layers):
            p = f"model.layers.{i}."
            h = self._norm(x, W[p + "input_layernorm.weight"])
            qkv = L["qkv"](h)
            nq, nk = sh.n_q * d, sh.n_kv * d
            q = qkv[:nq].reshape(sh.n_q, d)
            k = qkv[nq:nq + nk].reshape(sh.n_kv, d)
            v = qkv[nq + nk:].reshape(sh.n_kv, d)
            if sh.qk_norm:
                q = self._norm(q, W[p + "self_attn.q_norm.weight"])
                k = self._norm(k, W[p + "self_attn.k_norm.weight"])
            q, k = self._rot(q, c, s), self._rot(k, c, s)
            self.K[i].append(k)
            self.V[i].append(v)
            K = np.stack(self.K[i])            # [T, n_kv, d]
            V = np.stack(self.V[i])
            o = np.zeros((sh.n_q, d), F32)
            for hq in range(sh.n_q):
                sc = (K[:, hq // G] @ q[hq]) / F32(np.sqrt(d))
                e = np.exp(sc - sc.max())
                o[hq] = (e / e.sum()) @ V[:, hq // G]
            x = x + L["o"](o.reshape(-1))
            h = self._norm(x, W[p + "post_attention_layernorm.weight"])
            gu = L["gateup"](h)
            g, u = gu[:sh.ffn], gu[sh.ffn:]
            x = x + L["down"]((g / (1 + np.exp(-g))) * u)
        self.pos += 1
        return self.head(self._norm(x, W["model.norm.weight"])) if head else None

    def forced(self, prompt: list, tokens: list) -> np.ndarray:
        """Teacher forced: the logits [len(tokens), vocab] that chose each of `tokens` after the
        prompt, feeding the given tokens (not its own choices)."""
        self.reset()
        logits = None
        for j, tk in enumerate(prompt):
            logits = self.step(tk, head=j == len(prompt) - 1)
        rows = []
        for j, tk in enumerate(tokens):
            rows.append(logits)
            logits = self.step(tk, head=j < len(tokens) - 1)
        return np.stack(rows)
