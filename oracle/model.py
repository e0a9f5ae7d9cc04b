"""CPU restatement of the decoder of opentpu_b200/model.py (oracle; test infrastructure only).

The float math is the reference's fp32 model, `qwen3.reference_logits` (opentpu/llm/qwen3.py:
701-743), in the same numpy float32 operations and order: rmsnorm (v / sqrt(mean(v^2) + eps) *
g), per-head q / k norms, rotate-half RoPE from float64 tables (qwen3.py:335-346), causal softmax
attention with GQA (a mask of -inf above the diagonal), SwiGLU, the tied LM head -- the whole
sequence at once (teacher forced), which is what the reference computes. With fmt=None every
projection is the float `h @ W.T` and the logits are reference_logits' (pinned by
tests/test_model_oracle.py against the reference's own output). Otherwise every projection is
the oracle's restatement of the quantized linear layer in that format, row by row:

- MX formats and int8-row: QACT of each row (per row, so a batch of rows quantizes exactly as
  the rows one at a time), then MM (oracle/mx.py, bit-exact with the reference's ISA
  simulator); the down projection's input in QACT ranges of `down_chunk` columns, one MM each,
  later ranges added in order (ACC), as the reference's MLP kernel quantizes it
  (kernels/mlp.py:8-30 _chunk, down_chunk; compiler.py:2622-2726 Builder.dot);
- int4-g32: the survey quantizer's float32 `deq`, `h @ deq.T` (reference.py:14-17).

`noise=True` multiplies the embedding rows by (1 + 2^-23 N(0, 1)) with a fixed seed: the
reference's noise floor of a golden (tools/validate.py Golden._noisy), the largest logit change
that fp32 rounding differences alone cause; a greedy step whose top two logits are closer than
that is a near tie (tests/test_validate.py:124-164).
"""
from __future__ import annotations

import math

import numpy as np

from . import fp32 as F
from . import mx as X
from . import survey as SV

F32 = np.float32


def reference_down_chunk(F_: int, fmt: str | None, D: int = 128) -> int | None:
    """The QACT range of the down projection's input the reference's MLP uses
    (kernels/mlp.py:8-30: about F/8 columns, a multiple of D (2D for 4-bit rows), at least 2D
    where F allows); None for formats without QACT (float, int4-g32)."""
    if fmt in (None, "int4-g32"):
        return None
    q = D if fmt in ("int8", "int8-row") else 2 * D
    if F_ % q:
        raise ValueError(f"F {F_} is not a multiple of {q}")
    lo = min(F_, -(-2 * D // q) * q)
    c = max(lo, (F_ // 8) // q * q)
    while F_ % c and c > lo:
        c -= q
    while F_ % c:
        c += q
    return c


class Linear:
    """One projection [N, K] in format fmt (None: float32 W itself), quantized by the oracle.
    ranges: the QACT ranges' widths of the input (None: one range)."""

    def __init__(self, W, fmt: str | None, ranges: int | None = None):
        self.fmt = fmt
        W = np.asarray(W, F32)
        self.N, self.K = W.shape
        self.ranges = ranges if ranges and ranges < self.K else None
        if fmt is None:
            self.W = W
        elif fmt == "int4-g32":
            _, _, self.deq = SV.quantize_g32(W)   # float32, as the reference holds it
        elif fmt == "int8-row":
            self.rows, self.srows = X.quantize_rows_rsc(W)
        else:
            self.rows, self.srows = X.quantize_weights(W, fmt)

    def _mm(self, x, c0: int, c1: int):
        """QACT of x's columns [c0, c1) (one range a row) then MM with those weight columns."""
        mfmt = "int8" if self.fmt == "int8-row" else self.fmt
        K = c1 - c0
        q, S, d = F.quantize_rows(x[:, c0:c1], 32)
        if self.fmt == "int8-row":
            return X.mm_plain(q, S, d, self.rows[:, c0:c1], self.srows, mfmt, K)[0]
        if mfmt == "int8":
            rows = self.rows[:, c0:c1]
        else:
            rows = np.zeros((self.N, X.row_bytes(K, mfmt)), np.uint8)
            rows[:, :K // 2] = self.rows[:, c0 // 2:c1 // 2]
        return X.mm(q, S, d, rows, self.srows, mfmt, K, k0=c0 // 128)[0]

    def __call__(self, x):
        """x [M, K] (or [K]) float32 -> [M, N] float32."""
        x = np.asarray(x, F32)
        vec = x.ndim == 1
        x = np.atleast_2d(x)
        if self.fmt is None:
            y = x @ self.W.T
        elif self.fmt == "int4-g32":
            y = x @ self.deq.T    # the reference's `deq @ x` on float32 arrays
        else:
            C = self.ranges or self.K
            y = self._mm(x, 0, C)
            for c0 in range(C, self.K, C):
                y = F.fadd(y, self._mm(x, c0, c0 + C))
        return y[0] if vec else y


class Qwen3Oracle:
    def __init__(self, shape, weights: dict, fmt: str | None = "int8-row",
                 head_fmt: str | None = "int8-row", rope=None, down_chunk="reference"):
        """down_chunk: "reference" (the reference MLP's QACT ranges for fmt), None (one range)
        or a column count."""
        self.shape, self.W = shape, weights
        self.rope = rope          # rope(pos) -> (cos, sin) float32 [head_dim / 2]
        dc = reference_down_chunk(shape.ffn, fmt) if down_chunk == "reference" else down_chunk
        self.down_chunk = dc
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
                "down": Linear(weights[p + "mlp.down_proj.weight"], fmt, dc),
            })

    def _norm(self, v, g):
        return (v / np.sqrt(np.mean(v * v, axis=-1, keepdims=True) + self.shape.eps)) * g

    def forward(self, tokens, heads=None, noise: bool = False) -> np.ndarray:
        """The causal forward of the whole sequence (teacher forced): logits [len(heads), vocab]
        at the positions `heads` (default every position)."""
        sh, W = self.shape, self.W
        tokens = list(tokens)
        T, d, G = len(tokens), sh.head_dim, sh.n_q // sh.n_kv
        x = W["model.embed_tokens.weight"][tokens].astype(F32)
        if noise:
            x = (x * (1 + 2.0 ** -23 * np.random.default_rng(1).standard_normal(x.shape))
                 ).astype(F32)
        cs = [self.rope(p) for p in range(T)]
        cos = np.stack([c for c, _ in cs])[:, None, :]
        sin = np.stack([s for _, s in cs])[:, None, :]

        def rot(v):
            h = v.shape[-1] // 2
            v1, v2 = v[..., :h], v[..., h:]
            return np.concatenate([v1 * cos - v2 * sin, v2 * cos + v1 * sin], axis=-1)

        mask = np.triu(np.full((T, T), -np.inf, F32), 1)
        nq, nk = sh.n_q * d, sh.n_kv * d
        for i, L in enumerate(self.layers):
            p = f"model.layers.{i}."
            h = self._norm(x, W[p + "input_layernorm.weight"])
            qkv = L["qkv"](h)
            q = qkv[:, :nq].reshape(T, sh.n_q, d)
            k = qkv[:, nq:nq + nk].reshape(T, sh.n_kv, d)
            v = qkv[:, nq + nk:].reshape(T, sh.n_kv, d)
            if sh.qk_norm:
                q = self._norm(q, W[p + "self_attn.q_norm.weight"])
                k = self._norm(k, W[p + "self_attn.k_norm.weight"])
            q, k = rot(q), rot(k)
            o = np.zeros((T, sh.n_q, d), F32)
            for hq in range(sh.n_q):
                s = q[:, hq] @ k[:, hq // G].T / math.sqrt(d) + mask
                s = np.exp(s - s.max(axis=1, keepdims=True))
                o[:, hq] = (s / s.sum(axis=1, keepdims=True)) @ v[:, hq // G]
            x = x + L["o"](o.reshape(T, -1))
            h = self._norm(x, W[p + "post_attention_layernorm.weight"])
            gu = L["gateup"](h)
            g, u = gu[:, :sh.ffn], gu[:, sh.ffn:]
            x = x + L["down"]((g / (1 + np.exp(-g))) * u)
        rows = x if heads is None else x[list(heads)]
        return self.head(self._norm(rows, W["model.norm.weight"]))

    def forced(self, prompt: list, tokens: list, noise: bool = False) -> np.ndarray:
        """Teacher forced: the logits [len(tokens), vocab] that chose each of `tokens` after the
        prompt (the positions from the prompt's last token on), feeding the given tokens."""
        seq = list(prompt) + list(tokens[:-1])
        heads = range(len(prompt) - 1, len(seq))
        return self.forward(seq, heads, noise)


def noise_floor(oracle: Qwen3Oracle, prompt: list, tokens: list, clean=None) -> float:
    """The largest |logit| change 1-ulp input noise causes on these steps (the reference's
    floor, tools/validate.py Golden._noisy): max |forced(noise) - forced|."""
    a = oracle.forced(prompt, tokens) if clean is None else clean
    b = oracle.forced(prompt, tokens, noise=True)
    return float(np.abs(a.astype(np.float64) - b).max())


def noise_run(oracle: Qwen3Oracle, prompt: list, tokens: list, clean) -> tuple:
    """The 1-ulp input noise run against the clean logits: (its largest |logit| change -- the
    noise floor --, its smallest per-step cosine to the clean logits)."""
    b = oracle.forced(prompt, tokens, noise=True).astype(np.float64)
    a = np.asarray(clean, np.float64)
    cos = (a * b).sum(-1) / np.linalg.norm(a, axis=-1) / np.linalg.norm(b, axis=-1)
    return float(np.abs(a - b).max()), float(cos.min())


def clear_steps(ref_logits, noise: float) -> np.ndarray:
    """Steps whose top-1 leads its runner-up by more than the noise floor (not near ties)."""
    top2 = np.sort(np.asarray(ref_logits), -1)[:, -2:]
    return top2[:, 1] - top2[:, 0] > noise
