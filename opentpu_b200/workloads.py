"""Seeded synthetic inputs and model shapes of the benchmark configurations.

The reference publishes no dataset for this path; its configurations are random-init models
and N(0, 1) activations. Every generator here uses `numpy.random.default_rng(seed)` so the
tests, the golden-vector script and the benchmark draw identical arrays on any machine.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def gemv_config1(seed: int = 0):
    """Configuration 1: W [1024, 1024] ~ N(0, 0.02) fp32, x [1024] ~ N(0, 1) fp32."""
    rng = np.random.default_rng(seed)
    W = rng.normal(0.0, 0.02, (1024, 1024)).astype(np.float32)
    x = rng.standard_normal(1024).astype(np.float32)
    return W, x


def spread_rows(rng, N: int, K: int, s: float = 3.0, g: int = 32) -> np.ndarray:
    """Rows whose groups of g have log-normal scales (offsets reach the window and past it)."""
    return (rng.standard_normal((N, K)) * np.exp(s * rng.standard_normal((N, K // g, 1)))
            .repeat(g, 2).reshape(N, K) * 0.02).astype(np.float32)


def spread_acts(rng, M: int, K: int, s: float = 2.0, g: int = 8) -> np.ndarray:
    return (rng.standard_normal((M, K)) * np.exp(s * rng.standard_normal((M, K // g, 1)))
            .repeat(g, 2).reshape(M, K)).astype(np.float32)


@dataclass(frozen=True)
class DecoderShape:
    """A decoder's projection shapes (the reference's qwen3.Spec fields, qwen3.py:65-77)."""
    name: str
    hidden: int
    layers: int
    n_q: int
    n_kv: int
    head_dim: int
    ffn: int
    vocab: int
    eps: float = 1e-6
    theta: float = 1e6
    qk_norm: bool = True

    def projections(self):
        """(name, N, K) of one layer's quantized linears, in the order a decode step runs them."""
        H, d = self.hidden, self.head_dim
        return [("q_proj", self.n_q * d, H), ("k_proj", self.n_kv * d, H),
                ("v_proj", self.n_kv * d, H), ("o_proj", H, self.n_q * d),
                ("gate_proj", self.ffn, H), ("up_proj", self.ffn, H), ("down_proj", H, self.ffn)]


QWEN3_0_6B = DecoderShape("Qwen3-0.6B", hidden=1024, layers=28, n_q=16, n_kv=8, head_dim=128,
                          ffn=3072, vocab=151936)
SMOLLM3_3B = DecoderShape("SmolLM3-3B", hidden=2048, layers=36, n_q=16, n_kv=4, head_dim=128,
                          ffn=11008, vocab=128256, qk_norm=False)
PHI4_MINI = DecoderShape("Phi-4-mini", hidden=3072, layers=32, n_q=24, n_kv=8, head_dim=128,
                         ffn=8192, vocab=200064, qk_norm=False)
# the reference's tiny test model (tests/test_qwen3.py:22-35): hidden 256, 2 layers, vocab 1000
TINY = DecoderShape("tiny-qwen3", hidden=256, layers=2, n_q=4, n_kv=2, head_dim=128, ffn=512,
                    vocab=1000)


def decoder_weights(shape: DecoderShape, seed: int = 0) -> dict:
    """Random-init float32 weights of a Qwen3-shaped decoder (the configurations' N(0, 0.02)
    projections and embedding, norm gains 1 as a fresh HF model has them), named as the
    reference's checkpoints are (qwen3.reference_logits): model.embed_tokens.weight (tied to the
    LM head, as Qwen3-0.6B is), model.layers.{i}.self_attn.{q,k,v,o}_proj.weight,
    ...q_norm / k_norm, mlp.{gate,up,down}_proj.weight, input / post_attention layernorms,
    model.norm.weight."""
    rng = np.random.default_rng(seed)
    H, d = shape.hidden, shape.head_dim

    def w(N, K):
        return rng.normal(0.0, 0.02, (N, K)).astype(np.float32)

    W = {"model.embed_tokens.weight": w(shape.vocab, H),
         "model.norm.weight": np.ones(H, np.float32)}
    for i in range(shape.layers):
        p = f"model.layers.{i}."
        W[p + "input_layernorm.weight"] = np.ones(H, np.float32)
        W[p + "post_attention_layernorm.weight"] = np.ones(H, np.float32)
        W[p + "self_attn.q_proj.weight"] = w(shape.n_q * d, H)
        W[p + "self_attn.k_proj.weight"] = w(shape.n_kv * d, H)
        W[p + "self_attn.v_proj.weight"] = w(shape.n_kv * d, H)
        W[p + "self_attn.o_proj.weight"] = w(H, shape.n_q * d)
        if shape.qk_norm:
            W[p + "self_attn.q_norm.weight"] = np.ones(d, np.float32)
            W[p + "self_attn.k_norm.weight"] = np.ones(d, np.float32)
        W[p + "mlp.gate_proj.weight"] = w(shape.ffn, H)
        W[p + "mlp.up_proj.weight"] = w(shape.ffn, H)
        W[p + "mlp.down_proj.weight"] = w(H, shape.ffn)
    return W


def rope_tables(shape: DecoderShape, pos: int):
    """cos, sin [head_dim / 2] float32 of one position, rotate-half convention, computed in
    float64 (reference opentpu/llm/qwen3.py:335-346 rope_tables, without LongRoPE factors)."""
    half = shape.head_dim // 2
    inv = 1.0 / (shape.theta ** (np.arange(half, dtype=np.float64) * 2 / shape.head_dim))
    ang = pos * inv
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def prompt_ids(shape: DecoderShape, n: int, seed: int = 0) -> list:
    """A random prompt: n token ids uniform in [0, vocab) (the configurations' random prompt)."""
    return [int(t) for t in np.random.default_rng(seed).integers(0, shape.vocab, n)]
