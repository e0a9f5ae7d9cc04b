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
