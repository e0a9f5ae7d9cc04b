"""`opentpu.reference`'s float64 layer math (reference opentpu/reference.py:5-55) on the GPU, with
the linear layers through this library.

Same names, signatures and numpy float64 results as the reference's `rmsnorm`, `silu`, `mlp`,
`attention`, `rope` and `attention_layer`: `from opentpu_b200 import reference as R` stands in
for `from opentpu import reference as R`. The arithmetic runs in float64 on the current CUDA
device. A weight argument may be

- a float matrix [N, K] (numpy): `x @ w.T` in float64 on the GPU, the reference's math (sums in
  another order than numpy's BLAS: equal to float64 rounding);
- a `linear.PackedWeight` (a quantized weight resident on the GPU): the quantized linear layer
  itself, QACT + MM bit-exact with the reference's MM for the MX formats and int8-row, the
  fp32 weight-only GEMV for int4-g32, its fp32 output widened to float64. This is how a model
  runs its MLP on the quantized layer (`mlp` with packed gate / up / down weights).
- an `quant.MXW` (the float64 emulation of a quantized weight): `quant.mx_matmul`.

There is no CPU path: without a CUDA device every function raises.
"""
from __future__ import annotations

import numpy as np


def _torch():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("opentpu_b200.reference runs on the GPU and no CUDA device is visible")
    return torch


def _t(a):
    torch = _torch()
    if isinstance(a, torch.Tensor):
        return a.to(device="cuda", dtype=torch.float64)
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float64))).cuda()


def _np(t):
    return t.cpu().numpy()


def _linear(x, w):
    """x [..., K] (float64 tensor) times w^T for a float matrix, a PackedWeight or an MXW."""
    torch = _torch()
    from . import linear
    from . import quant as Q
    if isinstance(w, linear.PackedWeight):
        x2 = x.reshape(-1, w.K).to(torch.float32).contiguous()
        return linear.qlinear(x2, w).to(torch.float64).reshape(*x.shape[:-1], w.N)
    if isinstance(w, Q.MXW):
        return _t(np.asarray(_np(x)) @ w.T)
    return x @ _t(w).T


def _rmsnorm(x, gamma, eps):
    return x / (x * x).mean(-1, keepdim=True).add(eps).sqrt() * gamma


def rmsnorm(x, gamma, eps):
    return _np(_rmsnorm(_t(x), _t(gamma), eps))


def _silu(x):
    return x / (1.0 + (-x).exp())


def silu(x):
    return _np(_silu(_t(x)))


def mlp(h, gamma, w_gate, w_up, w_down, eps):
    """h + (silu(xn @ w_gate.T) * (xn @ w_up.T)) @ w_down.T, xn = rmsnorm(h): the SwiGLU MLP
    block with its residual, the three projections through `_linear` (the quantized layer for
    packed weights)."""
    xh = _t(h)
    xn = _rmsnorm(xh, _t(gamma), eps)
    a = _silu(_linear(xn, w_gate)) * _linear(xn, w_up)
    return _np(xh + _linear(a, w_down))


def _attention(q, k, v, n_kv_heads):
    torch = _torch()
    Hq, d = q.shape
    G = Hq // n_kv_heads
    kk = k.repeat_interleave(G, dim=0)                       # [Hq, T, d]
    vv = v.repeat_interleave(G, dim=0)
    s = torch.einsum("htd,hd->ht", kk, q)
    s = s / torch.full_like(s, float(np.sqrt(d)))   # a true division, as numpy's
    p = (s - s.amax(-1, keepdim=True)).exp()
    return torch.einsum("ht,htd->hd", p / p.sum(-1, keepdim=True), vv)


def attention(q, k, v, n_kv_heads):
    """q [Hq, d]; k, v [Hkv, T, d] -> [Hq, d] (softmax attention, GQA)."""
    return _np(_attention(_t(q), _t(k), _t(v), n_kv_heads))


def _rope(x, cos, sin):
    torch = _torch()
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def rope(x, cos, sin):
    return _np(_rope(_t(x), _t(cos), _t(sin)))


def attention_layer(h, gamma, wq, wk, wv, wo, cos, sin, k_cache, v_cache, n_q_heads,
                    n_kv_heads, pos, eps):
    """One decode step. k_cache/v_cache [Hkv, >=pos, d] hold positions < pos. Returns (h + the
    attention output's projection [1, H], k [Hkv, d], v [Hkv, d])."""
    torch = _torch()
    d = np.asarray(k_cache).shape[-1] if not isinstance(k_cache, torch.Tensor) else \
        k_cache.shape[-1]
    hh = _t(h)
    xn = _rmsnorm(hh, _t(gamma), eps)[0]
    q = _linear(xn, wq).reshape(n_q_heads, d)
    k = _linear(xn, wk).reshape(n_kv_heads, d)
    v = _linear(xn, wv).reshape(n_kv_heads, d)
    c, s = _t(cos), _t(sin)
    q, k = _rope(q, c, s), _rope(k, c, s)
    K = torch.cat([_t(k_cache)[:, :pos], k[:, None]], dim=1)
    V = torch.cat([_t(v_cache)[:, :pos], v[:, None]], dim=1)
    o = _attention(q, K, V, n_kv_heads)
    return _np(hh + _linear(o.reshape(-1), wo)[None, :]), _np(k), _np(v)
