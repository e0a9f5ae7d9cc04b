"""A Qwen3-shaped decoder whose projections are this library's quantized linear layer.

The float math around the projections follows the reference's fp32 model
(opentpu/llm/qwen3.py:701-743 reference_logits), one token at a time with a KV cache:

    x = embed[token]
    per layer: h = rmsnorm(x); q, k, v = h @ Wqkv^T (one QACT + MM: q, k and v share the input
               and its QACT range); per-head rmsnorm of q and k; RoPE (rotate-half, tables from
               float64); causal softmax attention over the cache (GQA); x += o @ Wo^T;
               h = rmsnorm(x); g, u = h @ Wgateup^T (one QACT + MM); x += (silu(g) * u) @ Wdown^T
    logits = rmsnorm(x) @ Whead^T (Whead = embed, tied as in Qwen3-0.6B)

Every projection runs through linear.qlinear (QACT + MM bit-exact with the reference's MM for
the MX formats; weight-only fp32 accumulation for int4-g32); the norms, RoPE, attention and
SwiGLU are fp32 torch on the GPU. Greedy decoding takes the first maximal logit (the
reference's greedy sink, opentpu/llm/generate.py:252-280).
"""
from __future__ import annotations

import numpy as np
import torch

from . import linear
from . import workloads as WL


class Qwen3Decoder:
    def __init__(self, shape: WL.DecoderShape, weights: dict, fmt: str = "int8-row",
                 head_fmt: str = "int8-row", max_pos: int = 1024, device: str = "cuda"):
        self.shape, self.fmt, self.head_fmt, self.max_pos = shape, fmt, head_fmt, max_pos
        dev = torch.device(device)
        H, d = shape.hidden, shape.head_dim
        self.d = d

        def t(a):
            return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

        def q(a, f):
            return linear.PackedWeight.from_float(t(a), f)

        self.embed = t(weights["model.embed_tokens.weight"])
        self.norm = t(weights["model.norm.weight"])
        self.head = q(weights["model.embed_tokens.weight"], head_fmt)
        self.layers = []
        for i in range(shape.layers):
            p = f"model.layers.{i}."
            L = {
                "in": t(weights[p + "input_layernorm.weight"]),
                "post": t(weights[p + "post_attention_layernorm.weight"]),
                "qkv": q(np.concatenate([weights[p + "self_attn.q_proj.weight"],
                                         weights[p + "self_attn.k_proj.weight"],
                                         weights[p + "self_attn.v_proj.weight"]]), fmt),
                "o": q(weights[p + "self_attn.o_proj.weight"], fmt),
                "gateup": q(np.concatenate([weights[p + "mlp.gate_proj.weight"],
                                            weights[p + "mlp.up_proj.weight"]]), fmt),
                "down": q(weights[p + "mlp.down_proj.weight"], fmt),
            }
            if shape.qk_norm:
                L["qn"] = t(weights[p + "self_attn.q_norm.weight"])
                L["kn"] = t(weights[p + "self_attn.k_norm.weight"])
            self.layers.append(L)
        cs = [WL.rope_tables(shape, p) for p in range(max_pos)]
        self.cos = t(np.stack([c for c, _ in cs]))
        self.sin = t(np.stack([s for _, s in cs]))
        self.K = torch.zeros((shape.layers, max_pos, shape.n_kv, d), device=dev)
        self.V = torch.zeros_like(self.K)
        self.pos = 0

    def _norm(self, v, g):
        return (v / torch.sqrt(torch.mean(v * v, dim=-1, keepdim=True) + self.shape.eps)) * g

    def _rot(self, v, pos):
        h = self.d // 2
        c, s = self.cos[pos], self.sin[pos]
        v1, v2 = v[..., :h], v[..., h:]
        return torch.cat([v1 * c - v2 * s, v2 * c + v1 * s], dim=-1)

    def reset(self):
        self.pos = 0

    def step(self, token: int) -> torch.Tensor:
        """One decode step at the next position: the logits [vocab] (fp32)."""
        sh, d, pos = self.shape, self.d, self.pos
        if pos >= self.max_pos:
            raise ValueError(f"position {pos} past the cache ({self.max_pos})")
        G = sh.n_q // sh.n_kv
        x = self.embed[token].clone()
        for i, L in enumerate(self.layers):
            h = self._norm(x, L["in"])
            qkv = linear.qlinear(h, L["qkv"])
            nq, nk = sh.n_q * d, sh.n_kv * d
            q = qkv[:nq].view(sh.n_q, d)
            k = qkv[nq:nq + nk].view(sh.n_kv, d)
            v = qkv[nq + nk:].view(sh.n_kv, d)
            if sh.qk_norm:
                q, k = self._norm(q, L["qn"]), self._norm(k, L["kn"])
            q, k = self._rot(q, pos), self._rot(k, pos)
            self.K[i, pos] = k
            self.V[i, pos] = v
            Kc = self.K[i, :pos + 1].repeat_interleave(G, dim=1)      # [T, n_q, d]
            Vc = self.V[i, :pos + 1].repeat_interleave(G, dim=1)
            s = torch.einsum("hd,thd->ht", q, Kc) / float(np.sqrt(d))
            p = torch.exp(s - s.max(dim=1, keepdim=True).values)
            o = torch.einsum("ht,thd->hd", p / p.sum(dim=1, keepdim=True), Vc)
            x = x + linear.qlinear(o.reshape(-1), L["o"])
            h = self._norm(x, L["post"])
            gu = linear.qlinear(h, L["gateup"])
            g, u = gu[:sh.ffn], gu[sh.ffn:]
            x = x + linear.qlinear((g / (1 + torch.exp(-g))) * u, L["down"])
        self.pos += 1
        return linear.qlinear(self._norm(x, self.norm), self.head)

    def generate(self, prompt: list, n_new: int):
        """Greedy decoding: the prompt token by token, then n_new tokens each the first maximal
        logit of the step before. Returns (new tokens, the logits of every step after the
        prompt's last token as a host array [n_new, vocab])."""
        self.reset()
        logits = None
        for tk in prompt:
            logits = self.step(tk)
        out, rows = [], []
        for _ in range(n_new):
            tk = int(torch.argmax(logits).item())
            out.append(tk)
            rows.append(logits.float().cpu().numpy())
            logits = self.step(tk)
        return out, np.stack(rows)
