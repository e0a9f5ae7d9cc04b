"""A Qwen3-shaped decoder whose projections are this library's quantized linear layer.

The float math around the projections follows the reference's fp32 model
(opentpu/llm/qwen3.py:701-743 reference_logits):

    x = embed[token]
    per layer: h = rmsnorm(x); q, k, v = h @ Wqkv^T (one QACT + MM: q, k and v share the input
               and its QACT range); per-head rmsnorm of q and k; RoPE (rotate-half, tables from
               float64); causal softmax attention over the cache (GQA); x += o @ Wo^T;
               h = rmsnorm(x); g, u = h @ Wgateup^T (one QACT + MM);
               x += (silu(g) * u) @ Wdown^T, the down projection's input quantized in QACT
               ranges of `down_chunk` columns, one MM each, later ones added in order (ACC), as
               the reference's MLP kernel does (kernels/mlp.py:8-30; compiler.py:2622-2726)
    logits = rmsnorm(x) @ Whead^T (Whead = embed, tied as in Qwen3-0.6B)

`prefill(prompt)` runs the prompt's rows together (each projection one launch over all rows:
QACT is per row, so each row's bits are those of a row alone), `step(token)` one token with the
KV cache, and `generate` picks each next token on the device (otq_argmax: the first maximal
logit, the reference's greedy sink, opentpu/llm/generate.py:252-280).

Every projection runs through linear.qlinear (QACT + MM bit-exact with the reference's MM for
the MX formats and int8-row; weight-only fp32 accumulation for int4-g32); the norms, RoPE,
attention and SwiGLU are fp32 torch on the GPU.
"""
from __future__ import annotations

import numpy as np
import torch

from . import linear
from . import workloads as WL

D = 128


def reference_down_chunk(F: int, fmt: str) -> int | None:
    """The QACT range of the down projection's input in the reference's MLP (kernels/mlp.py:8-30
    _chunk / down_chunk: about F/8 columns, a multiple of D -- 2D for 4-bit rows -- and at least
    2D where F allows); None for the weight-only int4-g32 (no QACT)."""
    if fmt == "int4-g32":
        return None
    q = D if fmt in ("int8", "int8-row") else 2 * D
    if F % q:
        raise ValueError(f"F {F} is not a multiple of {q}")
    lo = min(F, -(-2 * D // q) * q)
    c = max(lo, (F // 8) // q * q)
    while F % c and c > lo:
        c -= q
    while F % c:
        c += q
    return c


def column_parts(w: linear.PackedWeight, C: int) -> list:
    """The weight's column blocks of C as PackedWeights (views of its rows; MX scale rows read
    from block k0 = c0 / 128): MM over one QACT range each (quant.column_parts' layout)."""
    parts = []
    for c0 in range(0, w.K, C):
        if w.fmt in ("int8", "int8-row"):
            rows = w.rows[:, c0:c0 + C]
        else:
            rows = w.rows[:, c0 // 2:(c0 + C) // 2]
        parts.append(linear.PackedWeight(w.fmt, w.N, C, rows, w.srows, w.k0 + c0 // D, w.rsc))
    return parts


class Qwen3Decoder:
    def __init__(self, shape: WL.DecoderShape, weights: dict, fmt: str = "int8-row",
                 head_fmt: str = "int8-row", max_pos: int = 1024, device: str = "cuda",
                 down_chunk="reference"):
        self.shape, self.fmt, self.head_fmt, self.max_pos = shape, fmt, head_fmt, max_pos
        dev = torch.device(device)
        H, d = shape.hidden, shape.head_dim
        self.d = d
        dc = reference_down_chunk(shape.ffn, fmt) if down_chunk == "reference" else down_chunk
        self.down_chunk = dc if dc and dc < shape.ffn else None

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
            L["down_parts"] = column_parts(L["down"], self.down_chunk) if self.down_chunk \
                else [L["down"]]
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
        self.token = torch.zeros(2, dtype=torch.int64, device=dev)

    def _norm(self, v, g):
        return (v / torch.sqrt(torch.mean(v * v, dim=-1, keepdim=True) + self.shape.eps)) * g

    def _rot(self, v, pos):
        """RoPE of v [..., n_heads, d] at positions pos (an int, or a tensor of T positions for
        v [T, n_heads, d])."""
        h = self.d // 2
        c, s = self.cos[pos], self.sin[pos]
        if isinstance(pos, torch.Tensor):
            c, s = c[:, None, :], s[:, None, :]
        v1, v2 = v[..., :h], v[..., h:]
        return torch.cat([v1 * c - v2 * s, v2 * c + v1 * s], dim=-1)

    def _down(self, a, L):
        """The down projection of a [M, F] over its QACT ranges (ACC in range order)."""
        parts = L["down_parts"]
        if len(parts) == 1:
            return linear.qlinear(a, parts[0])
        C = self.down_chunk
        y = linear.qlinear(a[..., :C], parts[0])
        for i, w in enumerate(parts[1:], 1):
            linear.qlinear(a[..., i * C:(i + 1) * C], w, out=y, acc=True)
        return y

    def _layers(self, x, pos0: int):
        """x [T, H] at positions pos0 .. pos0 + T - 1 through every layer (the KV cache holds
        positions < pos0 and receives these)."""
        sh, d = self.shape, self.d
        T = x.shape[0]
        G = sh.n_q // sh.n_kv
        nq, nk = sh.n_q * d, sh.n_kv * d
        pos = torch.arange(pos0, pos0 + T, device=x.device)
        end = pos0 + T
        causal = None
        if T > 1:
            causal = torch.full((T, end), float("-inf"), device=x.device).triu(pos0 + 1)
        for i, L in enumerate(self.layers):
            h = self._norm(x, L["in"])
            qkv = linear.qlinear(h, L["qkv"])
            q = qkv[:, :nq].reshape(T, sh.n_q, d)
            k = qkv[:, nq:nq + nk].reshape(T, sh.n_kv, d)
            v = qkv[:, nq + nk:].reshape(T, sh.n_kv, d)
            if sh.qk_norm:
                q, k = self._norm(q, L["qn"]), self._norm(k, L["kn"])
            q, k = self._rot(q, pos), self._rot(k, pos)
            self.K[i, pos0:end] = k
            self.V[i, pos0:end] = v
            Kc = self.K[i, :end].repeat_interleave(G, dim=1)      # [end, n_q, d]
            Vc = self.V[i, :end].repeat_interleave(G, dim=1)
            s = torch.einsum("thd,uhd->htu", q, Kc) / float(np.sqrt(d))
            if causal is not None:
                s = s + causal
            p = torch.exp(s - s.max(dim=-1, keepdim=True).values)
            o = torch.einsum("htu,uhd->thd", p / p.sum(dim=-1, keepdim=True), Vc)
            x = x + linear.qlinear(o.reshape(T, -1), L["o"])
            h = self._norm(x, L["post"])
            gu = linear.qlinear(h, L["gateup"])
            g, u = gu[:, :sh.ffn], gu[:, sh.ffn:]
            x = x + self._down((g / (1 + torch.exp(-g))) * u, L)
        return x

    def reset(self):
        self.pos = 0

    def prefill(self, prompt: list) -> torch.Tensor:
        """The prompt's tokens at positions 0 .. T - 1, all rows of a projection in one launch:
        the logits [vocab] (fp32) after its last token."""
        T = len(prompt)
        if T > self.max_pos:
            raise ValueError(f"a prompt of {T} past the cache ({self.max_pos})")
        self.pos = 0
        ids = torch.tensor(prompt, dtype=torch.long, device=self.embed.device)
        x = self._layers(self.embed[ids].clone(), 0)
        self.pos = T
        return linear.qlinear(self._norm(x[-1:], self.norm), self.head).reshape(-1)

    def step(self, token: int) -> torch.Tensor:
        """One decode step at the next position: the logits [vocab] (fp32)."""
        if self.pos >= self.max_pos:
            raise ValueError(f"position {self.pos} past the cache ({self.max_pos})")
        x = self._layers(self.embed[token].clone().reshape(1, -1), self.pos)
        self.pos += 1
        return linear.qlinear(self._norm(x, self.norm), self.head).reshape(-1)

    def generate(self, prompt: list, n_new: int, keep_logits: bool = True):
        """Greedy decoding: the prompt (prefill), then n_new tokens, each the first maximal
        logit of the step before (on the device). Returns (new tokens, the logits of every step
        that chose one, as a host array [n_new, vocab], or None)."""
        logits = self.prefill(prompt)
        out, rows = [], []
        for _ in range(n_new):
            linear.argmax(logits, out=self.token)
            tk = int(self.token[0].item())
            out.append(tk)
            if keep_logits:
                rows.append(logits.float().cpu().numpy())
            logits = self.step(tk)
        return out, (np.stack(rows) if keep_logits else None)


def interleave_gate_up(w: linear.PackedWeight) -> linear.PackedWeight:
    """The fused [gate; up] projection's rows reordered for the step kernel's SwiGLU epilogue:
    blocks of 8 gate rows then the matching 8 up rows (rows 16j .. 16j + 7 = gate 8j .. 8j + 7,
    16j + 8 .. 16j + 15 = up 8j .. 8j + 7), scale rows alike; a copy on the GPU."""
    F = w.N // 2
    if w.N % 16:
        raise ValueError("the gate/up projection's rows must be a multiple of 16")
    idx = torch.arange(w.N, device=w.rows.device).view(2, F // 8, 8).permute(1, 0, 2).reshape(-1)
    srows = None if w.srows is None else w.srows.index_select(0, idx).contiguous()
    return linear.PackedWeight(w.fmt, w.N, w.K, w.rows.index_select(0, idx).contiguous(), srows,
                               w.k0, w.rsc)


class FusedDecoder:
    """The decode step of a Qwen3Decoder as ONE persistent launch (otq_decode_step with decoder
    stages): per layer the QKV projection on RMSNorm(residual) (the residual the embedding row
    of the token, or plus the previous layer's down projection), the attention of the token over
    the KV cache (per-head q / k norms, RoPE, causal softmax; the new key and value appended),
    the O projection on the attention output, GateUp on RMSNorm(residual + O), Down on
    SwiGLU(GateUp); then the head on RMSNorm(residual + Down) and the greedy token, which is
    also the next step's input: steps run back to back on the device with no host round trip.

    Shares the decoder's packed weights, norms, RoPE tables and KV cache (so a prompt prefilled
    by Qwen3Decoder.prefill continues here). The down projection's input is one QACT range; the
    decoder should be built with down_chunk=None for the two paths to agree. The float math
    (norms, attention, SwiGLU) is fp32 in another order than the torch path's: equal to fp32
    rounding, then the quantized projections amplify what QACT's rounding makes of it."""

    def __init__(self, dec: "Qwen3Decoder", swiglu_epilogue: bool = True):
        import ctypes
        from . import _lib as L
        if dec.down_chunk is not None:
            raise ValueError("the fused step quantizes the down projection's input as one range: "
                             "build the decoder with down_chunk=None")
        sh, d = dec.shape, dec.d
        if d != 128 or sh.n_q % sh.n_kv or sh.n_q // sh.n_kv > 4:
            raise ValueError("the fused step takes head_dim 128 and at most 4 query heads a KV head")
        self.dec = dec
        maxch = -(-dec.max_pos // 32)
        stages = []          # (kind, fields)

        def proj(w, **kw):
            stages.append(("proj", w, kw))
            return len(stages) - 1

        prev_down = -2
        for i, Lr in enumerate(dec.layers):
            qkv = proj(Lr["qkv"], input=L.IN_NORM, res=prev_down, gamma=Lr["in"])
            stages.append(("attn", None, dict(src=qkv, layer=i)))
            att = len(stages) - 1
            o = proj(Lr["o"], input=L.IN_ATTN, src=att)
            if swiglu_epilogue:   # silu(gate) * up written by the GateUp projection itself
                gu = proj(interleave_gate_up(Lr["gateup"]), input=L.IN_NORM, res=o,
                          gamma=Lr["post"], epilogue=L.EPI_SWIGLU)
                prev_down = proj(Lr["down"], input=L.IN_DEFAULT, src=gu)
            else:                 # ... or computed by the Down projection from both halves
                gu = proj(Lr["gateup"], input=L.IN_NORM, res=o, gamma=Lr["post"])
                prev_down = proj(Lr["down"], input=L.IN_SWIGLU, src=gu)
        proj(dec.head, input=L.IN_NORM, res=prev_down, gamma=dec.norm)
        n = len(stages)
        if n > 160:
            raise ValueError(f"{n} stages: more than the step takes")
        self.projs = (L.StepProj * n)()
        self._keep = []
        for k, (kind, w, kw) in enumerate(stages):
            p = self.projs[k]
            if kind == "attn":
                Lr = dec.layers[kw["layer"]]
                p.fmt, p.src = L.STEP_ATTN, kw["src"]
                p.N, p.K = sh.n_q * d + sh.n_q * maxch * (d + 2), 0
                p.q_gain = Lr["qn"].data_ptr() if sh.qk_norm else None
                p.k_gain = Lr["kn"].data_ptr() if sh.qk_norm else None
                p.kcache = dec.K[kw["layer"]].data_ptr()
                p.vcache = dec.V[kw["layer"]].data_ptr()
                p.n_q, p.n_kv, p.head_dim = sh.n_q, sh.n_kv, d
                continue
            p.rows, p.rs = w.rows.data_ptr(), w.rows.stride(0)
            p.srows = w.srows.data_ptr()
            p.srs = w.srows.stride(0) * w.srows.element_size()
            p.N, p.K = w.N, w.K
            p.fmt = L.STEP_G32 if w.fmt == "int4-g32" else L.STEP_RSC
            p.input = kw["input"]
            p.src = kw.get("src", -1)
            p.res = kw.get("res", -1)
            p.epilogue = kw.get("epilogue", L.EPI_NONE)
            self._keep.append(w)
            if "gamma" in kw:
                p.gamma = kw["gamma"].data_ptr()
        offs = (ctypes.c_int64 * n)()
        total = ctypes.c_int64(0)
        L.call("otq_step_layout", ctypes.addressof(self.projs), n, 1, ctypes.addressof(offs),
               ctypes.byref(total))
        self.offsets, self.stages = list(offs), stages
        dev = dec.embed.device
        self.words = torch.zeros(2 * total.value, dtype=torch.float32, device=dev)
        self.counters = torch.zeros(4, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.token = torch.zeros(2, dtype=torch.int64, device=dev)   # in and out: self-feeding
        st = L.Step()
        st.projs, st.count, st.rank, st.world = ctypes.addressof(self.projs), n, 0, 1
        st.x0, st.out = None, self.words.data_ptr()
        st.counters, st.token = self.counters.data_ptr(), self.token.data_ptr()
        st.eps = sh.eps
        st.rope_cos, st.rope_sin = dec.cos.data_ptr(), dec.sin.data_ptr()
        st.max_pos, st.pos = dec.max_pos, self.pos.data_ptr()
        st.embed, st.token_in, st.vocab = dec.embed.data_ptr(), self.token.data_ptr(), sh.vocab
        self.step_args = st
        nb = ctypes.c_int64(0)
        L.call("otq_step_table_bytes", ctypes.byref(nb))
        self.table = torch.empty(nb.value, dtype=torch.uint8, device=dev)
        L.call("otq_step_prepare", ctypes.addressof(st), self.table.data_ptr())
        self.graph = None
        self.stream = torch.cuda.Stream()

    def logits(self) -> torch.Tensor:
        """The last step's logits [vocab] (the head's output words)."""
        k = len(self.stages) - 1
        N = self.dec.shape.vocab
        o = self.offsets[k]
        return self.words[2 * o:2 * (o + N)].view(N, 2)[:, 0]

    def launch(self):
        import ctypes
        from . import _lib as L
        L.call("otq_decode_step", ctypes.addressof(self.step_args), self.table.data_ptr(),
               torch.cuda.current_stream().cuda_stream)

    def start(self, token: int, pos: int):
        """The next step decodes `token` at position `pos` (the KV cache holds positions < pos)."""
        if not 0 <= pos < self.dec.max_pos:
            raise ValueError(f"position {pos} past the cache ({self.dec.max_pos})")
        self.token[0] = token
        self.pos[0] = pos

    def capture(self):
        """A CUDA graph of one step (the step's state lives on the device: replays continue)."""
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.launch()
        torch.cuda.synchronize()

    def generate(self, prompt: list, n_new: int, keep_logits: bool = True):
        """Greedy decoding: the prompt through the decoder's prefill, then n_new fused steps,
        each feeding its greedy token to the next on the device. Returns (tokens, logits of
        every step that chose one [n_new, vocab] or None)."""
        logits = self.dec.prefill(prompt)
        first = int(torch.argmax(logits).item())
        rows = [logits.float().cpu().numpy()] if keep_logits else None
        out = [first]
        self.start(first, len(prompt))
        for _ in range(n_new - 1):
            self.launch()
            tk = int(self.token[0].item())
            out.append(tk)
            if keep_logits:
                rows.append(self.logits().cpu().numpy())
        return out, (np.stack(rows) if keep_logits else None)
