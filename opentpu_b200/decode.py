"""The quantized projections of one decode token, replayed as one CUDA graph.

A decoder layer's projections in the order a decode step runs them (the reference's
qwen3_step: _attention's q/k/v/o dots, _mlp's gate/up/down, then _lm_head; qwen3.py:1550-2087):

    QKV   [n_q*d + 2*n_kv*d, H]   one GEMV: q, k and v share the input and its QACT range, so
                                  the fused rows give the same bits as three MMs
    O     [H, n_q*d]
    GateUp[2F, H]                 one GEMV for the same reason
    Down  [H, F]
and the LM head [vocab, H] after the last layer.

With world > 1 every projection's rows are split over the ranks (runtime.Weight(shard=0),
runtime.py:138-142) and an all-gather assembles each output on every rank (the reference's
GATHER, isasim.py:1413-1438), captured in the same graph. gather="fused" (the default) fuses it
into the GEMV: every projection's full output row lives in one symmetric buffer (torch
symmetric memory, mapped into every rank) as tagged 8-byte words (value, tag), each rank's
kernel stores its rows' words into every rank's copy over NVLink, and the next projection's
kernel reads its input words until their tags show every rank's output has arrived
(linear.qlinear_peer): no fence, flag or extra launch. gather="nccl" runs an NCCL all-gather
after each projection instead.

gather="tagged" runs a dependent chain of QACT + MM projections on one GPU with the same
tagged words in its own memory (no fan-out): a launch reads its input words until their tags
show the previous launch's output is complete instead of waiting for that launch to end. It is
bit-identical to the plain chain but slower on a B200 (0.672 against 0.623 ms for the
Qwen3-0.6B int8 step: the 8-byte tagged words cost more than the launch-end wait they remove),
so one GPU keeps plain outputs by default.

dependent=True (the default) chains the projections through their outputs the way a decode
step does: each projection reads the first K outputs of the previous one (QKV's q part feeds O,
O feeds GateUp, GateUp's gate part feeds Down, Down feeds the next layer's QKV and, after the
last layer, the head), so every launch waits for the one before it -- the serialization of a
real decode step without the non-linear-layer ops in between. dependent=False gives every
projection its own fixed input.

chained=True runs the whole step as one persistent launch (linear.qlinear_chain: the
projections in order with a grid barrier between them, the next projection's weights streaming
while the grid waits); the default launches one kernel a projection (what world > 1 needs, with
the all-gathers in between).
"""
from __future__ import annotations

import torch

from . import linear
from .workloads import DecoderShape


def shard_rows(N: int, world: int, rank: int) -> tuple[int, int]:
    """Rank `rank`'s contiguous rows [n0, n1) of an N-row projection split over `world` ranks
    (runtime.Weight(shard=0), runtime.py:138-142: equal contiguous row blocks); an all-gather of
    the ranks' outputs in rank order is the whole output row."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if N % world:
        raise ValueError(f"{N} rows do not split over {world} ranks")
    n = N // world
    return rank * n, (rank + 1) * n


def step_plan(shape: DecoderShape, fmt: str, head_fmt: str):
    """(name, N, K, fmt) of every projection of a decode step, in order: per layer QKV, O,
    GateUp, Down, then the head."""
    H, d = shape.hidden, shape.head_dim
    qkv = shape.n_q * d + 2 * shape.n_kv * d
    layer = [("qkv", qkv, H), ("o", H, shape.n_q * d), ("gateup", 2 * shape.ffn, H),
             ("down", H, shape.ffn)]
    plan = [(f"layers.{i}.{n}", N, K, fmt) for i in range(shape.layers) for n, N, K in layer]
    plan.append(("head", shape.vocab, H, head_fmt))
    return plan


def seeded_weights(plan, seed: int, world: int, rank: int, std: float = 0.02, whole=()):
    """The step's packed weights (this rank's row shard of each; all rows of the projections
    whose indices are in `whole`) and first-input rows, drawn from one generator in plan order:
    every world size and rank sees the same matrices. Returns (weights, inputs {K: [1, K]},
    the step's weight bytes -- each projection once)."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    weights, inputs, nbytes = [], {}, 0
    for i, (name, N, K, f) in enumerate(plan):
        try:
            n0, n1 = (0, N) if i in whole else shard_rows(N, world, rank)
        except ValueError as e:
            raise ValueError(f"{name}: {e}") from None
        W = torch.randn((N, K), generator=gen, device="cuda")[n0:n1] * std
        w = linear.PackedWeight.from_float(W, f)
        del W
        weights.append(w)
        nbytes += w.stream_bytes * (1 if i in whole else world)
        if K not in inputs:
            inputs[K] = torch.randn((1, K), generator=gen, device="cuda")
    return weights, inputs, nbytes


class DecodeStep:
    """The decode step as ONE persistent launch (otq_decode_step): the same projections, seeded
    weights and chaining as DecodeChain(dependent=True) -- each projection reads the first K
    outputs of the one before, the first reads a fixed input -- ordered by tagged output words
    instead of kernel boundaries, the greedy token folded into the head's epilogue. Layers in
    int8-row (bit-identical to DecodeChain) or int4-g32 (weight-only, fp32 sums in another
    order than otq_linear_g32's); the head in int8-row. With world > 1 the rows are sharded and
    every output word is stored into every rank's copy of a symmetric buffer over NVLink (the
    all-gather fused in): bit-identical to one GPU. shard="head" shards only the LM head and
    has every rank compute the layers' projections whole (their outputs never cross NVLink:
    at this model size a projection's NVLink hand-off costs more than its rows take to stream).
    """

    def __init__(self, shape: DecoderShape, fmt: str = "int8-row", head_fmt: str = "int8-row",
                 seed: int = 0, world: int = 1, rank: int = 0, group=None, shard: str = "all"):
        import ctypes
        from . import _lib as L
        if fmt not in ("int8-row", "int4-g32") or head_fmt != "int8-row":
            raise ValueError("the persistent decode step takes int8-row or int4-g32 layers and "
                             "an int8-row head")
        if shard not in ("all", "head"):
            raise ValueError("shard is 'all' or 'head'")
        self.shape, self.world, self.rank, self.group = shape, world, rank, group
        self.plan = step_plan(shape, fmt, head_fmt)
        n = len(self.plan)
        whole = set(range(n - 1)) if (shard == "head" and world > 1) else set()
        self.weights, self.inputs, self.weight_bytes = seeded_weights(self.plan, seed, world, rank,
                                                                      whole=whole)
        # the bytes this rank streams a step
        self.rank_bytes = sum(w.stream_bytes for w in self.weights)
        self.projs = (L.StepProj * n)()
        for i, w in enumerate(self.weights):
            p = self.projs[i]
            p.rows, p.rs = w.rows.data_ptr(), w.rows.stride(0)
            p.srows = w.srows.data_ptr()
            p.srs = w.srows.stride(0) * w.srows.element_size()
            p.N, p.K, p.src = w.N, w.K, i - 1
            p.fmt = L.STEP_G32 if w.fmt == "int4-g32" else L.STEP_RSC
            p.replicated = 1 if i in whole else 0
        offs = (ctypes.c_int64 * n)()
        total = ctypes.c_int64(0)
        L.call("otq_step_layout", ctypes.addressof(self.projs), n, world, ctypes.addressof(offs),
               ctypes.byref(total))
        self.offsets = list(offs)
        words = total.value
        if world > 1:
            import torch.distributed as dist
            import torch.distributed._symmetric_memory as symm
            try:
                symm.set_backend("CUDA")
            except Exception:
                pass
            buf = symm.empty(2 * words, dtype=torch.float32, device="cuda")
            buf.zero_()
            grp = group if group is not None else dist.group.WORLD
            handle = symm.rendezvous(buf, grp)
            torch.cuda.synchronize()
            dist.barrier(group=grp)
            ptrs = handle.buffer_ptrs
        else:
            buf = torch.zeros(2 * words, dtype=torch.float32, device="cuda")
            handle, ptrs = None, [buf.data_ptr()]
        self._buf = (buf, handle)
        self.counters = torch.zeros(4, dtype=torch.int32, device="cuda")
        self.token = torch.zeros(2, dtype=torch.int64, device="cuda")
        self.x0 = self.inputs[self.plan[0][2]]
        st = L.Step()
        st.projs, st.count, st.rank, st.world = ctypes.addressof(self.projs), n, rank, world
        for r in range(world):
            st.delta[r] = ptrs[r] - ptrs[rank]
        st.x0, st.out = self.x0.data_ptr(), buf.data_ptr()
        st.counters, st.token = self.counters.data_ptr(), self.token.data_ptr()
        self.step_args = st
        nb = ctypes.c_int64(0)
        L.call("otq_step_table_bytes", ctypes.byref(nb))
        self.table = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
        L.call("otq_step_prepare", ctypes.addressof(st), self.table.data_ptr())
        self.graph = None
        self.stream = torch.cuda.Stream()

    @property
    def launches(self) -> int:
        return 1

    def full_out(self, i: int) -> torch.Tensor:
        """Projection i's whole output row [1, N] (the values of its tagged words)."""
        N = self.plan[i][1]
        o = self.offsets[i]
        return self._buf[0][2 * o:2 * (o + N)].view(N, 2)[:, 0].unsqueeze(0)

    def logits(self) -> torch.Tensor:
        return self.full_out(len(self.plan) - 1)

    def step_eager(self):
        import ctypes
        from . import _lib as L
        L.call("otq_decode_step", ctypes.addressof(self.step_args), self.table.data_ptr(),
               torch.cuda.current_stream().cuda_stream)

    def capture(self, warmup: int = 3):
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                self.step_eager()
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.step_eager()
        torch.cuda.synchronize()

    def replay(self, n: int = 1):
        with torch.cuda.stream(self.stream):
            for _ in range(n):
                self.graph.replay()

    def run_host(self, inputs_host: dict, token_host: torch.Tensor):
        """One step from host buffers: the first input copied from pinned host memory, the
        step, the greedy token copied back into token_host (pinned; all asynchronous on the
        step's stream)."""
        K = self.plan[0][2]
        with torch.cuda.stream(self.stream):
            self.x0.copy_(inputs_host[K], non_blocking=True)
            self.graph.replay()
            token_host.copy_(self.token[:1], non_blocking=True)

    def release(self):
        self.graph = None


class DecodeChain:
    def __init__(self, shape: DecoderShape, fmt: str = "int8-row", head_fmt: str = "int8-row",
                 seed: int = 0, world: int = 1, rank: int = 0, group=None, pdl: bool = True,
                 std: float = 0.02, dependent: bool = True, chained: bool | None = None,
                 gather: str = "fused"):
        self.shape, self.world, self.rank, self.group, self.pdl = shape, world, rank, group, pdl
        if gather not in ("fused", "nccl", "tagged"):
            raise ValueError("gather must be 'fused', 'nccl' or 'tagged'")
        mm_only = fmt != "int4-g32" and head_fmt != "int4-g32"   # the tagged path is QACT + MM
        if gather == "tagged" and (world > 1 or not (dependent and mm_only) or chained):
            raise ValueError("gather='tagged' is a dependent QACT + MM chain on one GPU")
        self.fused = (world > 1 and gather == "fused") or gather == "tagged"
        self.dependent = dependent
        # chained: the whole step as one persistent launch (linear.qlinear_chain). Measured on
        # a B200 it is slower today than one launch a projection (1.12 vs 0.61 ms for the
        # Qwen3-0.6B step: per projection the grid barrier and the QACT prologue cost as much as
        # a launch, and a warp's ring holds under one projection of look-ahead), so it is opt-in.
        self.chained = bool(chained)
        self.plan = step_plan(shape, fmt, head_fmt)
        self.weights, self.inputs, self.weight_bytes = seeded_weights(self.plan, seed, world,
                                                                      rank, std)
        self.outs, self.gathered = [], []
        if not self.fused:
            for w in self.weights:
                self.outs.append(torch.zeros((1, w.N), device="cuda"))
                self.gathered.append(torch.zeros((world, w.N), device="cuda") if world > 1
                                     else None)
        if self.fused:
            self._symmetric_outputs()
        # the input each projection reads: a fixed vector, or the previous projection's output
        self.x_of = []
        for i, (name, N, K, f) in enumerate(self.plan):
            if not dependent or i == 0:
                self.x_of.append(self.inputs[K])
            elif self.fused:   # the previous projection's tagged words
                if self.full[i - 1].shape[0] < K:
                    raise ValueError(f"{name}: the previous output has {self.full[i - 1].shape[0]} < {K}")
                self.x_of.append(self.full[i - 1][:K])
            else:
                prev = self.full_out(i - 1)
                if prev.shape[1] < K:
                    raise ValueError(f"{name}: the previous output has {prev.shape[1]} < {K}")
                self.x_of.append(prev[:, :K])
        self.graph = None
        self.stream = torch.cuda.Stream()
        self.table = None
        # the greedy token of the step (the reference's device argmax over the head's logits,
        # llm/generate.py:252-280): word 0 of this buffer after every step
        self.token = torch.zeros(2, dtype=torch.int64, device="cuda")
        if self.chained:
            if world > 1:
                raise ValueError("a chained step has no all-gather: world must be 1")
            self.table = linear.chain_table([(x, w, y, False, False) for x, w, y in
                                             zip(self.x_of, self.weights, self.outs)])

    def _symmetric_outputs(self):
        """Every projection's full output row as tagged words ([N, 2] float32: value, tag bits)
        in one buffer (16-byte aligned slots): symmetric with world > 1, plain device memory on
        one GPU; this rank's step count and the last launch's CTA count in ordinary device
        memory. All zero before the first launch. The launches use stepped tags: position i of
        the step waits on the tags of position i - 1's output, not on that launch's end."""
        from . import _lib as L
        offs, tot = [], 0
        for _, N, _, _ in self.plan:
            offs.append(tot)
            tot += 2 * (-(-N // 2) * 2)   # N words of 8 bytes, rounded to 16 bytes
        if self.world > 1:
            import torch.distributed as dist
            import torch.distributed._symmetric_memory as symm
            try:
                symm.set_backend("CUDA")
            except Exception:
                pass   # already chosen by an earlier allocation
            buf = symm.empty(tot, dtype=torch.float32, device="cuda")
            buf.zero_()
            group = self.group if self.group is not None else dist.group.WORLD
            handle = symm.rendezvous(buf, group)
            torch.cuda.synchronize()
            dist.barrier(group=group)
            ptrs = handle.buffer_ptrs
        else:
            buf = torch.zeros(tot, dtype=torch.float32, device="cuda")
            handle, ptrs = None, [buf.data_ptr()]
        self._symm = (buf, handle)
        self.counters = torch.zeros(2, dtype=torch.int32, device="cuda")   # steps, done CTAs
        self.full, self.peers = [], []
        for i, (o, (_, N, _, _)) in enumerate(zip(offs, self.plan)):
            words = buf[o:o + 2 * N].view(N, 2)
            n0, n1 = shard_rows(N, self.world, self.rank)
            self.full.append(words)
            self.outs.append(words[n0:n1])
            self.gathered.append(None)
            pr = L.Peer()
            pr.rank, pr.world = self.rank, self.world
            pr.wait = int(self.dependent and i > 0)
            for r in range(self.world):
                pr.delta[r] = ptrs[r] - ptrs[self.rank]
            pr.seq = self.counters.data_ptr()
            pr.done = self.counters.data_ptr() + 4
            pr.tags = L.TAGS_STEPPED
            pr.step_pos = i
            pr.step_last = int(i == len(self.plan) - 1)
            self.peers.append(pr)

    @property
    def launches(self) -> int:
        return (1 if self.chained else len(self.plan)) + 1   # + the argmax

    def full_out(self, i: int) -> torch.Tensor:
        """Projection i's whole output row [1, N] (the gathered one with world > 1)."""
        if self.fused:   # the values of the tagged words
            return self.full[i][:, 0].unsqueeze(0)
        return self.gathered[i].reshape(1, -1) if self.world > 1 else self.outs[i]

    def step_eager(self):
        import torch.distributed as dist
        if self.chained:
            linear.qlinear_chain(self.table)
        elif self.fused:
            for x, w, y, pr in zip(self.x_of, self.weights, self.outs, self.peers):
                linear.qlinear_peer(x, w, y, pr, pdl=self.pdl)
        else:
            for x, w, y, g in zip(self.x_of, self.weights, self.outs, self.gathered):
                linear.qlinear(x, w, out=y, pdl=self.pdl)
                if self.world > 1:
                    dist.all_gather_into_tensor(g, y, group=self.group)
        linear.argmax(self.logits(), out=self.token)

    def capture(self, warmup: int = 3):
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                self.step_eager()
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.step_eager()
        torch.cuda.synchronize()

    def replay(self, n: int = 1):
        with torch.cuda.stream(self.stream):
            for _ in range(n):
                self.graph.replay()

    def run_host(self, inputs_host: dict, token_host: torch.Tensor):
        """One step from host buffers: each input vector copied from pinned host memory, the
        graph replayed, the greedy token id copied back into token_host (int64 [1], pinned; all
        on the chain's stream, asynchronous)."""
        with torch.cuda.stream(self.stream):
            for K, t in inputs_host.items():
                if not self.dependent or K == self.plan[0][2]:
                    self.inputs[K].copy_(t, non_blocking=True)
            self.graph.replay()
            token_host.copy_(self.token[:1], non_blocking=True)

    def logits(self) -> torch.Tensor:
        return self.full_out(len(self.plan) - 1)

    def release(self):
        self.graph = None
        self.table = None
