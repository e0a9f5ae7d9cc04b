"""Benchmark of the quantized linear layer's hot path.

Main line (configuration 2): one step = one decode token through every quantized projection of
a Qwen3-0.6B-shaped decoder (28 layers x q, k, v, o, gate, up, down, then the 151936 x 1024 LM
head; int8 per-row weights from N(0, 0.02), the first input N(0, 1)). q/k/v and gate/up share
their input and QACT range, so each group is one launch: 113 fused QACT+MM launches a step, each
reading the previous launch's output as a decode step does (opentpu_b200.decode.DecodeChain,
dependent), then the greedy token (device argmax of the logits), replayed as one CUDA graph.
The weights (598 MB) exceed the 126 MB L2, so each step streams them from HBM.

metric: decode weight GB/s (whole job) with tok/s = steps / s beside it. With --gpus N each
projection's output rows are split over the N ranks (the reference's Weight(shard=0)) and every
projection's output is assembled on every rank (the reference's GATHER) inside the GEMV itself:
each rank stores its rows' tagged 8-byte words into every rank's copy over NVLink and the next
projection reads them when their tags arrive (DecodeChain gather="fused"). After timing, rank 0
replays the same seeded step on one GPU and compares the logits bit for bit ("parity").

Objects of the same line:
- "roofline": the dominant kernel, the 112 layer-projection launches of a step (95 % of its
  time), timed as their own graph with CUDA events; "roofline_head" the LM-head launch alone.
- "e2e": a closed greedy loop through the public API (DecodeChain.run_host): each step copies
  its input vector from pinned host memory (the row of a host table picked by the previous
  token), replays the step, copies the token back, waits for it and reads it on the host.
- "cpu_baseline": the reference's exact MM algorithm (oracle port, all host cores) on a bounded
  sample; "cpu_baseline_blas": the reference's weight-only float path `deq @ x` (numpy fp32
  BLAS, all host cores) on a bounded sample.
- "config1": BASELINE configuration 1 (1024 x 1024 int8 per-row GEMV) as a latency, over a
  rotating pool of 256 distinct weight copies (257 MB > 2 x L2) and L2-resident.
- "decode_4bit": configuration 3 (int4-g32 layers, int8-row head) with its own roofline, CPU
  baseline and closed-loop e2e.
- "phi4_sweep": configuration 5 (Phi-4-mini projections and head, int8-row and int4-g32, batch
  1 / 8 / 64, row-sharded with an all-gather per output when N > 1).
- "prefill": configuration 4 (36 SmolLM3-3B-shaped int8-row layers, 512 bf16 tokens, tcgen05
  GEMM); with N > 1 each projection's rows are sharded and its output all-gathered (NCCL) in the
  timed graph, and rank 0 checks layer 0 against the unsharded GEMM within the tolerance.

--profile head|step|prefill|g32|stepkernel|stepkernel4 runs a few launches and exits (the commands the ncu summaries
under profiles/ were captured with). --impl reference times the reference's CPU algorithm (the
numpy port under oracle/, the same arithmetic as the reference's MM) on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from opentpu_b200 import workloads as WL  # noqa: E402

METRIC = "decode weight GB/s"
UNIT = "GB/s"
PREFILL_TOKENS = 512


def peaks():
    """(HBM GB/s, bf16 burst TFLOP/s, kind): MEASURED_PEAKS.json, else the pool's fallback."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def host_threads():
    """Every host core for the CPU baselines, whatever OMP_NUM_THREADS torchrun set: (the
    threadpoolctl context or None, the thread count)."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits
        return threadpool_limits(limits=n), n
    except Exception:
        return None, 1


def threads_used():
    try:
        from threadpoolctl import threadpool_info
        return max([i.get("num_threads", 1) for i in threadpool_info()] + [1])
    except Exception:
        return 1


class Clocks:
    """nvidia-smi sampling while the timed regions run (SM clock, throttle reasons). The first
    sample is awaited before the timed region starts."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.rows and time.time() - t0 < 5 and self.proc.poll() is None:
                time.sleep(0.02)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.15)   # one more sample after the last timed kernel
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        mhz = [v for v in (num(r[1]) for r in self.rows if len(r) > 1) if v is not None]
        mx = [v for v in (num(r[2]) for r in self.rows if len(r) > 2) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 5 + i and r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


# ------------------------------------------------------------------------------ timing helpers
def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def graph_ms(graph, stream, reps: int, world: int) -> float:
    """Milliseconds a replay of `graph` (CUDA events on its stream, max over ranks)."""
    import torch
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    return max_over_ranks(e0.elapsed_time(e1) / reps, world)


def capture(fn, stream, warm: int = 2):
    """A CUDA graph of fn() on `stream` (after `warm` eager runs)."""
    import torch
    with torch.cuda.stream(stream):
        for _ in range(warm):
            fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    torch.cuda.synchronize()
    return g


def read_traffic(name: str, world: int):
    """dram bytes per launch from a committed ncu summary (one GPU only), or None."""
    tp = ROOT / "profiles" / name
    if tp.exists() and world == 1:
        for line in tp.read_text().splitlines():
            if line.startswith("| dram_bytes_per_launch |"):
                return int(line.split("|")[2])
    return None


# ------------------------------------------------------------------------------ CPU baselines
def cpu_exact_sample(budget_s: float = 10.0, shape=WL.QWEN3_0_6B):
    """The oracle's exact decode GEMV (the reference's MM algorithm) on every host core over a
    bounded sample of the step's projections: (GB/s of weight bytes, description, threads)."""
    from oracle import fp32 as F
    from oracle import mx as X
    lim, n = host_threads()
    try:
        rng = np.random.default_rng(0)
        shapes = [(N, K) for _, N, K in shape.projections()] + [(16384, shape.hidden)]
        mats = []
        for N, K in shapes:
            W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
            q, s = X.quantize_rows_rsc(W)
            mats.append((q, s, rng.standard_normal(K).astype(np.float32), K))
        nbytes = sum(q.shape[0] * (q.shape[1] + 4) for q, _, _, _ in mats)
        done, t0 = 0, time.perf_counter()
        while True:
            for q, s, x, K in mats:
                qa, Sa, da = F.quantize_rows(x[None, :], 32)
                X.mm(qa, Sa, da, q, s, "int8", K, rsc=True)
            done += 1
            el = time.perf_counter() - t0
            if el > budget_s or done >= 50:
                break
        th = threads_used()
    finally:
        if lim is not None:
            lim.restore_original_limits()
    desc = (f"{done} passes over 1 layer (7 projections) + a 16384-row head slice "
            f"({nbytes / 1e6:.1f} MB of int8 rows), exact MM port (QACT + integer MM), numpy, "
            f"{n} host threads allowed")
    return done * nbytes / el / 1e9, desc, th


def cpu_blas_sample(fmt: str = "int8-row", budget_s: float = 4.0, shape=WL.QWEN3_0_6B):
    """The reference's weight-only float path, `deq @ x` in numpy fp32 BLAS (reference.py:14-17
    on quant.quantize's deq), on every host core: one layer's seven projections + a 16384-row
    head slice, GB/s of the format's packed weight bytes. (value, description, threads)."""
    from oracle import survey as SV
    lim, n = host_threads()
    try:
        rng = np.random.default_rng(0)
        shapes = [(N, K, fmt) for _, N, K in shape.projections()] + [(16384, shape.hidden,
                                                                      "int8-row")]
        mats, nbytes = [], 0
        for N, K, f in shapes:
            W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
            if f == "int4-g32":
                _, _, deq = SV.quantize_g32(W)
                nbytes += N * K // 2 + N * K // 32 * 2
            else:
                sw = np.abs(W).max(1, keepdims=True) / 127
                deq = (np.rint(W / sw) * sw).astype(np.float32)
                nbytes += N * (K + 4)
            mats.append((np.ascontiguousarray(deq), rng.standard_normal(K).astype(np.float32)))
        done, t0 = 0, time.perf_counter()
        while True:
            for d, x in mats:
                d @ x
            done += 1
            el = time.perf_counter() - t0
            if el > budget_s or done >= 2000:
                break
        th = threads_used()
    finally:
        if lim is not None:
            lim.restore_original_limits()
    desc = (f"{done} passes of `deq @ x` (numpy fp32 BLAS) over 1 layer ({fmt}) + a 16384-row "
            f"int8-row head slice, {nbytes / 1e6:.1f} MB of packed weights a pass")
    return done * nbytes / el / 1e9, desc, th


def prefill_cpu_sample(budget_s: float = 6.0):
    """The oracle's float64 `deq @ x` (oracle/prefill.py) on every host core over one 2048 x
    2048 projection at 512 tokens: (TFLOP/s, description, threads)."""
    from oracle import prefill as PF
    lim, n = host_threads()
    try:
        rng = np.random.default_rng(0)
        K = N = 2048
        x = PF.bf16_round(rng.standard_normal((PREFILL_TOKENS, K)).astype(np.float32))
        rows = rng.integers(-127, 128, (N, K), dtype=np.int8).view(np.uint8)
        srows = (rng.random(N).astype(np.float32) * 1e-3).view(np.uint8).reshape(N, 4)
        done, t0 = 0, time.perf_counter()
        while True:
            PF.gemm_w8a16(x, rows, srows, K)
            done += 1
            el = time.perf_counter() - t0
            if el > budget_s or done >= 20:
                break
        th = threads_used()
    finally:
        if lim is not None:
            lim.restore_original_limits()
    flops = 2.0 * PREFILL_TOKENS * N * K
    desc = (f"{done} x one 2048x2048 projection at 512 tokens, float64 numpy (oracle, also "
            "forms the error bound |x| @ |deq|^T)")
    return done * flops / el / 1e12, desc, th


# ------------------------------------------------------------------------------ decode objects
def layers_roofline(chain, world, reps, hbm, peak_kind, kernel, traffic_name=None):
    """The step's layer projections (all launches but the head's and the argmax) as their own
    graph, launched as in the step: bytes (weights + scales + x + y) / CUDA-event time."""
    import torch
    from opentpu_b200 import linear
    items = list(zip(chain.x_of[:-1], chain.weights[:-1], chain.outs[:-1]))

    def run():
        for x, w, y in items:
            linear.qlinear(x, w, out=y, pdl=chain.pdl)
    g = capture(run, chain.stream)
    graph_ms(g, chain.stream, 3, world)
    ms = graph_ms(g, chain.stream, reps, world)
    nbytes = sum(w.stream_bytes + 4 * w.K + 4 * w.N for _, w, _ in items)
    achieved = nbytes / (ms * 1e-3) / 1e9
    del g
    torch.cuda.synchronize()
    return {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
            "frac": achieved / hbm, "traffic": read_traffic(traffic_name, world)
            if traffic_name else None,
            "kernel": kernel, "launches_per_step": len(items), "bytes_per_step": nbytes,
            "us_per_step": ms * 1e3, "us_per_launch": ms * 1e3 / len(items),
            "peak_kind": f"{peak_kind} (copy)"}


def head_roofline(chain, stream, world, hbm, peak_kind):
    """The LM-head launch alone (this rank's rows), 20 launches in a graph, launched as in the
    step (programmatic dependent launch)."""
    import torch
    from opentpu_b200 import linear
    head, hx = chain.weights[-1], chain.inputs[chain.shape.hidden]
    hy = torch.empty((1, head.N), device="cuda")

    def run():
        for _ in range(20):
            linear.qlinear(hx, head, out=hy, pdl=True)
    g = capture(run, stream, warm=1)
    graph_ms(g, stream, 1, world)
    ms = graph_ms(g, stream, 5, world) / 20
    nbytes = head.stream_bytes + head.K * 4 + head.N * 4
    achieved = nbytes / (ms * 1e-3) / 1e9
    del g
    return {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
            "frac": achieved / hbm,
            "traffic": read_traffic("gemv_kernel_lm_head_int8row_151936x1024_m1.md", world),
            "kernel": f"gemv_kernel (LM head launch, {head.N}x{head.K} {head.fmt}, M=1)",
            "bytes_per_launch": nbytes, "us_per_launch": ms * 1e3,
            "peak_kind": f"{peak_kind} (copy)"}


def closed_loop(chain, n: int, world: int):
    """Greedy decode through the public API from host buffers: each step's input is the row of
    a pinned host table picked by the previous step's token (copied to the device), the step's
    graph replays, the token comes back to pinned host memory, the host waits for it and reads
    it. Returns (wall ms a token, max over ranks; h2d bytes, d2h bytes, tokens seen)."""
    import torch
    K = chain.plan[0][2]
    table = torch.randn((64, K), generator=torch.Generator().manual_seed(5)).pin_memory()
    tok_host = torch.zeros(1, dtype=torch.int64).pin_memory()
    tok, seen = 0, []
    for _ in range(3):
        chain.run_host({K: table[tok % 64]}, tok_host)
        chain.stream.synchronize()
        tok = int(tok_host[0])
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(n):
        chain.run_host({K: table[tok % 64]}, tok_host)
        chain.stream.synchronize()
        tok = int(tok_host[0])
        seen.append(tok)
    wall = (time.perf_counter() - t0) / n * 1e3
    return max_over_ranks(wall, world), K * 4, 8, seen


def config1(world: int, reps: int):
    """W N(0, 0.02) [1024, 1024] -> int8 per row + fp32 scale, x
    N(0, 1) [1024], M = 1, as a latency. Rotating pool: 256 distinct copies of the packed
    weight (257 MB, more than twice the 126 MB L2), one launch each, in one graph; L2-resident:
    one copy launched 256 times. Bytes a launch = 1 060 864 (W + Sw + x + y)."""
    import torch
    from opentpu_b200 import linear
    W, x = WL.gemv_config1(0)
    w0 = linear.PackedWeight.from_float(torch.from_numpy(W).cuda(), "int8-row")
    xs = torch.from_numpy(x).cuda().reshape(1, -1)
    pool = [linear.PackedWeight("int8-row", w0.N, w0.K, w0.rows.clone(), w0.srows.clone())
            for _ in range(256)]
    y = torch.empty((1, 1024), device="cuda")
    stream = torch.cuda.Stream()
    nbytes = 1024 * 1024 + 4096 + 4096 + 4096
    out = {}
    for name, ws in (("pool", pool), ("l2_resident", [w0] * 256)):
        def run(ws=ws):
            for w in ws:
                linear.qlinear(xs, w, out=y, pdl=True)
        g = capture(run, stream, warm=1)
        graph_ms(g, stream, 2, world)
        ms = graph_ms(g, stream, reps, world) / len(ws)
        out[name] = {"us_per_gemv": ms * 1e3, "GB/s": nbytes / (ms * 1e-3) / 1e9}
        del g
    del pool
    torch.cuda.synchronize()
    return {"metric": "1024x1024 int8-row GEMV latency", "unit": "us",
            "value": out["pool"]["us_per_gemv"], "higher_is_better": False,
            "bytes_per_gemv": nbytes, **out,
            "config": {"workload": "BASELINE configuration 1: W N(0,0.02) 1024x1024 int8 per "
                                   "row + fp32 scale, x N(0,1) fp32 [1024], seed 0, M=1",
                       "pool": "256 distinct packed copies (257 MB > 2 x 126 MB L2), one "
                               "launch each in one CUDA graph (PDL)",
                       "l2_resident": "one copy launched 256 times"}}


def g32_gemv_roofline(hbm, peak_kind):
    """The standalone int4-g32 GEMV (otq_linear_g32, one activation row) on a 65536 x 4096
    weight (151 MB of codes and fp16 scales, more than L2): 20 launches in a CUDA graph with
    programmatic dependent launch, CUDA events."""
    import torch
    from opentpu_b200 import linear
    gen = torch.Generator(device="cuda").manual_seed(3)
    N, K = 65536, 4096
    codes = torch.randint(0, 256, (N, K // 2), dtype=torch.int32, device="cuda",
                          generator=gen).to(torch.uint8)
    sc = (torch.rand((N, K // 32), device="cuda", generator=gen) * 1e-3 + 1e-4).half()
    w = linear.PackedWeight("int4-g32", N, K, codes, sc)
    x = torch.randn((1, K), device="cuda", generator=gen)
    y = torch.empty((1, N), device="cuda")
    stream = torch.cuda.Stream()
    g = capture(lambda: [linear.qlinear(x, w, out=y, pdl=True) for _ in range(20)], stream, warm=1)
    graph_ms(g, stream, 2, 1)
    ms = graph_ms(g, stream, 10, 1) / 20
    del g
    nbytes = w.stream_bytes + 4 * K + 4 * N
    ach = nbytes / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
            "kernel": "linear_g32_mma_kernel (65536x4096 int4-g32, M=1)",
            "bytes_per_launch": nbytes, "us_per_launch": ms * 1e3,
            "peak_kind": f"{peak_kind} (copy)"}


def decode_4bit(args, world, rank, group, hbm, peak_kind):
    """BASELINE configuration 3's decode step: the Qwen3-0.6B step with int4-g32 layers (fp16
    group scales, weight-only, fp32 activations) and the int8-row head, as one persistent launch
    a step (row shards over the ranks, every projection's output words stored to every rank)."""
    import torch
    from opentpu_b200.decode import DecodeStep
    shape = WL.QWEN3_0_6B
    c4 = DecodeStep(shape, fmt="int4-g32", head_fmt="int8-row", world=world, rank=rank,
                    group=group, shard=args.shard)
    c4.capture()
    c4.replay(args.warmup)
    torch.cuda.synchronize()
    n4 = max(10, args.steps)
    ms4 = graph_ms(c4.graph, c4.stream, n4, world)
    per_rank = c4.rank_bytes + sum(4 * K + 8 * N for _, N, K, _ in c4.plan)
    ach = per_rank / (ms4 * 1e-3) / 1e9
    roof = {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
            "traffic": read_traffic("step_kernel_qwen3_0_6b_int4g32.md", world),
            "kernel": "step_kernel (the whole 4-bit decode step, one persistent launch)",
            "bytes_per_launch": per_rank, "us_per_launch": ms4 * 1e3,
            "peak_kind": f"{peak_kind} (copy)"}
    e2e_ms, h2d, d2h, _ = closed_loop(c4, max(10, min(args.steps, 200)), world)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, desc, th = cpu_blas_sample("int4-g32")
        cpu = {"value": v, "unit": UNIT, "cores": th, "kind": "port", "sample": desc}
    out = {"metric": METRIC, "value": c4.weight_bytes / (ms4 * 1e-3) / 1e9, "unit": UNIT,
           "ms_per_step": ms4, "tok_s": 1e3 / ms4, "steps": n4,
           "config": {"workload": "Qwen3-0.6B-shaped decode step, layers int4 group-32 fp16 "
                                  "scales (weight-only, fp32 activations), 151936x1024 "
                                  "int8-row LM head, M=1 (BASELINE configuration 3)",
                      "weights_bytes_per_step": c4.weight_bytes,
                      "parallelism": f"row-shard x{world}" + (" + each projection's output "
                                                             "words stored to every rank "
                                                             "inside the step kernel"
                                                             if world > 1 else "")},
           "roofline": roof, "cpu_baseline": cpu,
           "e2e": {"value": c4.weight_bytes / (e2e_ms * 1e-3) / 1e9, "unit": UNIT,
                   "ms_per_token": e2e_ms, "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": d2h, "api": "DecodeStep.run_host, closed loop"},
           "gpu_launches": c4.launches * n4}
    c4.release()
    del c4
    torch.cuda.synchronize()
    out["mx_int4x"] = decode_mx_int4(args, world, rank, group)
    if world == 1:
        out["gemv_roofline"] = g32_gemv_roofline(hbm, peak_kind)
    return out


def decode_mx_int4(args, world, rank, group):
    """The same step with the reference's own MX 4-bit format (int4x: a byte of offsets and 4-bit
    multipliers a 128-element block, opentpu/quant.py:325-369) in the layers and the int8-row
    head, exact QACT + MM, through the launch chain (one launch a projection; the step kernel
    takes int8-row and int4-g32 only)."""
    import torch
    from opentpu_b200.decode import DecodeChain
    shape = WL.QWEN3_0_6B
    ch = DecodeChain(shape, fmt="int4", head_fmt="int8-row", world=world, rank=rank, group=group)
    ch.capture()
    ch.replay(args.warmup)
    torch.cuda.synchronize()
    n = max(10, args.steps)
    ms = graph_ms(ch.graph, ch.stream, n, world)
    res = {"metric": METRIC, "value": ch.weight_bytes / (ms * 1e-3) / 1e9, "unit": UNIT,
           "ms_per_step": ms, "tok_s": 1e3 / ms, "steps": n,
           "weights_bytes_per_step": ch.weight_bytes,
           "launch": "one gemv launch a projection + the argmax, one CUDA graph a step",
           "gpu_launches": ch.launches * n}
    ch.release()
    del ch
    torch.cuda.synchronize()
    return res


def parity_vs_one_gpu(chain, world, rank):
    """Rank 0: the same seeded step replayed unsharded on one GPU; the sharded step's logits and
    token compared bit for bit (the other ranks wait at a barrier)."""
    import torch
    res = None
    torch.cuda.synchronize()
    if rank == 0:
        one = type(chain)(chain.shape, seed=0)
        one.step_eager()
        torch.cuda.synchronize()
        a = chain.logits().float().contiguous().cpu().numpy().view(np.uint32)
        b = one.logits().float().contiguous().cpu().numpy().view(np.uint32)
        same = bool(np.array_equal(a, b))
        res = {"vs_1gpu": "bit-identical" if same else "differs",
               "token": int(chain.token[0]), "token_1gpu": int(one.token[0]),
               "logits_differing": int((a != b).sum())}
        one.release()
        del one
        torch.cuda.synchronize()
    barrier(world)
    return res


# ------------------------------------------------------------------------------ Phi-4-mini sweep
def phi4_sweep(args, world, rank, group, hbm):
    """the Phi-4-mini-shaped quantized linears (one layer's q 3072x3072,
    k / v 1024x3072, o 3072x3072, gate / up 8192x3072, down 3072x8192, and the 200064x3072 LM
    head) in int8-row and int4-g32 (head int8-row), batches of 1 / 8 / 64 activation rows
    N(0, 1), each projection's output rows sharded over the ranks with an NCCL all-gather of its
    output (in the timed graph) when world > 1. One CUDA graph replays the eight launches (and
    gathers); value = weight bytes (whole job) / time. Weights are random int8 rows / nibbles (the
    GEMV's cost does not depend on their values), the same on every rank for its shard."""
    import torch
    import torch.distributed as dist
    from opentpu_b200 import linear
    shape = WL.PHI4_MINI
    projs = shape.projections() + [("head", shape.vocab, shape.hidden)]
    gen = torch.Generator(device="cuda").manual_seed(77)
    out = []
    gemv_roof = None
    stream = torch.cuda.Stream()
    for fmt in ("int8-row", "int4-g32"):
        ws, nbytes = [], 0
        for name, N, K in projs:
            f = "int8-row" if name == "head" else fmt
            n = N // world
            if f == "int8-row":
                rows = torch.randint(-127, 128, (n, K), dtype=torch.int8, device="cuda",
                                     generator=gen).view(torch.uint8)
                sw = (torch.rand(n, device="cuda", generator=gen) * 1e-3 + 1e-4)
                w = linear.PackedWeight(f, n, K, rows, sw.view(torch.uint8).reshape(n, 4))
            else:
                codes = torch.randint(0, 256, (n, K // 2), dtype=torch.int32, device="cuda",
                                      generator=gen).to(torch.uint8)
                sc = (torch.rand((n, K // 32), device="cuda", generator=gen) * 1e-3 + 1e-4).half()
                w = linear.PackedWeight(f, n, K, codes, sc)
            ws.append(w)
            nbytes += w.stream_bytes * world
        for B, tc in ((1, False), (8, False), (8, True), (64, False), (64, True)):
            xs = {K: torch.randn((B, K), device="cuda", generator=gen) for _, _, K in projs}
            ys = [torch.empty((B, w.N), device="cuda") for w in ws]
            gath = [torch.empty((world, B, w.N), device="cuda") for w in ws] if world > 1 else None
            planes = {K: linear.QActPlanes(B, K) for _, _, K in projs} if tc else None

            def run():
                for i, ((_, N, K), w) in enumerate(zip(projs, ws)):
                    if tc and w.fmt == "int8-row":   # QACT + the exact MM on tcgen05
                        linear.qlinear_tc(xs[K], w, out=ys[i], planes=planes[K])
                    else:
                        linear.qlinear(xs[K], w, out=ys[i], pdl=True)
                    if world > 1:
                        dist.all_gather_into_tensor(gath[i], ys[i], group=group)
            g = capture(run, stream, warm=1)
            graph_ms(g, stream, 2, world)
            ms = graph_ms(g, stream, max(5, min(args.steps, 20)), world)
            del g
            out.append({"format": fmt, "batch": B, "ms": ms,
                        "int8_path": "tcgen05 kind::i8 (otq_qmm_tc)" if tc else "cuda-core GEMV",
                        "launches": sum(2 if tc and w.fmt == "int8-row" else 1 for w in ws),
                        "GB/s": nbytes / (ms * 1e-3) / 1e9,
                        "hbm_frac_per_gpu": nbytes / world / (ms * 1e-3) / 1e9 / hbm,
                        "weights_bytes": nbytes})
        if fmt == "int8-row":
            # the 614 MB head alone at batch 1: the GEMV's streaming rate on a large matrix
            head = ws[-1]
            hx = torch.randn((1, head.K), device="cuda", generator=gen)
            hy = torch.empty((1, head.N), device="cuda")
            g = capture(lambda: [linear.qlinear(hx, head, out=hy, pdl=True) for _ in range(10)],
                        stream, warm=1)
            graph_ms(g, stream, 1, world)
            hms = graph_ms(g, stream, 5, world) / 10
            del g
            hb = head.stream_bytes + 4 * head.K + 4 * head.N
            gemv_roof = {"bound": "hbm", "achieved": hb / (hms * 1e-3) / 1e9, "peak": hbm,
                         "unit": "GB/s", "frac": hb / (hms * 1e-3) / 1e9 / hbm,
                         "kernel": f"gemv_kernel ({head.N}x{head.K} int8-row head, M=1, this "
                                   "rank's rows; 10 launches in a graph)",
                         "bytes_per_launch": hb, "us_per_launch": hms * 1e3}
        del ws
        torch.cuda.synchronize()
    return {"metric": "quantized linear GB/s (Phi-4-mini shapes)", "unit": "GB/s",
            "gemv_roofline": gemv_roof,
            "value": max(r["GB/s"] for r in out), "results": out,
            "config": {"workload": "BASELINE configuration 5: Phi-4-mini projections q 3072x3072, "
                                   "k/v 1024x3072, o 3072x3072, gate/up 8192x3072, down 3072x8192 "
                                   "+ head 200064x3072; int8-row and int4-g32 layers (int8-row "
                                   "head); batch 1/8/64; one CUDA graph of the 8 launches",
                       "parallelism": f"row-shard x{world}" + (" + NCCL all-gather of every "
                                                              "output" if world > 1 else "")},
            "gpu_launches": sum(r["launches"] for r in out)}


# ------------------------------------------------------------------------------ prefill
def decoder_bench(args, hbm, peak_kind, fmt="int8-row"):
    """BASELINE configurations 2 (fmt int8-row) and 3 (int4-g32 layers, int8-row head) as the
    model runs them: the Qwen3-0.6B-shaped decoder with random-init N(0, 0.02) weights
    quantized, a seeded random 512-token prompt
    through the decoder's prefill, then fused decode steps -- one launch a token doing both
    norms, QKV, q/k norms and RoPE, attention over the KV cache, O, the SwiGLU MLP, the LM head
    and the greedy token, fed to the next step on the device. Timed: a CUDA graph of one step
    replayed (each replay decodes the next position). e2e: steps launched from the host, each
    step's token written from pinned host memory and read back (generate()'s loop)."""
    import torch
    from opentpu_b200.model import FusedDecoder, Qwen3Decoder
    shape = WL.QWEN3_0_6B
    n_e2e = 32
    prompt_len = 512
    max_pos = prompt_len + args.warmup + args.steps + n_e2e + 8
    W = WL.decoder_weights(shape, seed=0)
    dec = Qwen3Decoder(shape, W, fmt=fmt, head_fmt="int8-row", max_pos=max_pos, down_chunk=None)
    del W
    fd = FusedDecoder(dec)
    prompt = np.random.default_rng(1).integers(0, shape.vocab, prompt_len).tolist()
    first = int(torch.argmax(dec.prefill(prompt)).item())
    fd.start(first, prompt_len)
    fd.capture()
    with torch.cuda.stream(fd.stream):
        for _ in range(args.warmup):
            fd.graph.replay()
    torch.cuda.synchronize()
    pos0 = int(fd.pos[0].item())
    ms = graph_ms(fd.graph, fd.stream, args.steps, 1)
    # bytes a step: every packed weight (int8 rows + fp32 row scales) and the KV cache read by
    # the attention (both caches, every layer, at the timed region's mean position)
    def packed(w):   # int8 rows + an fp32 scale a row, or nibbles + an fp16 scale a group
        return w.N * w.K // 2 + w.N * (w.K // 32) * 2 if w.fmt == "int4-g32" else w.N * w.K + 4 * w.N
    wbytes = sum(packed(L[k]) for L in dec.layers for k in ("qkv", "o", "gateup", "down"))
    wbytes += packed(dec.head)
    mean_pos = pos0 + args.steps / 2
    kv = 2 * shape.layers * mean_pos * shape.n_kv * shape.head_dim * 4
    tok_host = torch.zeros(1, dtype=torch.int64).pin_memory()
    tok = int(fd.token[0].item())
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        tok_host[0] = tok
        fd.token[0:1].copy_(tok_host, non_blocking=True)
        fd.launch()
        tok_host.copy_(fd.token[0:1], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        tok = int(tok_host[0])
    e2e_ms = (time.perf_counter() - t0) / n_e2e * 1e3
    ach = (wbytes + kv) / (ms * 1e-3) / 1e9
    out = {
        "workload": f"Qwen3-0.6B-shaped decoder, layers {fmt}, int8-row head (28 layers, hidden "
                    "1024, 16/8 heads of 128, SwiGLU 3072, vocab 151936, random N(0, 0.02) "
                    "weights): 512-token seeded prompt, then fused greedy steps",
        "tok_s": 1e3 / ms, "ms_per_token": ms, "weight_gb_s": wbytes / (ms * 1e-3) / 1e9,
        "weights_bytes_per_token": wbytes, "positions": [pos0, pos0 + args.steps],
        "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                     "frac": ach / hbm,
                     "traffic": read_traffic("step_kernel_qwen3_0_6b_decoder_int8row_pos512.md", 1)
                     if fmt == "int8-row" else None,
                     "traffic_note": "ncu capture of one step at position 513 (KV cache 117 MB)",
                     "kernel": "step_kernel (the whole decoder step, 141 stages, one launch)",
                     "bytes_per_launch": wbytes + kv, "us_per_launch": ms * 1e3,
                     "peak_kind": f"{peak_kind} (copy)"},
        "e2e": {"ms_per_token": e2e_ms, "tok_s": 1e3 / e2e_ms,
                "value": wbytes / (e2e_ms * 1e-3) / 1e9, "unit": UNIT,
                "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8,
                "api": "FusedDecoder.launch with the token written from and read to pinned host "
                       "memory every step"},
        "gpu_launches": args.steps + n_e2e,
    }
    fd.graph = None
    del fd, dec
    torch.cuda.empty_cache()
    return out


def prefill_layer(shape, world, rank, gen, xs=None):
    """One layer's seven projections for the prefill GEMM: int8-row
    weights (uniform int8 rows, Sw ~ 1e-3: the GEMM's cost does not depend on the values),
    drawn whole from a generator every rank seeds alike and cut to this rank's row shard, bf16
    activations N(0, 1) [512, K] (shared across layers when xs is given) and fp32 outputs.
    Returns (gemm_w8a16_group items, the full weights' (rows, Sw) for a parity check)."""
    import torch
    from opentpu_b200 import linear
    items, full = [], []
    for i, (_, N, K) in enumerate(shape.projections()):
        n = N // world
        rows = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda",
                             generator=gen).view(torch.uint8)
        sw = torch.rand(N, device="cuda", generator=gen) * 1e-3 + 1e-4
        mine_r = rows[rank * n:(rank + 1) * n].clone()
        mine_s = sw[rank * n:(rank + 1) * n].clone()
        w = linear.PackedWeight("int8-row", n, K, mine_r, mine_s.view(torch.uint8).reshape(n, 4))
        x = xs[i] if xs is not None else torch.randn((PREFILL_TOKENS, K), device="cuda",
                                                      generator=gen).to(torch.bfloat16)
        y = torch.empty((PREFILL_TOKENS, n), device="cuda")
        items.append((x, w, y, False))
        full.append((rows, sw))
    return items, full


def prefill_bench(args, world, rank, local, group, steps, warmup):
    """BASELINE configuration 4 on this rank: 36 SmolLM3-3B layers, each one grouped launch of
    its seven projections (row shard 1/world of each), one CUDA graph a step. With world > 1 the
    seven projections write column ranges of one fp32 buffer a layer, which is rounded to bf16
    (the next layer's activation type) and all-gathered by one NCCL call a layer, in the same
    graph."""
    import torch
    import torch.distributed as dist
    from opentpu_b200 import linear
    shape = WL.SMOLLM3_3B
    gen = torch.Generator(device="cuda").manual_seed(1234)
    first, full0 = prefill_layer(shape, world, rank, gen)
    xs = [it[0] for it in first]
    layers = [first] + [prefill_layer(shape, world, rank, gen, xs)[0]
                        for _ in range(shape.layers - 1)]
    flops_layer = sum(2.0 * PREFILL_TOKENS * it[1].N * it[1].K for it in first)
    gathered = ybf = None
    if world > 1:
        # one fp32 output buffer a layer, the projections in column ranges of it
        ntot = sum(it[1].N for it in first)
        ybufs = []
        for li, items in enumerate(layers):
            Y = torch.empty((PREFILL_TOKENS, ntot), device="cuda")
            c0, new = 0, []
            for x, w, _, acc in items:
                new.append((x, w, Y[:, c0:c0 + w.N], acc))
                c0 += w.N
            layers[li] = new
            ybufs.append(Y)
        ybf = [torch.empty((PREFILL_TOKENS, ntot), dtype=torch.bfloat16, device="cuda")
               for _ in layers]
        gathered = [torch.empty((world, PREFILL_TOKENS, ntot), dtype=torch.bfloat16,
                                device="cuda") for _ in layers]

    def layer(li):
        linear.gemm_w8a16_group(layers[li])
        if world > 1:
            ybf[li].copy_(ybufs[li])
            dist.all_gather_into_tensor(gathered[li], ybf[li], group=group)

    def step():
        for li in range(shape.layers):
            layer(li)
    stream = torch.cuda.Stream()
    g = capture(step, stream, warm=1)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            g.replay()
    torch.cuda.synchronize()
    ms = graph_ms(g, stream, steps, world)
    # the GEMM launches alone (no all-gather): the kernel's roofline
    gk = capture(lambda: [linear.gemm_w8a16_group(items) for items in layers], stream, warm=1)
    graph_ms(gk, stream, 1, world)
    kms = graph_ms(gk, stream, steps, world)
    del gk
    total_flops = flops_layer * world * shape.layers
    tflops = total_flops / (ms * 1e-3) / 1e12
    launch_us = kms * 1e3 / shape.layers
    achieved = flops_layer / (launch_us * 1e-6) / 1e12
    _, bf16_peak, peak_kind = peaks()
    traffic = read_traffic("w8a16_kernel_smollm3_layer_m512.md", world)

    # end to end from host buffers: the seven activation matrices H2D (pinned bf16), the step,
    # the last layer's outputs D2H (pinned fp32), waited for on the host
    hx = [x.cpu().pin_memory() for x in xs]
    last = [gathered[-1]] if world > 1 else [it[2] for it in layers[-1]]
    hy = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in last]
    h2d = sum(t.numel() * t.element_size() for t in hx)
    d2h = sum(t.numel() * t.element_size() for t in hy)

    def e2e_step():
        with torch.cuda.stream(stream):
            for d, h in zip(xs, hx):
                d.copy_(h, non_blocking=True)
            g.replay()
            for h, d in zip(hy, last):
                h.copy_(d, non_blocking=True)
        stream.synchronize()
    e2e_step()
    barrier(world)
    ne = max(3, min(steps, 20))
    t0 = time.perf_counter()
    for _ in range(ne):
        e2e_step()
    e2e_ms = max_over_ranks((time.perf_counter() - t0) / ne * 1e3, world)

    parity = None
    if world > 1:
        # layer 0 unsharded on rank 0 against the gathered sharded outputs (fp32 sums in
        # different orders: within 2^-18 of |x| @ |deq|^T elementwise)
        torch.cuda.synchronize()
        g32 = torch.empty((world,) + tuple(ybufs[0].shape), device="cuda")
        dist.all_gather_into_tensor(g32, ybufs[0], group=group)   # layer 0's fp32 outputs
        torch.cuda.synchronize()
        if rank == 0:
            worst = 0.0
            c0 = 0
            for (x, w, y, _), (rows, sw) in zip(layers[0], full0):
                gth = g32[:, :, c0:c0 + w.N]
                c0 += w.N
                wf = linear.PackedWeight("int8-row", rows.shape[0], w.K, rows,
                                         sw.view(torch.uint8).reshape(-1, 4))
                ref = linear.gemm_w8a16(x, wf)
                got = gth.permute(1, 0, 2).reshape(PREFILL_TOKENS, -1)
                deq = rows.view(torch.int8).float().abs() * sw[:, None]
                bound = x.float().abs() @ deq.t()
                worst = max(worst, float(((got - ref).abs() / (bound + 1e-30)).max()))
            parity = {"vs_1gpu": "within tolerance" if worst <= 2.0 ** -18 else "differs",
                      "max_err_over_bound": worst, "tolerance": 2.0 ** -18, "layer": 0}
        barrier(world)
    del g
    torch.cuda.synchronize()
    w8a8 = None
    if world == 1 and not args.no_w8a8:
        w8a8 = prefill_w8a8_bench(steps, warmup, layers)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, desc, threads = prefill_cpu_sample()
        cpu = {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": desc}
    return {
        "metric": "prefill TFLOP/s", "value": tflops, "unit": "TFLOP/s", "ms_per_step": ms,
        "steps": steps, "warmup": warmup, "scaling": "strong", "dtype": "bf16 x int8 -> fp32",
        "config": {"workload": "SmolLM3-3B-shaped prefill GEMMs: 36 layers x (q 2048x2048, k/v "
                               "512x2048, o 2048x2048, gate/up 11008x2048, down 2048x11008) "
                               "int8 per-row weights, 512 tokens bf16 N(0,1)",
                   "flops_per_step": total_flops, "launch": "one grouped launch a layer "
                   "(7 projections), 36 in one CUDA graph",
                   "parallelism": f"row-shard x{world}" + (" + one NCCL all-gather a layer of "
                                                          "its seven outputs rounded to bf16 "
                                                          "(in the timed graph)"
                                                          if world > 1 else ""),
                   "l2": "weights 2.8 GB > 126 MB L2 (no flush needed)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": bf16_peak,
                     "unit": "TFLOP/s", "frac": achieved / bf16_peak, "traffic": traffic,
                     "kernel": "w8a16_kernel (one SmolLM3-3B layer, 7 projections, M=512)",
                     "flops_per_launch": flops_layer, "us_per_launch": launch_us,
                     "peak_kind": f"{peak_kind} bf16 (burst)"},
        "e2e": {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "gemm_w8a16_group graph from pinned host bf16 X to host fp32 y of the "
                       "last layer"},
        "parity": parity,
        "cpu_baseline": cpu,
        "gpu_launches": shape.layers * steps,
        "w8a8": w8a8,
    }


def prefill_w8a8_bench(steps, warmup, layers_in=None):
    """The exact prefill of BASELINE configuration 4's shapes (one GPU): the reference's own
    prefill numerics, QACT of fp32 activations and the exact integer MM (otq_qact_planes +
    otq_gemm_w8a8_group on tcgen05 kind::i8), bit-identical to the reference's MM. A layer is
    four QACT launches (the inputs of q / k / v, of o, of gate / up, of down: the layer's data
    flow) and one grouped MM launch of its seven projections; 36 layers in one CUDA graph.
    Activations are bf16 N(0, 1) values widened to fp32."""
    import torch
    from opentpu_b200 import linear
    shape = WL.SMOLLM3_3B
    gen = torch.Generator(device="cuda").manual_seed(4321)
    projs = shape.projections()          # q, k, v, o, gate, up, down
    src = [0, 0, 0, 1, 2, 2, 3]          # which of the layer's four inputs each reads
    Ks = [projs[0][2], projs[3][2], projs[4][2], projs[6][2]]
    xs = [torch.randn((PREFILL_TOKENS, K), device="cuda", generator=gen)
          .to(torch.bfloat16).float() for K in Ks]
    planes = [linear.QActPlanes(PREFILL_TOKENS, K) for K in Ks]
    if layers_in is None:
        layers_in = [prefill_layer(shape, 1, 0, gen)[0] for _ in range(shape.layers)]
    layers = [[(planes[src[i]], it[1], it[2], False) for i, it in enumerate(items)]
              for items in layers_in]
    flops_layer = sum(2.0 * PREFILL_TOKENS * it[1].N * it[1].K for it in layers_in[0])

    def fill():
        for x, p in zip(xs, planes):
            p.fill(x)

    def step():
        for items in layers:
            fill()
            linear.gemm_w8a8_group(items)
    stream = torch.cuda.Stream()
    g = capture(step, stream, warm=1)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            g.replay()
    ms = graph_ms(g, stream, steps, 1)
    gk = capture(lambda: [linear.gemm_w8a8_group(items) for items in layers], stream, warm=1)
    graph_ms(gk, stream, 1, 1)
    kms = graph_ms(gk, stream, steps, 1)
    del g, gk
    # parity: every projection of layer 0 against the CUDA-core MM (otq_qmm), bit for bit
    outs = [torch.empty_like(it[2]) for it in layers[0]]
    with torch.cuda.stream(stream):
        fill()
        linear.gemm_w8a8_group([(p, w, y, a) for (p, w, _, a), y in zip(layers[0], outs)])
    stream.synchronize()
    differ = 0
    for i, ((_, w, _, _), y) in enumerate(zip(layers[0], outs)):
        ref = linear.qlinear(xs[src[i]], w)
        differ += int((ref.view(torch.int32) != y.view(torch.int32)).sum().item())
    counts = []
    for p in planes:
        Mp = -(-PREFILL_TOKENS // 128) * 128
        counts += p.buf[8 * Mp: 8 * Mp + PREFILL_TOKENS].tolist()
    _, bf16_peak, peak_kind = peaks()
    launch_us = kms * 1e3 / shape.layers
    achieved = flops_layer / (launch_us * 1e-6) / 1e12
    total = flops_layer * shape.layers
    return {
        "metric": "prefill TOP/s (exact W8A8)", "value": total / (ms * 1e-3) / 1e12,
        "unit": "TOP/s", "ms_per_step": ms, "steps": steps,
        "dtype": "int8 x int8 -> int64 exact, fp32 epilogue",
        "config": {"workload": "SmolLM3-3B-shaped prefill, 36 layers x 7 projections, 512 "
                               "tokens, QACT of fp32 activations (bf16 N(0,1) values) + exact "
                               "MM; the reference's prefill numerics",
                   "launch": "4 QACT launches + one grouped MM launch a layer, 36 layers in "
                             "one CUDA graph"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": 2 * bf16_peak,
                     "unit": "TOP/s", "frac": achieved / (2 * bf16_peak), "traffic": None,
                     "kernel": "w8a8_kernel (one layer's 7 projections, M=512)",
                     "us_per_launch": launch_us, "ops_per_launch": flops_layer,
                     "peak_kind": f"2 x {peak_kind} bf16 burst (int8 dense is twice bf16)",
                     "planes_per_row": {str(k): counts.count(k) for k in (1, 2, 3)},
                     "note": "a row with offsets 1..8 runs two int8 planes (exactness), so "
                             "tensor work is planes x the algorithmic ops"},
        "parity": {"vs_cuda_core_mm": "bit-identical" if differ == 0 else "differs",
                   "outputs_differing": differ, "layer": 0},
        "gpu_launches": 5 * shape.layers * steps,
    }


# ------------------------------------------------------------------------------ profile runs
def profile_run(what: str):
    """A few launches for an ncu capture: the LM head GEMV alone, two decode steps, three
    grouped prefill launches of one SmolLM3-3B layer, five int4-g32 GEMVs of one activation
    row over a 65536 x 4096 matrix (144 MB of codes and scales, more than L2), three one-launch
    decode steps (int8-row or int4-g32 layers), or three fused decoder steps at position 512."""
    import torch
    from opentpu_b200 import linear
    from opentpu_b200.decode import DecodeChain
    torch.cuda.set_device(0)
    shape = WL.QWEN3_0_6B
    if what == "head":
        W = torch.randn((shape.vocab, shape.hidden), device="cuda") * 0.02
        w = linear.PackedWeight.from_float(W, "int8-row")
        del W
        x = torch.randn((1, shape.hidden), device="cuda")
        y = torch.empty((1, shape.vocab), device="cuda")
        for _ in range(5):
            linear.qlinear(x, w, out=y)
    elif what == "g32":
        W = torch.randn((65536, 4096), device="cuda") * 0.02
        w = linear.PackedWeight.from_float(W, "int4-g32")
        del W
        x = torch.randn((1, 4096), device="cuda")
        y = torch.empty((1, 65536), device="cuda")
        for _ in range(5):
            linear.qlinear(x, w, out=y)
    elif what in ("stepkernel", "stepkernel4"):
        from opentpu_b200.decode import DecodeStep
        st = DecodeStep(shape, fmt="int4-g32" if what == "stepkernel4" else "int8-row")
        for _ in range(3):
            st.step_eager()
    elif what == "decoderkernel":
        from opentpu_b200.model import FusedDecoder, Qwen3Decoder
        W = WL.decoder_weights(shape, seed=0)
        dec = Qwen3Decoder(shape, W, fmt="int8-row", max_pos=640, down_chunk=None)
        del W
        fd = FusedDecoder(dec)
        prompt = np.random.default_rng(1).integers(0, shape.vocab, 512).tolist()
        fd.start(int(torch.argmax(dec.prefill(prompt)).item()), 512)
        for _ in range(3):
            fd.launch()
    elif what == "prefill":
        items, _ = prefill_layer(WL.SMOLLM3_3B, 1, 0,
                                 torch.Generator(device="cuda").manual_seed(0))
        for _ in range(3):
            linear.gemm_w8a16_group(items)
    elif what == "w8a8":
        items, _ = prefill_layer(WL.SMOLLM3_3B, 1, 0,
                                 torch.Generator(device="cuda").manual_seed(0))
        planes = {}
        for x, w, _, _ in items:
            if w.K not in planes:
                planes[w.K] = linear.QActPlanes(PREFILL_TOKENS, w.K).fill(x.float())
        group = [(planes[w.K], w, y, False) for _, w, y, _ in items]
        for _ in range(3):
            linear.gemm_w8a8_group(group)
    elif what == "phi4tc":
        shape = WL.PHI4_MINI
        W = torch.randint(-127, 128, (shape.vocab, shape.hidden), dtype=torch.int8,
                          device="cuda").view(torch.uint8)
        sw = torch.rand(shape.vocab, device="cuda") * 1e-3 + 1e-4
        w = linear.PackedWeight("int8-row", shape.vocab, shape.hidden, W,
                                sw.view(torch.uint8).reshape(-1, 4))
        x = torch.randn((64, shape.hidden), device="cuda")
        y = torch.empty((64, shape.vocab), device="cuda")
        planes = linear.QActPlanes(64, shape.hidden)
        for _ in range(3):
            linear.qlinear_tc(x, w, out=y, planes=planes)
    else:
        chain = DecodeChain(shape)
        chain.capture()
        chain.replay(2)
        chain.release()
    torch.cuda.synchronize()


# ------------------------------------------------------------------------------ arms
def run_reference(args, rank, world):
    """The reference's CPU algorithm for the decode GEMV (the exact QACT + MM of the oracle
    port) on every host core, on rank 0 only; the other ranks exit without work."""
    if rank != 0:
        return
    vals = []
    desc, threads = "", 1
    for i in range(args.warmup + args.steps):
        v, desc, threads = cpu_exact_sample(budget_s=6.0 if i >= args.warmup else 1.0)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": "Qwen3-0.6B-shaped int8 per-row decode GEMV chain (sample)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", choices=["head", "step", "prefill", "w8a8", "phi4tc", "g32",
                                          "stepkernel",
                                          "stepkernel4", "decoderkernel"])
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-w8a8", action="store_true")
    ap.add_argument("--no-4bit", action="store_true")
    ap.add_argument("--no-config1", action="store_true")
    ap.add_argument("--no-phi4", action="store_true")
    ap.add_argument("--no-decoder", action="store_true")
    ap.add_argument("--shard", choices=["head", "all"], default="head",
                    help="with more than one GPU: shard only the LM head (every rank computes the "
                         "layers whole) or every projection")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.profile:
        profile_run(args.profile)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    from opentpu_b200.decode import DecodeStep

    torch.cuda.set_device(local)
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    hbm, _, peak_kind = peaks()
    shape = WL.QWEN3_0_6B
    fmt = "int8-row"
    chain = DecodeStep(shape, fmt=fmt, head_fmt=fmt, world=world, rank=rank, group=group,
                       shard=args.shard)
    chain.capture()
    total_bytes = chain.weight_bytes
    chain.replay(args.warmup)
    torch.cuda.synchronize()

    with Clocks(local) as clocks:
        ms = graph_ms(chain.graph, chain.stream, args.steps, world)
        value = total_bytes / (ms * 1e-3) / 1e9
        # (before the closed loop, which replaces the step's seeded input)
        parity = parity_vs_one_gpu(chain, world, rank) if world > 1 else None
        e2e_ms, h2d, d2h, _ = closed_loop(chain, max(10, min(args.steps, 200)), world)
        # the dominant (only) kernel: the step's one launch; its bytes are this rank's weights
        # and scales plus every projection's input row and output words
        per_rank = chain.rank_bytes + sum(4 * K + 8 * N for _, N, K, _ in chain.plan)
        ach = per_rank / (ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                "frac": ach / hbm,
                "traffic": read_traffic("step_kernel_qwen3_0_6b_int8row.md", world),
                "kernel": "step_kernel (the whole decode step, 113 projections + greedy token, "
                          "one persistent launch" + (f", this rank's rows ({args.shard} sharded)"
                                                     if world > 1 else "") + ")",
                "bytes_per_launch": per_rank, "us_per_launch": ms * 1e3,
                "peak_kind": f"{peak_kind} (copy)"}
        head = None
        decoder = decoder4 = None
        if not args.no_decoder and world == 1:
            decoder = decoder_bench(args, hbm, peak_kind, "int8-row")
            decoder4 = decoder_bench(args, hbm, peak_kind, "int4-g32")
        c1 = None if args.no_config1 else config1(world, max(3, min(args.steps, 50)))
        dec4 = None if args.no_4bit else decode_4bit(args, world, rank, group, hbm, peak_kind)
        phi4 = None if args.no_phi4 else phi4_sweep(args, world, rank, group, hbm)
        prefill = None if args.no_prefill else prefill_bench(
            args, world, rank, local, group, max(3, min(100, args.steps // 4)),
            max(3, min(5, args.warmup)))

    cpu = blas = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, desc, threads = cpu_exact_sample()
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": desc}
        v, desc, threads = cpu_blas_sample("int8-row")
        blas = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": desc}

    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic",
            "config": {"workload": "Qwen3-0.6B-shaped int8 per-row decode step: 28 layers x "
                                   "(QKV, O, GateUp, Down) + 151936x1024 LM head + greedy "
                                   "token, M=1",
                       "weights_bytes_per_step": total_bytes, "format": fmt,
                       "parallelism": (f"row-shard x{world} of " + ("the LM head (every rank "
                                       "computes the layers' projections whole)" if args.shard
                                       == "head" else "every projection") + ", the sharded "
                                       "outputs' words stored to every rank over NVLink inside "
                                       "the step kernel") if world > 1 else "one GPU",
                       "l2": "weights 598 MB > 126 MB L2 (no flush needed)",
                       "launch": "one persistent launch a step (otq_decode_step), replayed "
                                 "from a CUDA graph"},
            "tok_s": 1e3 / ms,
            "hbm_frac": value / world / hbm,
            "roofline": roof,
            "roofline_head": head,
            "cpu_baseline": cpu,
            "cpu_baseline_blas": blas,
            "e2e": {"value": total_bytes / (e2e_ms * 1e-3) / 1e9, "unit": UNIT,
                    "ms_per_token": e2e_ms, "tok_s": 1e3 / e2e_ms,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "DecodeChain.run_host, closed loop (each input picked by the "
                           "previous token, read on the host)"},
            "parity": parity,
            "gpu_launches": chain.launches * args.steps,
            "clocks": clocks.summary(),
            "decoder": decoder,
            "decoder_4bit": decoder4,
            "config1": c1,
            "decode_4bit": dec4,
            "prefill": prefill,
            "phi4_sweep": phi4,
        }), flush=True)
    chain.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
