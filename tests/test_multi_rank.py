"""The multi-GPU path's host logic on CPU ranks (gloo, world size 2): row shards of each
projection (runtime.Weight(shard=0), runtime.py:138-142), the exact MM on each shard, and the
all-gather that assembles the output (the reference's GATHER, isasim.py:1413-1438). QACT runs
on the whole replicated x on every rank, so the gathered outputs are bit-identical to the
unsharded MM for every world size; a rank that fails is seen by the others as an error, not a
hang."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import fp32 as F
from oracle import mx as X
from opentpu_b200.decode import shard_rows


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))


def _sharded_mm(rank, world, port, fmt, out):
    _init(rank, world, port)
    try:
        rng = np.random.default_rng(7)
        N, K = 96, 256
        W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        x = rng.standard_normal((1, K)).astype(np.float32)
        n0, n1 = shard_rows(N, world, rank)
        if fmt == "int8-row":
            rows, srows = X.quantize_rows_rsc(W[n0:n1])
            y = X.qlinear(x, rows, srows, "int8", rsc=True)
        else:
            rows, srows = X.quantize_weights(W[n0:n1], fmt)
            y = X.qlinear(x, rows, srows, fmt)
        parts = [torch.empty((1, n1 - n0), dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(y, np.float32)))
        if rank == 0:
            out.put(torch.cat(parts, 1).numpy().copy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt", ["int8-row", "int4"])
def test_row_shards_gather_to_the_unsharded_mm(fmt):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_mm, args=(r, world, port, fmt, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(7)
    W = (rng.standard_normal((96, 256)) * 0.02).astype(np.float32)
    x = rng.standard_normal((1, 256)).astype(np.float32)
    if fmt == "int8-row":
        rows, srows = X.quantize_rows_rsc(W)
        want = X.qlinear(x, rows, srows, "int8", rsc=True)
    else:
        rows, srows = X.quantize_weights(W, fmt)
        want = X.qlinear(x, rows, srows, fmt)
    assert np.array_equal(F.to_bits(got), F.to_bits(np.asarray(want, np.float32)))


def _failing_rank(rank, world, port, out):
    _init(rank, world, port)
    try:
        if rank == 1:
            raise SystemExit(3)   # leaves between steps, before the collective
        t = torch.zeros(4)
        try:
            dist.all_reduce(t)
            out.put("completed")
        except Exception as e:   # the process group's timeout ends the collective
            out.put(type(e).__name__)
    finally:
        if rank == 0:
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def test_a_rank_that_leaves_is_an_error_not_a_hang():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert res != "completed"
    assert procs[1].exitcode == 3


def test_shard_rows_rules():
    assert shard_rows(151936, 8, 7) == (132944, 151936)
    assert [shard_rows(11008, 8, r)[1] - shard_rows(11008, 8, r)[0] for r in range(8)] == [1376] * 8
    with pytest.raises(ValueError):
        shard_rows(100, 8, 0)
    with pytest.raises(ValueError):
        shard_rows(64, 2, 2)
