"""The fused NVLink all-gather of the row-sharded decode (otq_qmm_peer, DecodeChain
gather="fused") on 2 GPUs, one process a GPU: after several graph-replayed steps the outputs
equal, bit for bit, both the NCCL all-gather path and the unsharded single-GPU chain (row
shards keep every output's exact sum on one rank, and QACT runs on the whole replicated row).
Skipped on a box with fewer than 2 GPUs."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from opentpu_b200 import workloads as WL
        from opentpu_b200.decode import DecodeChain
        res = {}
        for gather in ("fused", "nccl"):
            ch = DecodeChain(WL.TINY, world=world, rank=rank, gather=gather, seed=3)
            ch.capture()
            ch.replay(5)
            torch.cuda.synchronize()
            res[gather] = [ch.full_out(i).cpu().clone() for i in range(len(ch.plan))]
            ch.release()
        if rank == 0:
            one = DecodeChain(WL.TINY, seed=3)
            one.capture()
            one.replay(5)
            torch.cuda.synchronize()
            res["single"] = [one.full_out(i).cpu().clone() for i in range(len(one.plan))]
            one.release()
            import ctypes
            from opentpu_b200 import _lib as L
            v = ctypes.c_int(0)
            L.call("otq_status_word", ctypes.addressof(v), 0)
            res["status"] = v.value
        same = all(torch.equal(a, b) for a, b in zip(res["fused"], res["nccl"]))
        q.put((rank, same, res if rank == 0 else None))
        dist.barrier()
    finally:
        dist.destroy_process_group()


CASES = [("int8-row", "all"), ("int4-g32", "all"), ("int8-row", "head"), ("int4-g32", "head")]


def _rank_step(rank, world, port, q):
    """One rank of the one-launch decode step (DecodeStep) on `world` GPUs: int8-row and 4-bit
    layers, several graph replays; rank 0 compares with the unsharded step on one GPU."""
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from opentpu_b200 import workloads as WL
        from opentpu_b200.decode import DecodeStep
        res = {}
        for fmt, shard in CASES:
            st = DecodeStep(WL.TINY, fmt=fmt, world=world, rank=rank, seed=7, shard=shard)
            st.capture()
            st.replay(4)
            torch.cuda.synchronize()
            res[(fmt, shard)] = ([st.full_out(i).cpu().clone() for i in range(len(st.plan))],
                                 int(st.token[0]))
            dist.barrier()
            st.release()
        if rank == 0:
            for fmt in ("int8-row", "int4-g32"):
                one = DecodeStep(WL.TINY, fmt=fmt, seed=7)
                one.capture()
                one.replay(4)
                torch.cuda.synchronize()
                res["one_" + fmt] = ([one.full_out(i).cpu().clone() for i in range(len(one.plan))],
                                     int(one.token[0]))
                one.release()
            import ctypes
            from opentpu_b200 import _lib as L
            v = ctypes.c_int(0)
            L.call("otq_status_word", ctypes.addressof(v), 0)
            res["status"] = v.value
        q.put((rank, res if rank == 0 else None))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_step_on_two_gpus_equals_one_gpu():
    """The one-launch decode step row-sharded over 2 GPUs, the all-gather fused into the kernel
    (tagged words stored into both ranks' copies over NVLink), or only its head sharded (every
    rank computes the layers whole): every projection's output row and the greedy token
    bit-identical to the unsharded step on one GPU (int8-row layers: exact; int4-g32 layers:
    each output row computed by one rank in the same order as on one GPU)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_step, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=600) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = [r for _, r in got if r is not None][0]
    assert res["status"] == 0
    for fmt, shard in CASES:
        outs, tok = res[(fmt, shard)]
        one, tok1 = res["one_" + fmt]
        assert tok == tok1
        for a, b in zip(outs, one):
            assert torch.equal(a.view(torch.int32), b.view(torch.int32))


def test_fused_gather_equals_nccl_and_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=600) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, same, _ in got:
        assert same, f"rank {rank}: fused gather differs from the NCCL gather"
    res = [r for _, _, r in got if r is not None][0]
    assert res["status"] == 0
    for a, b in zip(res["fused"], res["single"]):
        assert torch.equal(a, b)
