"""The column-sharded LM head over NCCL on 2 GPUs equals the single-GPU head, and its
greedy token (per-shard argmax in the GEMV + an 8-byte all-gather) is the full argmax.

One process per GPU; skipped with fewer than 2 sm_100 devices.  NCCL's in-switch
reduction (NVLS) is off, so the test uses plain NCCL rings.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import importlib
    import sys
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, ROOT)
    w8 = importlib.import_module("gemma-npu_b200")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        gen = torch.Generator(device="cuda").manual_seed(0)
        vocab = 262144 + 3  # ragged: the last shard is short
        w = (torch.randn(vocab, 1536, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
        h = torch.randn(1536, device="cuda", generator=gen).to(torch.bfloat16)
        head = w8.ShardedInt8Head(w, cap=30.0)
        got = head(h)
        full_q, full_s = w8.quant_rows(w)
        want = w8.lm_head_logits(h, full_q, full_s.to(torch.bfloat16), 30.0)
        torch.cuda.synchronize()
        greedy = int(head.greedy(h))
        ok = bool(torch.equal(got, want)) and greedy == int(want.argmax())
        q.put((rank, ok, float((got - want).abs().max())))
    finally:
        dist.destroy_process_group()


def test_sharded_head_nccl_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert all(ok for _, ok, _ in res), res
    assert all(p.exitcode == 0 for p in procs)


def _peer_worker(rank, world, port, q):
    """transport="peer": the GEMV stores the logits into every rank's buffer itself."""
    import importlib
    import sys
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, ROOT)
    w8 = importlib.import_module("gemma-npu_b200")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    head = None
    try:
        gen = torch.Generator(device="cuda").manual_seed(0)
        vocab = 262144 + 3  # ragged: the last shard is short
        w = (torch.randn(vocab, 1536, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
        hs = [torch.randn(1536, device="cuda", generator=gen).to(torch.bfloat16) for _ in range(4)]
        full_q, full_s = w8.quant_rows(w)
        full_s = full_s.to(torch.bfloat16)
        want = [w8.lm_head_logits(h, full_q, full_s, 30.0) for h in hs]
        head = w8.ShardedInt8Head(w, cap=30.0, transport="peer")
        ok = True
        for h, wl in zip(hs, want):  # eager calls, each consumed before the next
            got = head(h).clone()
            ok &= bool(torch.equal(got, wl))
            ok &= int(head.greedy(h)) == int(wl.argmax())
        # the same kernel captured in a CUDA graph: each replay is a new call (epoch)
        x = torch.empty_like(hs[0])
        x.copy_(hs[0])
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            head(x)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = head(x)
        for h, wl in zip(hs[1:], want[1:]):
            x.copy_(h)
            g.replay()
            torch.cuda.synchronize()
            ok &= bool(torch.equal(out, wl))
        del g
        ok &= w8.device_status() == 0
        q.put((rank, ok))
    finally:
        if head is not None:
            head.close()
        dist.destroy_process_group()


def _run(target, world):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    res = sorted(q.get(timeout=10) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    return res


def test_sharded_head_peer_transport_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run(_peer_worker, 2)
    assert all(ok for _, ok in res), res


def _peer_absent_worker(rank, world, port, q):
    """Rank 1 makes one call with rank 0, then does not make the second (it stays alive,
    its buffer mapped, between calls): rank 0's second call must end by itself with a
    timeout status instead of waiting for good."""
    import importlib
    import sys
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, ROOT)
    w8 = importlib.import_module("gemma-npu_b200")
    from gemma_npu_b200 import _lib

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    head = None
    try:
        gen = torch.Generator(device="cuda").manual_seed(1)
        w = (torch.randn(4096, 1536, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
        h = torch.randn(1536, device="cuda", generator=gen).to(torch.bfloat16)
        head = w8.ShardedInt8Head(w, cap=30.0, transport="peer")
        head(h)
        torch.cuda.synchronize()
        ok = w8.device_status() == 0
        dist.barrier()
        if rank == 0:
            head(h)  # rank 1 never makes this call
            try:
                w8.device_status()
                ok = False
            except _lib.W8DeviceTimeout:
                pass
        dist.barrier()  # rank 1 leaves only after rank 0's kernel has ended
        q.put((rank, ok))
    finally:
        if head is not None:
            head.close()
        dist.destroy_process_group()


def test_sharded_head_peer_rank_absent_times_out():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run(_peer_absent_worker, 2)
    assert all(ok for _, ok in res), res
