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
