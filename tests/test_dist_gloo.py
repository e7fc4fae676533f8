"""Multi-rank host logic on CPU ranks (gloo, world size 2): the column-sharded LM head's
shard ranges and logit all-gather reassemble the single-rank result, the row partition of
config 4's concatenated prompts gives every row to exactly one rank with the same product,
and a rank that fails before the collective ends the others' wait with an error instead of
a hang."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import w8a8_numpy as ref

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _import_pkg():
    import importlib
    import sys

    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    return importlib.import_module("gemma-npu_b200")


def _head_worker(rank, world, port, vocab, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pkg = _import_pkg()
        from gemma_npu_b200.lm_head import gather_logits, shard_rows

        rng = np.random.default_rng(0)
        w = rng.integers(-127, 128, size=(vocab, 64), dtype=np.int8)
        s = ref.f32_to_bf16_bits(rng.uniform(0.001, 0.01, vocab).astype(np.float32))
        h = ref.f32_to_bf16_bits(rng.standard_normal(64).astype(np.float32))
        r0, r1, per = shard_rows(vocab, world, rank)
        local = torch.zeros(per, dtype=torch.float32)
        # This rank's slice, computed by the oracle (the GPU kernel's job on a B200).
        local[: r1 - r0] = torch.from_numpy(ref.int8_linear(h[None], w[r0:r1], s[r0:r1])[0].astype(np.float32))
        full = torch.empty(world * per, dtype=torch.float32)
        got = gather_logits(local, full, vocab)
        want = ref.int8_linear(h[None], w, s)[0].astype(np.float32)
        q.put((rank, bool(np.array_equal(got.numpy(), want)), pkg.__name__))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("vocab", [1024, 1001])
def test_sharded_head_gather_matches_single_rank(vocab):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_head_worker, args=(r, 2, port, vocab, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    results = sorted(q.get(timeout=5) for _ in range(2))
    assert [r[1] for r in results] == [True, True]
    assert all(p.exitcode == 0 for p in procs)


def _failing_worker(rank, world, port, q):
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "raised"))
        q.close()
        q.join_thread()  # flush before dying
        os._exit(3)  # this rank dies between steps, before its collective
    try:
        dist.all_gather_into_tensor(torch.empty(4), torch.ones(2))
        q.put((rank, "completed"))
    except Exception as e:  # noqa: BLE001 -- the failure the test expects
        q.put((rank, "error:" + type(e).__name__))
    q.close()
    q.join_thread()
    os._exit(0)


def test_dead_rank_ends_the_collective_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert all(p.exitcode is not None for p in procs), "a rank hung"
    got = dict(q.get(timeout=5) for _ in range(2))
    assert got[1] == "raised"
    assert got[0].startswith("error:")


def _rows_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _import_pkg()
        from gemma_npu_b200.gemm import partition_rows

        lengths = [300, 17, 129, 64]  # prompts of uneven length, rows concatenated
        total = sum(lengths)
        rng = np.random.default_rng(1)
        a = rng.integers(-127, 128, size=(total, 32), dtype=np.int8)
        b = rng.integers(-127, 128, size=(32, 48), dtype=np.int8)
        r0, r1 = partition_rows(total, world, rank)
        # This rank's rows through the linear (the GPU GEMM's job on a B200: the oracle here).
        mine = ref.int_mm(a[r0:r1], b)
        sizes = [None] * world
        dist.all_gather_object(sizes, (r0, r1))  # test-side reassembly only
        parts = [None] * world
        dist.all_gather_object(parts, mine)
        covered = sorted(r for lo, hi in sizes for r in range(lo, hi)) == list(range(total))
        balanced = max(hi - lo for lo, hi in sizes) - min(hi - lo for lo, hi in sizes) <= 1
        same = np.array_equal(np.concatenate(parts), ref.int_mm(a, b))
        q.put((rank, covered and balanced and same))
    finally:
        dist.destroy_process_group()


def test_row_partition_covers_rows_once_and_matches_one_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rows_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert all(ok for _, ok in res), res
    assert all(p.exitcode == 0 for p in procs)
