"""The decode GEMV chain (w8_gemv_chain): a decode step's GEMVs in one persistent launch.

Every output must be bit-identical to the standalone call of its step
(w8_int8_linear_bf16 / w8_lm_head_f32, themselves checked against the reference's
cpu_int8_linear and Int8Head + softcap in test_gemv_gpu.py), including when a step reads
the previous step's output as its activation row -- which shows the grid-wide ordering
between steps holds: a step that read its x early would see a stale or half-written row.
"""
import numpy as np
import pytest
import torch

import gemma_npu_b200 as w8
from gemma_npu_b200 import _lib
from gemma_npu_b200.kernels import argmax_token
from oracle import w8a8_numpy as ref

pytestmark = pytest.mark.gpu


def weights(n, k, gen, dev):
    wq, sw = w8.quant_rows((torch.randn(n, k, generator=gen, device=dev) * 0.02).to(torch.bfloat16))
    return wq, sw.to(torch.bfloat16)


def row(k, gen, dev):
    return torch.randn(k, generator=gen, device=dev).to(torch.bfloat16)


def bits(t):
    return t.view(torch.int16) if t.dtype == torch.bfloat16 else t.view(torch.int32)


# config 2's four layer shapes (N, K), twice, then the LM head
LAYER = [(2560, 1536), (1536, 2048), (12288, 1536), (1536, 6144)]


def test_chain_matches_standalone_calls(cuda):
    gen = torch.Generator(device=cuda).manual_seed(1)
    steps, want = [], []
    for n, k in LAYER * 2 + [(100, 16), (333, 12288), (7, 4096)]:  # + ragged: n < SMs, k = 16, max k
        wq, s = weights(n, k, gen, cuda)
        x = row(k, gen, cuda)
        y = torch.full((n,), float("nan"), dtype=torch.bfloat16, device=cuda)
        steps.append((x, wq, s, y))
        want.append(w8.int8_linear(x[None], wq, s)[0])
    hq, hs = weights(262144, 1536, gen, cuda)
    h = row(1536, gen, cuda)
    logits = torch.zeros(262144, dtype=torch.float32, device=cuda)
    best = torch.zeros(1, dtype=torch.int64, device=cuda)
    steps.append((h, hq, hs, logits, 30.0, best))
    want_logits, want_key = w8.lm_head_logits(h, hq, hs, 30.0, argmax="key")
    chain = w8.GemvChain(steps)
    for _ in range(2):  # twice: the counters are zero again after a launch
        for st in steps:
            st[3].fill_(float("nan"))
        chain()
        torch.cuda.synchronize()
        for i, (st, w_) in enumerate(zip(steps, want)):
            assert torch.equal(bits(st[3]), bits(w_)), f"step {i} {tuple(st[1].shape)}"
        assert torch.equal(logits.view(torch.int32), want_logits.view(torch.int32))
        assert int(best) == int(want_key)
    assert int(argmax_token(best)) == int(want_logits.argmax())
    assert w8.device_status() == _lib.W8_OK


def test_chain_orders_dependent_steps(cuda):
    """x of each step is the y of the step before it (shapes chained N -> K)."""
    gen = torch.Generator(device=cuda).manual_seed(2)
    shapes = [(2048, 1536), (1536, 2048), (6144, 1536), (1536, 6144), (12288, 1536), (1536, 12288),
              (2560, 1536), (1536, 2560)] * 3
    x0 = row(1536, gen, cuda)
    ws = [weights(n, k, gen, cuda) for n, k in shapes]
    ys = [torch.empty(n, dtype=torch.bfloat16, device=cuda) for n, _ in shapes]
    steps = [(x0 if i == 0 else ys[i - 1], wq, s, ys[i]) for i, (wq, s) in enumerate(ws)]
    hq, hs = weights(4096, 1536, gen, cuda)
    logits = torch.empty(4096, dtype=torch.float32, device=cuda)
    steps.append((ys[-1], hq, hs, logits, 30.0))
    # sequential standalone calls, each reading the previous output
    x, want = x0, []
    for wq, s in ws:
        x = w8.int8_linear(x[None], wq, s)[0]
        want.append(x)
    want_logits = w8.lm_head_logits(x, hq, hs, 30.0)
    chain = w8.GemvChain(steps)
    stream = torch.cuda.Stream(device=cuda)
    with torch.cuda.stream(stream):
        chain()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        chain()
    for rep in range(4):  # eager once, then graph replays
        if rep:
            for y in ys:
                y.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
        for i, (y, w_) in enumerate(zip(ys, want)):
            assert torch.equal(bits(y), bits(w_)), f"replay {rep} step {i}"
        assert torch.equal(logits.view(torch.int32), want_logits.view(torch.int32))
    del graph


def test_chain_head_against_oracle(cuda):
    gen = torch.Generator(device=cuda).manual_seed(3)
    wq, s = weights(3000, 1536, gen, cuda)
    x = row(1536, gen, cuda)
    y = torch.empty(3000, dtype=torch.float32, device=cuda)
    w8.GemvChain([(x, wq, s, y, 30.0)])()
    xb = x.cpu().view(torch.int16).numpy().view(np.uint16)[None]
    sb = s.cpu().view(torch.int16).numpy().view(np.uint16)
    exact = ref.int8_linear(xb, wq.cpu().numpy(), sb)[0].astype(np.float64)
    want = 30.0 * np.tanh(exact / 30.0)
    err = np.abs(y.cpu().numpy() - want).max() / np.abs(want).max()
    assert err <= 1e-2


def test_chain_rejects_bad_steps(cuda):
    gen = torch.Generator(device=cuda).manual_seed(4)
    wq, s = weights(64, 12304, gen, cuda)  # k beyond the chain's 12288
    x = row(12304, gen, cuda)
    y = torch.empty(64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(_lib.W8InvalidArgument):
        w8.GemvChain([(x, wq, s, y)])()
    with pytest.raises(ValueError):
        w8.GemvChain([])


def test_independent_chain_matches_standalone_calls(cuda):
    """independent=True (no waits between steps) gives the same bits on independent steps."""
    gen = torch.Generator(device=cuda).manual_seed(6)
    steps, want = [], []
    for n, k in LAYER * 3:
        wq, s = weights(n, k, gen, cuda)
        x = row(k, gen, cuda)
        y = torch.empty((n,), dtype=torch.bfloat16, device=cuda)
        steps.append((x, wq, s, y))
        want.append(w8.int8_linear(x[None], wq, s)[0])
    w8.GemvChain(steps, independent=True)()
    torch.cuda.synchronize()
    for i, (st, w_) in enumerate(zip(steps, want)):
        assert torch.equal(bits(st[3]), bits(w_)), f"step {i}"
