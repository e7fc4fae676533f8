"""The stream-K schedule of the GEMM: tiles split between SMs are finished exactly.

When whole tiles would leave a ragged last wave, w8_mm_i8_ws cuts the (tile, K-block)
work into equal ranges and sums split tiles with TMA reduce-adds, synchronised by
per-tile counters in the workspace.  The int32 result must be bit-identical to the
plain schedule (w8_mm_i8) and to torch._int_mm, on every launch and on every replay
of a captured graph, and the workspace must be all-zero again after each call.
"""
import pytest
import torch

import gemma_npu_b200 as w8
from gemma_npu_b200 import _lib, kernels

pytestmark = pytest.mark.gpu

# (M, N, K): pair-kernel shapes with ragged waves (o, down, qkv of config 1; short
# prompts) and single-kernel shapes with only a few tiles (M <= 128).
SHAPES = [(3658, 1536, 2048), (3658, 1536, 6144), (3658, 2560, 1536), (207, 1536, 6144),
          (858, 2560, 1536), (300, 512, 4096), (64, 1536, 256), (64, 256, 1536), (100, 1536, 6144),
          (16, 2560, 1536), (1, 2560, 1536), (129, 384, 2048),
          (600, 1536, 3200)]  # K / 128 = 25: the last 256-byte K stage of a CTA pair is half empty


def plain(a, w):
    c = torch.empty((a.shape[0], w.shape[0]), dtype=torch.int32, device=a.device)
    _lib.call("w8_mm_i8", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), _lib.W8_B_NK, c.data_ptr(),
              c.stride(0), a.shape[0], w.shape[0], a.shape[1], torch.cuda.current_stream().cuda_stream or None)
    return c


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_stream_k_bit_exact_and_workspace_reset(cuda, m, n, k):
    gen = torch.Generator(device=cuda).manual_seed(m * 7 + n + k)
    a = torch.randint(-128, 128, (m, k), dtype=torch.int8, device=cuda, generator=gen)
    w = torch.randint(-128, 128, (n, k), dtype=torch.int8, device=cuda, generator=gen)
    want = plain(a, w)
    if m > 16 and n % 8 == 0:
        assert torch.equal(want, torch._int_mm(a, w.t().contiguous()))
    ws = torch.zeros(_lib.lib().w8_mm_i8_workspace_bytes(m, n, k) // 4 + 7, dtype=torch.int32, device=cuda)
    c = torch.empty_like(want)
    stream = torch.cuda.current_stream().cuda_stream or None
    for _ in range(10):
        c.fill_(-1)
        _lib.call("w8_mm_i8_ws", a.data_ptr(), k, w.data_ptr(), k, _lib.W8_B_NK, c.data_ptr(), n, m, n, k,
                  ws.data_ptr(), ws.numel() * 4, stream)
        assert torch.equal(c, want)
        assert int(ws.abs().sum()) == 0
    # the reference's [K, N] layout takes the same schedule
    c2 = torch.empty_like(want)
    w8.mm_i8(a, w.t().contiguous(), c2)
    assert torch.equal(c2, want)


def test_stream_k_graph_replays(cuda):
    m, n, k = 3658, 1536, 6144
    gen = torch.Generator(device=cuda).manual_seed(3)
    a = torch.randint(-128, 128, (m, k), dtype=torch.int8, device=cuda, generator=gen)
    w = torch.randint(-128, 128, (n, k), dtype=torch.int8, device=cuda, generator=gen)
    want = plain(a, w)
    c = torch.empty_like(want)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        w8.mm_i8_nk(a, w, c)  # eager first: sets kernel attributes, allocates the workspace
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        w8.mm_i8_nk(a, w, c)
    for i in range(8):
        c.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(c, want), f"replay {i}"
    for ws in kernels._WORKSPACES.values():
        assert int(ws.abs().sum()) == 0
    assert w8.device_status() == 0
