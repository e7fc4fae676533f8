"""Parity of the tcgen05 W8A8 GEMM (w8_mm_i8) with the reference's int8 GEMM.

The int32 result must be bit-exact: against the golden vectors made with the
reference's torch._int_mm call (pipeline.py:237), against the numpy oracle on
seeded inputs, and at the BASELINE shapes against torch._int_mm on the same GPU
(an independent cuBLASLt implementation) plus oracle checks on sampled rows.
Both B layouts are covered: [K,N] (the reference's mm_i8 layout) and [N,K]
(the resident layout).
"""
import numpy as np
import pytest
import torch

import gemma_npu_b200 as w8
from gemma_npu_b200 import _lib
from oracle import w8a8_numpy as ref

pytestmark = pytest.mark.gpu


def _pitch(n, mult):
    return -(-n // mult) * mult


def run_mm(a, b_kn, layout, device):
    """C = a @ b_kn through the C ABI with B given in `layout`; pitches padded to 16 B."""
    M, K = a.shape
    N = b_kn.shape[1]
    ga = torch.zeros((M, _pitch(K, 16)), dtype=torch.int8, device=device)[:, :K]
    ga.copy_(a)
    c = torch.full((M, _pitch(N, 4)), -7, dtype=torch.int32, device=device)[:, :N]
    if layout == "kn":
        gb = torch.zeros((K, _pitch(N, 16)), dtype=torch.int8, device=device)[:, :N]
        gb.copy_(b_kn)
        w8.mm_i8(ga, gb, c)
    else:
        gb = torch.zeros((N, _pitch(K, 16)), dtype=torch.int8, device=device)[:, :K]
        gb.copy_(b_kn.t())
        w8.mm_i8_nk(ga, gb, c)
    torch.cuda.synchronize()
    return c


def test_golden_int_mm(cuda, golden):
    g, w = golden("int_mm"), golden("wquant")
    a = torch.from_numpy(g["a"])
    b = torch.from_numpy(np.ascontiguousarray(w["q"].T))
    for layout in ("kn", "nk"):
        c = run_mm(a, b, layout, cuda)
        np.testing.assert_array_equal(c.cpu().numpy(), g["c"])
    full = golden("int_mm_full")
    for layout in ("kn", "nk"):
        c = run_mm(torch.from_numpy(full["a"]), torch.from_numpy(full["b"]), layout, cuda)
        np.testing.assert_array_equal(c.cpu().numpy(), full["c"])


# CTA-pair tiles (M > 128, K % 128 == 0) stage 256 K bytes at a time; K / 128 odd leaves
# half of the last stage beyond K: (300, 384, 384), (257, 200, 128), (513, 264, 640).
SMALL = [(1, 16, 16), (7, 40, 32), (128, 256, 128), (129, 257, 144), (300, 384, 1536),
         (64, 256, 1536), (64, 1536, 256), (5, 1000, 48), (255, 520, 272),
         (300, 384, 384), (257, 200, 128), (513, 264, 640)]


@pytest.mark.parametrize("layout", ["kn", "nk"])
@pytest.mark.parametrize("m,n,k", SMALL)
def test_mm_matches_oracle(cuda, m, n, k, layout):
    gen = torch.Generator().manual_seed(1000 * m + 10 * n + k)
    a = torch.randint(-128, 128, (m, k), dtype=torch.int8, generator=gen)
    b = torch.randint(-128, 128, (k, n), dtype=torch.int8, generator=gen)
    c = run_mm(a, b, layout, cuda)
    np.testing.assert_array_equal(c.cpu().numpy(), ref.int_mm(a.numpy(), b.numpy()))


# BASELINE shapes: config 0 and the config-1/3 projection set at several M.
BIG = [(512, 12288, 1536), (3658, 2560, 1536), (3658, 1536, 2048), (3658, 12288, 1536),
       (3658, 1536, 6144), (3658, 8960, 1536), (207, 1536, 6144), (858, 2560, 1536), (1878, 12288, 1536)]


# The real E2B shape mix: the double-wide MLP of KV-shared layers
# (gate/up N = 24576, down K = 12288), full-attention layers with head_dim 512 (qkv
# N = (8 + 2) * 512, o K = 8 * 512), q-only qkv of KV-shared layers (N = 8 * 256), and the
# per-layer-input gate / projection (1536 -> 256, 256 -> 1536).
E2B = [(3658, 24576, 1536), (3658, 1536, 12288), (3658, 5120, 1536), (3658, 1536, 4096), (3658, 2048, 1536),
       (3658, 256, 1536), (3658, 1536, 256)]


@pytest.mark.parametrize("m,n,k", BIG + E2B)
def test_mm_baseline_shapes_bit_exact(cuda, m, n, k):
    gen = torch.Generator(device=cuda).manual_seed(m + n + k)
    a = torch.randint(-128, 128, (m, k), dtype=torch.int8, device=cuda, generator=gen)
    w = torch.randint(-128, 128, (n, k), dtype=torch.int8, device=cuda, generator=gen)
    c = torch.empty((m, n), dtype=torch.int32, device=cuda)
    w8.mm_i8_nk(a, w, c)
    want = torch._int_mm(a, w.t().contiguous())
    assert torch.equal(c, want)
    # the reference's [K, N] layout through mm_i8 gives the same bits
    c2 = torch.empty_like(c)
    w8.mm_i8(a, w.t().contiguous(), c2)
    assert torch.equal(c2, want)
    # and the oracle agrees on a sample of rows
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(0))[:6].tolist()
    np.testing.assert_array_equal(c[rows].cpu().numpy(), ref.int_mm(a[rows].cpu().numpy(), w.t().cpu().numpy()))


def test_extreme_values_no_overflow(cuda):
    # -128 * -128 summed over K = 16384 is 2^28; mixed signs cancel exactly.
    k = 16384
    a = torch.full((130, k), -128, dtype=torch.int8, device=cuda)
    a[1::2] = 127
    w = torch.full((304, k), -128, dtype=torch.int8, device=cuda)
    w[::3] = 127
    c = torch.empty((130, 304), dtype=torch.int32, device=cuda)
    w8.mm_i8_nk(a, w, c)
    assert torch.equal(c, torch._int_mm(a, w.t().contiguous()))
    assert int(c[0, 1]) == k * 128 * 128
    assert int(c[1, 0]) == k * 127 * 127 and int(c[1, 1]) == -k * 127 * 128


# The tile width follows the wave count: 64 or 128 columns for GEMMs with one wave of
# tiles or less (short prompts, the 1536 -> 256 PLE gate), 192 for qkv / o at M = 3658,
# 256 otherwise; ragged last n-tiles (N = 200, 264) included.
@pytest.mark.parametrize("m,n,k", [(300, 384, 1536), (257, 200, 128), (513, 264, 640), (207, 2560, 1536),
                                   (858, 1536, 2048), (3658, 256, 1536), (1878, 1536, 2048), (3658, 2560, 1536)])
def test_dequant_every_tile_width_bit_exact(cuda, m, n, k):
    gen = torch.Generator(device=cuda).manual_seed(m + 7 * n + k)
    a = torch.randint(-128, 128, (m, k), dtype=torch.int8, device=cuda, generator=gen)
    w = torch.randint(-128, 128, (n, k), dtype=torch.int8, device=cuda, generator=gen)
    sx = torch.rand((m,), device=cuda, generator=gen) * 1e-2
    sw = torch.rand((n,), device=cuda, generator=gen) * 1e-3
    y = w8.gemm_dequant(a, w, sx, sw)
    c = torch.empty((m, n), dtype=torch.int32, device=cuda)
    w8.mm_i8_nk(a, w, c)
    assert torch.equal(c, torch._int_mm(a, w.t().contiguous()))
    rows = sorted({0, m - 1} | set(torch.randperm(m, generator=torch.Generator().manual_seed(1))[:20].tolist()))
    want = ref.dequant(c[rows].cpu().numpy(), sx[rows].cpu().numpy(), sw.cpu().numpy())
    np.testing.assert_array_equal(y[rows].cpu().view(torch.int16).numpy().view(np.uint16), want)


@pytest.mark.parametrize("n", [300, 301, 37])
def test_any_output_pitch(cuda, n):
    # contiguous C with N % 4 != 0: row starts are not 16-byte aligned -> element stores
    gen = torch.Generator().manual_seed(n)
    a = torch.randint(-128, 128, (70, 64), dtype=torch.int8, generator=gen)
    w = torch.randint(-128, 128, (n, 64), dtype=torch.int8, generator=gen)
    c = torch.empty((70, n), dtype=torch.int32, device=cuda)
    w8.mm_i8_nk(a.to(cuda), w.to(cuda), c)
    np.testing.assert_array_equal(c.cpu().numpy(), ref.int_mm(a.numpy(), w.numpy().T))
    sx = torch.rand(70) * 0.01
    sw = torch.rand(n) * 0.01
    y = torch.empty((70, n), dtype=torch.bfloat16, device=cuda)
    w8.gemm_dequant(a.to(cuda), w.to(cuda), sx.to(cuda), sw.to(cuda), out=y)
    want = ref.dequant(ref.int_mm(a.numpy(), w.numpy().T), sx.numpy(), sw.numpy())
    np.testing.assert_array_equal(y.cpu().view(torch.int16).numpy().view(np.uint16), want)


def test_k_zero_gives_zeros(cuda):
    a = torch.empty((5, 0), dtype=torch.int8, device=cuda)
    b = torch.empty((0, 32), dtype=torch.int8, device=cuda)
    c = torch.full((5, 32), 9, dtype=torch.int32, device=cuda)
    w8.mm_i8(a, b, c)
    assert int(c.abs().sum()) == 0


def test_rejects_bad_inputs(cuda):
    a = torch.zeros((4, 24), dtype=torch.int8, device=cuda)  # K = 24 is not a multiple of 16
    with pytest.raises(_lib.W8InvalidArgument):
        w8.mm_i8(a, torch.zeros((24, 16), dtype=torch.int8, device=cuda),
                 torch.zeros((4, 16), dtype=torch.int32, device=cuda))
    big = torch.zeros((4, 33), dtype=torch.int8, device=cuda)
    with pytest.raises(_lib.W8AlignmentError):  # A starts one byte past a 16-byte boundary
        w8.mm_i8(big[:, 1:], torch.zeros((32, 16), dtype=torch.int8, device=cuda),
                 torch.zeros((4, 16), dtype=torch.int32, device=cuda))
    with pytest.raises(ValueError):
        w8.mm_i8(a.float(), a, a)


def test_streams_and_device_status(cuda):
    s = torch.cuda.Stream()
    a = torch.randint(-128, 128, (256, 512), dtype=torch.int8, device=cuda)
    w = torch.randint(-128, 128, (384, 512), dtype=torch.int8, device=cuda)
    c = torch.empty((256, 384), dtype=torch.int32, device=cuda)
    with torch.cuda.stream(s):
        w8.mm_i8_nk(a, w, c)
    s.synchronize()
    assert torch.equal(c, torch._int_mm(a, w.t().contiguous()))
    assert w8.device_status() == 0
