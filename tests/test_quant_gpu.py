"""Parity of the quant / dequant kernels and the fused-dequant GEMM with the reference.

quant_rows must reproduce pipeline._quant (pipeline.py:49-52) and the weight quant of
NPUGemm / Int8Head (gemma_npu.py:68-69,164-167) bit for bit; dequant and the fused
GEMM epilogue must reproduce pipeline._deq (pipeline.py:55-57) bit for bit (the
stated tolerance, max-rel <= 1e-2, is not needed: the fp32 operation order is the
reference's).
"""
import numpy as np
import pytest
import torch

import gemma_npu_b200 as w8
from oracle import w8a8_numpy as ref

pytestmark = pytest.mark.gpu


def bf16(bits, device):
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def test_golden_activation_quant(cuda, golden):
    g = golden("quant")
    q, s = w8.quant_rows(bf16(g["x"], cuda))
    np.testing.assert_array_equal(q.cpu().numpy(), g["q"])
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), g["s"].view(np.uint32))


def test_golden_weight_quant(cuda, golden):
    g = golden("wquant")
    wb = bf16(g["w"], cuda)
    for x in (wb, wb.float()):  # bf16 path and the reference's fp32 path
        q, s = w8.quant_rows(x)
        np.testing.assert_array_equal(q.cpu().numpy(), g["q"])
        np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), g["s_f32"].view(np.uint32))
        np.testing.assert_array_equal(bits(s.to(torch.bfloat16)), g["s"])


@pytest.mark.parametrize("k", [16, 40, 1536, 2048, 6144, 12288, 16400])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_quant_matches_oracle(cuda, k, dtype):
    gen = torch.Generator().manual_seed(k)
    x = (torch.randn(37, k, generator=gen) * torch.rand(37, 1, generator=gen) * 10).to(dtype)
    x[3] = 0
    q, s = w8.quant_rows(x.to(cuda))
    q0, s0 = ref.quant_rows(x.float().numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), q0)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), s0.view(np.uint32))


def test_quant_unaligned_rows_take_the_scalar_path(cuda):
    base = torch.randn(9, 1600, device=cuda).to(torch.bfloat16)
    x = base[:, 3:3 + 1531]  # odd offset and odd length
    q, s = w8.quant_rows(x)
    q0, s0 = ref.quant_rows(x.float().cpu().numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), q0)
    np.testing.assert_array_equal(s.cpu().numpy(), s0)


def test_golden_dequant(cuda, golden):
    g = golden("deq")
    acc = torch.from_numpy(g["acc"]).to(cuda)
    y = w8.dequant(acc, torch.from_numpy(g["sx"]).to(cuda), torch.from_numpy(g["sw"]).to(cuda))
    np.testing.assert_array_equal(bits(y), g["y"])


def test_golden_fused_gemm_dequant(cuda, golden):
    g, w, d = golden("int_mm"), golden("wquant"), golden("deq")
    a = torch.from_numpy(g["a"]).to(cuda)
    wq = torch.from_numpy(w["q"]).to(cuda)
    y = w8.gemm_dequant(a, wq, torch.from_numpy(d["sx"]).to(cuda), torch.from_numpy(d["sw"]).to(cuda))
    np.testing.assert_array_equal(bits(y), d["y"])


@pytest.mark.parametrize("m,n,k", [(3658, 2560, 1536), (512, 12288, 1536), (129, 300, 2048), (3, 1536, 6144)])
def test_fused_dequant_equals_mm_then_dequant(cuda, m, n, k):
    gen = torch.Generator(device=cuda).manual_seed(n)
    x = torch.randn((m, k), device=cuda, generator=gen).to(torch.bfloat16)
    wt = (torch.randn((n, k), device=cuda, generator=gen) * 0.02).to(torch.bfloat16)
    xq, sx = w8.quant_rows(x)
    wq, sw = w8.quant_rows(wt)
    y = w8.gemm_dequant(xq, wq, sx, sw)
    c = torch.empty((m, n), dtype=torch.int32, device=cuda)
    w8.mm_i8_nk(xq, wq, c)
    y2 = w8.dequant(c, sx, sw)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
    # and with the reference's CPU path on a sample of rows
    rows = list(range(0, m, max(1, m // 5)))[:5]
    want = ref.dequant(ref.int_mm(xq[rows].cpu().numpy(), wq.t().cpu().numpy()), sx[rows].cpu().numpy(),
                       sw.cpu().numpy())
    np.testing.assert_array_equal(bits(y[rows]), want)


def _near_ties(rows, k, seed):
    """fp32 rows whose quotients x / s sit on and next to the half-integers k + 0.5, where a
    division one ulp off would change round-half-even: row r has absmax 127 * s0 (so its
    scale s is s0 up to rounding) and its other entries are (j + 0.5) * s0 nudged by
    -2..2 ulps, over scales s0 spread across 40 binades."""
    rng = np.random.default_rng(seed)
    s0 = (2.0 ** rng.uniform(-30, 10, size=(rows, 1))).astype(np.float32)
    j = rng.integers(-127, 127, size=(rows, k)).astype(np.float32)
    x = ((j + np.float32(0.5)) * s0).astype(np.float32)
    nudge = rng.integers(-2, 3, size=(rows, k)).astype(np.int32)
    x = (x.view(np.int32) + nudge).view(np.float32)
    x[:, 0] = np.float32(127) * s0[:, 0]
    x[:, 1] = -np.float32(127) * s0[:, 0]
    return x


@pytest.mark.parametrize("seed", [0, 1])
def test_quant_division_is_correctly_rounded(cuda, seed):
    """The kernels divide with a reciprocal and one correction step; the int8 codes must
    equal those of an IEEE division (numpy) bit for bit, on near-tie quotients and on
    random rows, for fp32 and bf16 input."""
    x = _near_ties(1024, 2048, seed)
    rng = np.random.default_rng(seed + 10)
    x = np.concatenate([x, (rng.standard_normal((1024, 2048)) * 2.0 ** rng.uniform(-20, 20, (1024, 1)))
                        .astype(np.float32)])
    for t in (torch.from_numpy(x).to(cuda), torch.from_numpy(x).to(cuda).to(torch.bfloat16)):
        q, s = w8.quant_rows(t)
        qr, sr = ref.quant_rows(t.float().cpu().numpy())
        np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), sr.view(np.uint32))
        np.testing.assert_array_equal(q.cpu().numpy(), qr)
