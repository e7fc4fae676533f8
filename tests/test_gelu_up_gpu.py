"""The gate/up glue fused onto the GEMM (w8_gemm_gelu_up_quant) against the oracle.

The reference runs k_gelu (pipeline.py:102-107) on the CPU over the int32 gate/up GEMM
output: dequant, bf16(gelu_tanh(gate) * up), per-row int8 quant.  The CUDA path fuses
everything before the quant into the GEMM epilogue and finishes with a row quant.  The
oracle restatement (oracle/w8a8_numpy.gelu_up_quant) is pinned bit-exactly to the
reference's own function by tests/golden/gelu_up.npz.

Tolerance: the kernel forms 1 + tanh(z) from hardware exp2 / reciprocal approximations
(relative error a few 2^-23) where the oracle calls numpy's tanh, so an element of the
bf16 activation may differ by one bf16 step, which can move its int8 code by one.  So:
|q - q_ref| <= 1 everywhere with at most 0.5 % of codes different; the bf16 activation
within one bf16 step (relative 2^-7) plus an absolute 1e-6 of its row's absmax (the
deep negative tail of gelu, where both sides are within 1e-6 of zero); and the row
scales within max-rel 1e-2 (the north-star bound for dequantised outputs).
"""
import numpy as np
import pytest
import torch

import gemma_npu_b200 as w8
from oracle import w8a8_numpy as ref

pytestmark = pytest.mark.gpu


def _oracle_rows(x, w, sx, sw, rows, inter):
    acc = ref.int_mm(x[rows].cpu().numpy(), w.t().cpu().numpy())
    y = ref.bf16_bits_to_f32(ref.dequant(acc, sx[rows].cpu().numpy(), sw.cpu().numpy()))
    a = ref.bf16_bits_to_f32(ref.f32_to_bf16_bits(
        (ref.gelu_tanh_bf16(y[:, :inter]) * y[:, inter:]).astype(np.float32)))
    q, s = ref.gelu_up_quant(acc, sx[rows].cpu().numpy(), sw.cpu().numpy(), inter)
    return a, q, s


def _check(q, s, y, rows, a_ref, q_ref, s_ref):
    qd = np.abs(q[rows].cpu().numpy().astype(np.int32) - q_ref.astype(np.int32))
    assert qd.max() <= 1
    assert (qd != 0).mean() <= 5e-3
    yv = y[rows].float().cpu().numpy()
    floor = 1e-6 * np.abs(a_ref).max(axis=1, keepdims=True)  # far below one int8 step of the row
    assert np.all(np.abs(yv - a_ref) <= np.abs(a_ref) * 2.0 ** -7 + floor)
    sv = s[rows].cpu().numpy()
    assert float(np.abs(sv - s_ref).max() / max(np.abs(s_ref).max(), 1e-30)) <= 1e-2


def test_golden_vectors(cuda, golden):
    g = golden("gelu_up")
    inter = int(g["inter"])
    x = torch.from_numpy(g["x"]).to(cuda)
    wp, swp = w8.pack_gelu_up(torch.from_numpy(g["w"]).to(cuda), torch.from_numpy(g["sw"]).to(cuda))
    sx = torch.from_numpy(g["sx"]).to(cuda)
    q, s = w8.gelu_up_quant(x, sx, wp, swp)
    torch.cuda.synchronize()
    qd = np.abs(q.cpu().numpy().astype(np.int32) - g["q"].astype(np.int32))
    assert qd.max() <= 1 and (qd != 0).mean() <= 5e-3
    np.testing.assert_allclose(s.cpu().numpy(), g["s"], rtol=1e-2)
    assert s[0].item() == np.float32(1e-8) / np.float32(127)  # zero row: the scale floor
    assert not q[0].any()


# (M, I, K): config-1 gate/up (M = 3658, I = 6144, K = 1536); CTA pairs with K / 128 odd;
# a single-CTA M; K % 128 != 0 (single-CTA tiles at any M); the smallest I.
SHAPES = [(3658, 6144, 1536), (300, 256, 1664), (64, 6144, 1536), (200, 384, 208), (257, 128, 256),
          (3658, 12288, 1536)]  # the double-wide MLP of the real E2B mix


@pytest.mark.parametrize("m,inter,k", SHAPES)
def test_matches_oracle(cuda, m, inter, k):
    gen = torch.Generator(device=cuda).manual_seed(m + inter + k)
    x, sx = w8.quant_rows(torch.randn((m, k), device=cuda, generator=gen, dtype=torch.bfloat16))
    w, sw = w8.quant_rows(torch.randn((2 * inter, k), device=cuda, generator=gen, dtype=torch.bfloat16) * 0.02)
    wp, swp = w8.pack_gelu_up(w, sw)
    y = torch.empty((m, inter), dtype=torch.bfloat16, device=cuda)
    q, s = w8.gelu_up_quant(x, sx, wp, swp, y=y)
    torch.cuda.synchronize()
    rows = sorted({0, 1, m - 1} | set(torch.randint(0, m, (29,), generator=torch.Generator().manual_seed(m)).tolist()))
    a_ref, q_ref, s_ref = _oracle_rows(x, w, sx, sw, rows, inter)
    _check(q, s, y, rows, a_ref, q_ref, s_ref)


def test_repeat_calls_are_identical(cuda):
    """The row-absmax scratch is reset by every call: a second call gives the same bits."""
    m, inter, k = 1000, 1024, 1536
    gen = torch.Generator(device=cuda).manual_seed(5)
    x, sx = w8.quant_rows(torch.randn((m, k), device=cuda, generator=gen, dtype=torch.bfloat16))
    w, sw = w8.quant_rows(torch.randn((2 * inter, k), device=cuda, generator=gen, dtype=torch.bfloat16) * 0.02)
    wp, swp = w8.pack_gelu_up(w, sw)
    q1, s1 = w8.gelu_up_quant(x, sx, wp, swp)
    q2, s2 = w8.gelu_up_quant(x, sx, wp, swp)
    torch.cuda.synchronize()
    assert torch.equal(q1, q2) and torch.equal(s1, s2)


@pytest.mark.parametrize("m,inter,k", [(512, 1024, 1536), (3658, 6144, 1536)])
def test_equals_unfused_gpu_chain(cuda, m, inter, k):
    """Fused result == the unfused GPU chain: int32 GEMM, then the glue on the int32
    output (torch ops with the reference's expression), on all rows -- at config 1's full
    gate/up size too."""
    gen = torch.Generator(device=cuda).manual_seed(9 + m)
    x, sx = w8.quant_rows(torch.randn((m, k), device=cuda, generator=gen, dtype=torch.bfloat16))
    w, sw = w8.quant_rows(torch.randn((2 * inter, k), device=cuda, generator=gen, dtype=torch.bfloat16) * 0.02)
    wp, swp = w8.pack_gelu_up(w, sw)
    q, s = w8.gelu_up_quant(x, sx, wp, swp)
    acc = torch.empty((m, 2 * inter), dtype=torch.int32, device=cuda)
    w8.mm_i8_nk(x, w, acc)
    y = w8.dequant(acc, sx, sw)
    a = (torch.nn.functional.gelu(y[:, :inter], approximate="tanh") * y[:, inter:]).to(torch.bfloat16)
    q2, s2 = w8.quant_rows(a)
    torch.cuda.synchronize()
    qd = (q.int() - q2.int()).abs()
    assert qd.max().item() <= 1 and (qd != 0).float().mean().item() <= 5e-3
    assert torch.allclose(s, s2, rtol=1e-2, atol=0)
