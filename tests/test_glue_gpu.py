"""The RMSNorm / residual / quant glue (k_in, k_post_attn, k_post_ff, k_attn_out of
pipeline.py:66-99, 110-114) on the GPU against the oracle and the reference's own outputs.

The oracle restatements (oracle/w8a8_numpy.k_in / k_post / k_attn_out) reproduce the
reference's eager functions bit for bit on tests/golden/k_*.npz.  The kernels sum
mean(x^2) in another order than ATen, so the last bit of a mean can differ: a bf16
output may move by one bf16 step (relative 2^-7; for h = res + t one step of t plus h's
own rounding) and an
int8 code by one, on at most 1 % of the elements; scales within relative 2^-7.  k_attn_out has no reduction but the
absmax and is bit-exact.
"""
import numpy as np
import pytest
import torch

import gemma_npu_b200 as w8
from oracle import w8a8_numpy as ref

pytestmark = pytest.mark.gpu


def bf16(bits, dev):
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16).to(dev)


def bits(t):
    return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def close_bf16(a_bits, b_bits, frac=1e-2, res=None, per_vector=False):
    """Within one bf16 step.  For h = bf16(res + t), one step of t moves the exact sum by up
    to 2^-7 |t| <= 2^-7 (|h| + |res|) and the sum's own rounding then by up to one step of
    h, so the bound is 2^-7 (2 |h| + |res|) (res and t may nearly cancel).  RoPE's
    x * cos + rotate_half(x) * sin can cancel the same way: per_vector bounds by one step
    of the largest element of the (token, head) vector."""
    a, b = ref.bf16_bits_to_f32(a_bits), ref.bf16_bits_to_f32(b_bits)
    d = np.abs(a - b)
    scale = np.abs(b) if res is None else 2 * np.abs(b) + np.abs(np.asarray(res, np.float32))
    if per_vector:
        scale = scale + np.abs(b).max(axis=-1, keepdims=True)
    assert np.all(d <= scale * 2.0 ** -7 + 1e-30)
    assert (d != 0).mean() <= frac


def close_q(q, q_ref, frac=1e-2):
    d = np.abs(q.astype(np.int32) - q_ref.astype(np.int32))
    assert d.max() <= 1 and (d != 0).mean() <= frac


def test_golden_k_in(cuda, golden):
    g = golden("k_in")
    q, s = w8.rms_quant(bf16(g["h"], cuda), bf16(g["w"], cuda), float(g["eps"]))
    close_q(q.cpu().numpy(), g["q"])
    np.testing.assert_allclose(s.cpu().numpy(), g["s"], rtol=2.0 ** -7)


@pytest.mark.parametrize("name", ["k_post_attn", "k_post_ff"])
def test_golden_k_post(cuda, golden, name):
    g = golden(name)
    acc = torch.from_numpy(g["acc"]).to(cuda)
    y = w8.dequant(acc, torch.from_numpy(g["sx"]).to(cuda), torch.from_numpy(g["sw"]).to(cuda))
    w2 = bf16(g["w2"], cuda) if "w2" in g else None
    h, q, s = w8.post_norm_quant(y, bf16(g["res"], cuda), bf16(g["w1"], cuda), w2, float(g["eps"]))
    close_bf16(bits(h), g["h"], res=ref.bf16_bits_to_f32(g["res"]))
    close_q(q.cpu().numpy(), g["q"])
    np.testing.assert_allclose(s.cpu().numpy(), g["s"], rtol=2.0 ** -7)


def test_golden_k_attn_out_bit_exact(cuda, golden):
    g = golden("k_attn_out")
    q, s = w8.attn_out_quant(bf16(g["o"], cuda))
    np.testing.assert_array_equal(q.cpu().numpy(), g["q"])
    np.testing.assert_array_equal(s.cpu().numpy(), g["s"])


def _rows(t, seed):
    return sorted({0, t - 1} | set(torch.randint(0, t, (62,), generator=torch.Generator().manual_seed(seed)).tolist()))


@pytest.mark.parametrize("t,n", [(3658, 1536), (207, 2048), (5, 8)])
def test_k_in_matches_oracle(cuda, t, n):
    gen = torch.Generator(device=cuda).manual_seed(t + n)
    h = (torch.randn((t, n), device=cuda, generator=gen) * 3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn((n,), device=cuda, generator=gen)).to(torch.bfloat16)
    q, s = w8.rms_quant(h, w, 1e-6)
    rows = _rows(t, n)
    qr, sr = ref.k_in(h[rows].float().cpu().numpy(), w.float().cpu().numpy(), 1e-6)
    close_q(q[rows].cpu().numpy(), qr)
    np.testing.assert_allclose(s[rows].cpu().numpy(), sr, rtol=2.0 ** -7)


@pytest.mark.parametrize("two", [True, False])
@pytest.mark.parametrize("t,n", [(3658, 1536), (300, 512)])
def test_gemm_then_post_norm_matches_oracle(cuda, t, n, two):
    """o / down GEMM with the dequant fused, then k_post_attn (two) or k_post_ff glue."""
    k = 2048
    gen = torch.Generator(device=cuda).manual_seed(t + n + two)
    x, sx = w8.quant_rows(torch.randn((t, k), device=cuda, generator=gen, dtype=torch.bfloat16))
    wq, sw = w8.quant_rows(torch.randn((n, k), device=cuda, generator=gen, dtype=torch.bfloat16) * 0.02)
    res = torch.randn((t, n), device=cuda, generator=gen).to(torch.bfloat16)
    w1 = (1 + 0.1 * torch.randn((n,), device=cuda, generator=gen)).to(torch.bfloat16)
    w2 = (1 + 0.1 * torch.randn((n,), device=cuda, generator=gen)).to(torch.bfloat16) if two else None
    y = w8.gemm_dequant(x, wq, sx, sw)
    res0 = res.clone()
    h, q, s = w8.post_norm_quant(y, res, w1, w2, 1e-6, h=res)  # in place, as the residual stream
    assert h.data_ptr() == res.data_ptr()
    rows = _rows(t, n)
    acc = ref.int_mm(x[rows].cpu().numpy(), wq.t().cpu().numpy())
    yr = ref.bf16_bits_to_f32(ref.dequant(acc, sx[rows].cpu().numpy(), sw.cpu().numpy()))
    hr, qr, sr = ref.k_post(yr, res0[rows].float().cpu().numpy(), w1.float().cpu().numpy(),
                            None if w2 is None else w2.float().cpu().numpy(), 1e-6)
    close_bf16(bits(h[rows]), ref.f32_to_bf16_bits(hr), res=res0[rows].float().cpu().numpy())
    close_q(q[rows].cpu().numpy(), qr)
    np.testing.assert_allclose(s[rows].cpu().numpy(), sr, rtol=2.0 ** -7)


@pytest.mark.parametrize("d", [256, 512])
def test_attn_out_strided_bit_exact(cuda, d):
    """o as attention produces it ([H, T, D], here a slice of a wider buffer); D = 512 is a
    full-attention layer (H * D = 4096)."""
    H, T, D = 8, 1000, d
    gen = torch.Generator(device=cuda).manual_seed(3)
    big = torch.randn((H, T + 24, D), device=cuda, generator=gen).to(torch.bfloat16)
    o = big[:, 10:10 + T]
    q, s = w8.attn_out_quant(o)
    qr, sr = ref.k_attn_out(o.float().cpu().numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), qr)
    np.testing.assert_array_equal(s.cpu().numpy(), sr)


@pytest.mark.parametrize("name", ["k_qkv", "k_qkv_shared"])
def test_golden_k_qkv(cuda, golden, name):
    g = golden(name)
    nh, kv, d, shared = (int(v) for v in g["dims"])
    y = w8.dequant(torch.from_numpy(g["acc"]).to(cuda), torch.from_numpy(g["sx"]).to(cuda),
                   torch.from_numpy(g["sw"]).to(cuda))
    if shared:
        y = y[:, : nh * d].contiguous()
    q, k, v = w8.qkv_norm_rope(y, bf16(g["cos"], cuda), bf16(g["sin"], cuda), bf16(g["qw"], cuda),
                               None if shared else bf16(g["kw"], cuda), float(g["eps"]), nh, kv, d, bool(shared))
    for mine, theirs in ((q, g["q"]), (k, g["k"]), (v, g["v"])):
        close_bf16(bits(mine), theirs, per_vector=True)


def _rope_tables(t, d, dev):
    ang = torch.arange(t, device=dev)[:, None].float() * (1e6 ** (-torch.arange(0, d, 2, device=dev).float() / d))[None]
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)


@pytest.mark.parametrize("t,nh,kv,d,shared", [(3658, 8, 1, 256, False), (3658, 8, 1, 256, True),
                                              (300, 4, 2, 512, False), (129, 16, 4, 128, False),
                                              (64, 8, 2, 64, False)])
def test_qkv_gemm_then_norm_rope_matches_oracle(cuda, t, nh, kv, d, shared):
    """qkv GEMM with the dequant fused, then the k_qkv glue, against the oracle on sampled tokens."""
    k = 1536
    n = (nh if shared else nh + 2 * kv) * d
    gen = torch.Generator(device=cuda).manual_seed(t + d)
    x, sx = w8.quant_rows(torch.randn((t, k), device=cuda, generator=gen, dtype=torch.bfloat16))
    wq, sw = w8.quant_rows(torch.randn((n, k), device=cuda, generator=gen, dtype=torch.bfloat16) * 0.02)
    cos, sin = _rope_tables(t, d, cuda)
    qw = (1 + 0.1 * torch.randn((d,), device=cuda, generator=gen)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn((d,), device=cuda, generator=gen)).to(torch.bfloat16)
    y = w8.gemm_dequant(x, wq, sx, sw)
    q, kk, v = w8.qkv_norm_rope(y, cos, sin, qw, kw, 1e-6, nh, kv, d, shared)
    rows = _rows(t, d)
    acc = ref.int_mm(x[rows].cpu().numpy(), wq.t().cpu().numpy())
    f = lambda z: z.float().cpu().numpy()
    qr, kr, vr = ref.k_qkv(acc, f(sx[rows]), f(sw), f(cos[rows]), f(sin[rows]), f(qw), None if shared else f(kw),
                           1e-6, nh, kv, d, shared)
    for mine, theirs in ((q, qr), (kk, kr), (v, vr)):
        close_bf16(bits(mine[:, rows]), ref.f32_to_bf16_bits(theirs), per_vector=True)


# ---- the per-layer-input (PLE) branch: k_ple_gate / k_ple_out (pipeline.py:117-127).
# gelu's 1 + tanh comes from exp2 / reciprocal approximations (relative error a few
# 2^-23), so a gated value may move by one bf16 step and an int8 code by one.

def test_golden_k_ple_gate(cuda, golden):
    g = golden("k_ple_gate")
    acc = torch.from_numpy(g["acc"]).to(cuda)
    y = w8.dequant(acc, torch.from_numpy(g["sx"]).to(cuda), torch.from_numpy(g["sw"]).to(cuda))
    q, s = w8.ple_gate_quant(y, bf16(g["ple"], cuda))
    close_q(q.cpu().numpy(), g["q"])
    np.testing.assert_allclose(s.cpu().numpy(), g["s"], rtol=2.0 ** -7)
    assert s[0].item() == np.float32(1e-8) / np.float32(127)  # the gated-off row: the scale floor


@pytest.mark.parametrize("name", ["k_ple_out", "k_ple_out_one"])
def test_golden_k_ple_out(cuda, golden, name):
    g = golden(name)
    acc = torch.from_numpy(g["acc"]).to(cuda)
    y = w8.dequant(acc, torch.from_numpy(g["sx"]).to(cuda), torch.from_numpy(g["sw"]).to(cuda))
    scalar = bf16(g["scalar"], cuda)
    h = w8.ple_out(y, bf16(g["res"], cuda), bf16(g["w1"], cuda), scalar, float(g["eps"]))
    close_bf16(bits(h), g["h"], res=ref.bf16_bits_to_f32(g["res"]) * float(scalar.float().item()))


@pytest.mark.parametrize("t", [3658, 300])
def test_ple_branch_matches_oracle(cuda, t):
    """The whole PLE branch of a layer on the GPU: gate GEMM (1536 -> 256, dequant fused),
    k_ple_gate with a [:, layer] slice of the [T, layers, 256] per-layer inputs, projection
    GEMM (256 -> 1536), k_ple_out in place on the residual stream fused with the next
    layer's k_in.  Each stage is checked against the oracle on the GPU's own inputs."""
    hid, pn, layers, layer = 1536, 256, 35, 17
    gen = torch.Generator(device=cuda).manual_seed(t)
    x, sx = w8.quant_rows(torch.randn((t, hid), device=cuda, generator=gen, dtype=torch.bfloat16))
    wg, swg = w8.quant_rows(torch.randn((pn, hid), device=cuda, generator=gen, dtype=torch.bfloat16) * 0.02)
    wp, swp = w8.quant_rows(torch.randn((hid, pn), device=cuda, generator=gen, dtype=torch.bfloat16) * 0.02)
    ple_all = torch.randn((t, layers, pn), device=cuda, generator=gen).to(torch.bfloat16)
    ple = ple_all[:, layer]
    res = torch.randn((t, hid), device=cuda, generator=gen).to(torch.bfloat16)
    w_post = (1 + 0.1 * torch.randn((hid,), device=cuda, generator=gen)).to(torch.bfloat16)
    w_next = (1 + 0.1 * torch.randn((hid,), device=cuda, generator=gen)).to(torch.bfloat16)
    scalar = torch.tensor([0.4], device=cuda).to(torch.bfloat16)

    yg = w8.gemm_dequant(x, wg, sx, swg)
    q1, s1 = w8.ple_gate_quant(yg, ple)
    yp = w8.gemm_dequant(q1, wp, s1, swp)
    res0 = res.clone()
    h, q2, s2 = w8.ple_out(yp, res, w_post, scalar, 1e-6, w_next=w_next, h=res)
    assert h.data_ptr() == res.data_ptr()

    rows = _rows(t, 7)
    yr = ref.bf16_bits_to_f32(ref.dequant(ref.int_mm(x[rows].cpu().numpy(), wg.t().cpu().numpy()),
                                          sx[rows].cpu().numpy(), swg.cpu().numpy()))
    np.testing.assert_array_equal(bits(yg[rows]), ref.f32_to_bf16_bits(yr))
    qr1, sr1 = ref.k_ple_gate(yr, ple[rows].float().cpu().numpy())
    close_q(q1[rows].cpu().numpy(), qr1)
    np.testing.assert_allclose(s1[rows].cpu().numpy(), sr1, rtol=2.0 ** -7)

    yr2 = ref.bf16_bits_to_f32(ref.dequant(ref.int_mm(q1[rows].cpu().numpy(), wp.t().cpu().numpy()),
                                           s1[rows].cpu().numpy(), swp.cpu().numpy()))
    sc = float(scalar.float().item())
    hr = ref.k_ple_out(yr2, res0[rows].float().cpu().numpy(), w_post.float().cpu().numpy(), sc, 1e-6)
    close_bf16(bits(h[rows]), ref.f32_to_bf16_bits(hr), res=res0[rows].float().cpu().numpy() * sc)
    qr2, sr2 = ref.k_in(h[rows].float().cpu().numpy(), w_next.float().cpu().numpy(), 1e-6)
    close_q(q2[rows].cpu().numpy(), qr2)
    np.testing.assert_allclose(s2[rows].cpu().numpy(), sr2, rtol=2.0 ** -7)

    # Without the next layer's weight: h only, the same values.
    h2 = w8.ple_out(yp, res0, w_post, scalar, 1e-6)
    assert torch.equal(h2, h)


# ---- every row at config 1's size: the int32 product from torch._int_mm (cuBLASLt,
# bit-exact to the oracle's int_mm), the glue of all 3658 rows from the oracle.

def test_k_in_all_rows(cuda):
    t, n = 3658, 1536
    gen = torch.Generator(device=cuda).manual_seed(101)
    h = (torch.randn((t, n), device=cuda, generator=gen) * 3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn((n,), device=cuda, generator=gen)).to(torch.bfloat16)
    q, s = w8.rms_quant(h, w, 1e-6)
    qr, sr = ref.k_in(h.float().cpu().numpy(), w.float().cpu().numpy(), 1e-6)
    close_q(q.cpu().numpy(), qr)
    np.testing.assert_allclose(s.cpu().numpy(), sr, rtol=2.0 ** -7)


@pytest.mark.parametrize("two", [True, False])
def test_post_norm_all_rows(cuda, two):
    t, n, k = 3658, 1536, 2048 if two else 6144
    gen = torch.Generator(device=cuda).manual_seed(102 + two)
    x, sx = w8.quant_rows(torch.randn((t, k), device=cuda, generator=gen, dtype=torch.bfloat16))
    wq, sw = w8.quant_rows(torch.randn((n, k), device=cuda, generator=gen, dtype=torch.bfloat16) * 0.02)
    res = torch.randn((t, n), device=cuda, generator=gen).to(torch.bfloat16)
    w1 = (1 + 0.1 * torch.randn((n,), device=cuda, generator=gen)).to(torch.bfloat16)
    w2 = (1 + 0.1 * torch.randn((n,), device=cuda, generator=gen)).to(torch.bfloat16) if two else None
    res0 = res.clone()
    h, q, s = w8.post_norm_quant(w8.gemm_dequant(x, wq, sx, sw), res, w1, w2, 1e-6, h=res)
    acc = torch._int_mm(x, wq.t()).cpu().numpy()
    yr = ref.bf16_bits_to_f32(ref.dequant(acc, sx.cpu().numpy(), sw.cpu().numpy()))
    hr, qr, sr = ref.k_post(yr, res0.float().cpu().numpy(), w1.float().cpu().numpy(),
                            None if w2 is None else w2.float().cpu().numpy(), 1e-6)
    close_bf16(bits(h), ref.f32_to_bf16_bits(hr), res=res0.float().cpu().numpy())
    close_q(q.cpu().numpy(), qr)
    np.testing.assert_allclose(s.cpu().numpy(), sr, rtol=2.0 ** -7)


def test_qkv_norm_rope_all_rows(cuda):
    t, nh, kv, d, k = 3658, 8, 1, 256, 1536
    n = (nh + 2 * kv) * d
    gen = torch.Generator(device=cuda).manual_seed(103)
    x, sx = w8.quant_rows(torch.randn((t, k), device=cuda, generator=gen, dtype=torch.bfloat16))
    wq, sw = w8.quant_rows(torch.randn((n, k), device=cuda, generator=gen, dtype=torch.bfloat16) * 0.02)
    cos, sin = _rope_tables(t, d, cuda)
    qw = (1 + 0.1 * torch.randn((d,), device=cuda, generator=gen)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn((d,), device=cuda, generator=gen)).to(torch.bfloat16)
    q, kk, v = w8.qkv_norm_rope(w8.gemm_dequant(x, wq, sx, sw), cos, sin, qw, kw, 1e-6, nh, kv, d)
    acc = torch._int_mm(x, wq.t()).cpu().numpy()
    f = lambda z: z.float().cpu().numpy()
    qr, kr, vr = ref.k_qkv(acc, f(sx), f(sw), f(cos), f(sin), f(qw), f(kw), 1e-6, nh, kv, d, False)
    for mine, theirs in ((q, qr), (kk, kr), (v, vr)):
        close_bf16(bits(mine), ref.f32_to_bf16_bits(theirs), per_vector=True)
