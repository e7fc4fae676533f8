"""Prefill attention (pipeline.py:139-180) on the GPU against the reference's own outputs
(tests/golden/attn_*.npz, made by pipeline.sliding_attention / full_attention) and the
float64 oracle (oracle/w8a8_numpy.attention).

Tolerance: normwise max-rel <= 1e-2 (the north-star bound for bf16 outputs); the kernel
rounds P to bf16 before P @ V as flash attention does, the reference's CPU kernels keep
other roundings (the oracle itself is within 3e-3 of the reference's outputs).
"""
import numpy as np
import pytest
import torch

import gemma_npu_b200 as w8
from oracle import w8a8_numpy as ref

pytestmark = pytest.mark.gpu
MAX_REL = 1e-2


def bf16(bits, dev):
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16).to(dev)


def max_rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


SCHEDULES = ["tc", "mma"]  # tcgen05 (the product path) and the mma.sync cross-check


@pytest.mark.parametrize("schedule", SCHEDULES)
@pytest.mark.parametrize("name", ["attn_sliding", "attn_full"])
def test_golden(cuda, golden, name, schedule):
    g = golden(name)
    o = w8.attention_prefill(bf16(g["q"], cuda), bf16(g["k"], cuda), bf16(g["v"], cuda), int(g["window"]),
                             schedule=schedule)
    assert max_rel(o.float().cpu().numpy(), ref.bf16_bits_to_f32(g["o"])) <= MAX_REL
    assert w8.device_status() == 0


# (T, H, KV, D, window): Gemma E2B sliding (D 256, W 512) and full (D 512) layers at the
# config-1 length, ragged T, more KV heads, a window longer than the prompt.
# Grouped-query packing: group size 8 -> 8 heads x 16 queries per CTA, 4 -> 4 x 32, 16 -> 16 x 8,
# 3 -> one head per CTA (the largest power of two dividing 3 is 1).
SHAPES = [(3658, 8, 1, 256, 512), (3658, 8, 1, 512, 0), (1000, 4, 2, 256, 0), (77, 2, 1, 256, 512),
          (700, 8, 8, 512, 128), (1, 1, 1, 256, 0), (129, 2, 1, 512, 64), (500, 8, 2, 256, 512),
          (300, 16, 1, 256, 0), (200, 6, 2, 512, 100)]


@pytest.mark.parametrize("schedule", SCHEDULES)
@pytest.mark.parametrize("t,h,kv,d,window", SHAPES)
def test_matches_oracle(cuda, t, h, kv, d, window, schedule):
    gen = torch.Generator(device=cuda).manual_seed(t + d + window)
    scale = d ** -0.25  # logits O(1) at scale 1.0, as q_norm / k_norm keep them
    q = (torch.randn((h, t, d), device=cuda, generator=gen) * scale).to(torch.bfloat16)
    k = (torch.randn((kv, t, d), device=cuda, generator=gen) * scale).to(torch.bfloat16)
    v = torch.randn((kv, t, d), device=cuda, generator=gen).to(torch.bfloat16)
    o = w8.attention_prefill(q, k, v, window, schedule=schedule)
    torch.cuda.synchronize()
    assert w8.device_status() == 0
    # oracle on a sample of query rows (full rows of keys), every head
    sample = torch.randint(0, t, (13,), generator=torch.Generator().manual_seed(t)).tolist()
    rows = sorted(r for r in {0, 1, t - 1} | set(sample) if r < t)
    qn, kn, vn = q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy()
    group = h // kv
    for hh in range(h):
        s = qn[hh, rows].astype(np.float64) @ kn[hh // group].T.astype(np.float64)
        pos = np.arange(t)
        r = np.asarray(rows)[:, None]
        allowed = (pos[None, :] <= r) & ((r - pos[None, :]) < window if window else True)
        s = np.where(allowed, s, -np.inf)
        p = np.exp(s - s.max(axis=1, keepdims=True))
        want = (p / p.sum(axis=1, keepdims=True)) @ vn[hh // group].astype(np.float64)
        assert max_rel(o[hh, rows].float().cpu().numpy(), want) <= MAX_REL


@pytest.mark.parametrize("schedule", SCHEDULES)
@pytest.mark.parametrize("d", [256, 512])
def test_strided_views(cuda, d, schedule):
    """q / k / v as slices of the k_qkv glue's head-major buffer, o into a wider buffer."""
    t, h, kv = 300, 4, 1
    gen = torch.Generator(device=cuda).manual_seed(1)
    buf = (torch.randn((h + 2 * kv, t, d), device=cuda, generator=gen) * d ** -0.25).to(torch.bfloat16)
    q, k, v = buf[:h], buf[h:h + kv], buf[h + kv:]
    big = torch.zeros((h, t + 10, d), dtype=torch.bfloat16, device=cuda)
    o = w8.attention_prefill(q, k, v, 0, out=big[:, 5:5 + t], schedule=schedule)
    want = w8.attention_prefill(q.contiguous(), k.contiguous(), v.contiguous(), 0, schedule=schedule)
    assert torch.equal(o, want)
    assert not big[:, :5].any() and not big[:, 5 + t:].any()


@pytest.mark.parametrize("d,window", [(256, 512), (512, 0)])
def test_schedules_agree(cuda, d, window):
    """The tcgen05 and mma.sync schedules on the same inputs (Gemma E2B layer shapes, a
    ragged length): two independent implementations within the bf16 tolerance."""
    t, h, kv = 1234, 8, 1
    gen = torch.Generator(device=cuda).manual_seed(d + window)
    sc = d ** -0.25
    q = (torch.randn((h, t, d), device=cuda, generator=gen) * sc).to(torch.bfloat16)
    k = (torch.randn((kv, t, d), device=cuda, generator=gen) * sc).to(torch.bfloat16)
    v = torch.randn((kv, t, d), device=cuda, generator=gen).to(torch.bfloat16)
    a = w8.attention_prefill(q, k, v, window, schedule="tc").float()
    b = w8.attention_prefill(q, k, v, window, schedule="mma").float()
    assert float((a - b).abs().max() / b.abs().max()) <= MAX_REL
    assert w8.device_status() == 0


def test_large_logits(cuda):
    """Logits of +-60 (well past the 2^8 lazy-rescale threshold) with the maximum moving
    late in the keys: the tcgen05 schedule rescales O in TMEM and must stay within the
    tolerance of the float64 softmax."""
    t, h, d = 640, 2, 256
    gen = torch.Generator(device=cuda).manual_seed(5)
    q = (torch.randn((h, t, d), device=cuda, generator=gen) * 0.5).to(torch.bfloat16)
    k = (torch.randn((1, t, d), device=cuda, generator=gen) * 0.5).to(torch.bfloat16)
    k[:, t // 2:] *= 4  # later keys: larger logits, so row maxima move mid-row
    v = torch.randn((1, t, d), device=cuda, generator=gen).to(torch.bfloat16)
    o = w8.attention_prefill(q, k, v, 0, schedule="tc")
    torch.cuda.synchronize()
    qn, kn, vn = q.double().cpu().numpy(), k.double().cpu().numpy(), v.double().cpu().numpy()
    for hh in range(h):
        s = qn[hh] @ kn[0].T
        s = np.where(np.tril(np.ones((t, t), bool)), s, -np.inf)
        p = np.exp(s - s.max(axis=1, keepdims=True))
        want = (p / p.sum(axis=1, keepdims=True)) @ vn[0]
        assert max_rel(o[hh].float().cpu().numpy(), want) <= MAX_REL


@pytest.mark.parametrize("t,h,kv,window", [(3658, 8, 1, 512), (77, 8, 1, 512), (1000, 4, 1, 0), (300, 16, 1, 64),
                                           (500, 8, 2, 512)])
def test_attention_quant_fused(cuda, t, h, kv, window):
    """Attention with k_attn_out fused gives the bits of the two-step path (the fused kernel
    for one KV head; the two-step fallback for (8, 2))."""
    d = 256
    gen = torch.Generator(device=cuda).manual_seed(t + h + window)
    sc = d ** -0.25
    q = (torch.randn((h, t, d), device=cuda, generator=gen) * sc).to(torch.bfloat16)
    k = (torch.randn((kv, t, d), device=cuda, generator=gen) * sc).to(torch.bfloat16)
    v = torch.randn((kv, t, d), device=cuda, generator=gen).to(torch.bfloat16)
    xq, xs = w8.attention_quant(q, k, v, window)
    wq, ws = w8.attn_out_quant(w8.attention_prefill(q, k, v, window))
    assert torch.equal(xq, wq) and torch.equal(xs, ws)
    assert w8.device_status() == 0
