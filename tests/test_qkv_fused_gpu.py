"""The qkv GEMM with k_qkv fused into its epilogue (w8_gemm_qkv_norm_rope, head_dim 256).

The fused kernel must give, bit for bit over every token and head, what the two-step path
gives -- the qkv GEMM with the dequant fused (w8_gemm_dequant_bf16), then the k_qkv row
kernel (w8_qkv_norm_rope_bf16) -- and that path is checked against the reference's k_qkv
(golden vectors) and the oracle in test_glue_gpu.py.  Both the CTA-pair kernel (T > 128)
and the single-CTA kernel (T <= 128), KV-shared layers (q only), ragged token counts and
strided outputs are covered, plus one direct check against the oracle.
"""
import numpy as np
import pytest
import torch

import gemma_npu_b200 as w8
from oracle import w8a8_numpy as ref

pytestmark = pytest.mark.gpu


def rope_tables(t, d, dev, pitch=None):
    ang = torch.arange(t, device=dev)[:, None].float() * (1e4 ** (-torch.arange(0, d, 2, device=dev).float() / d))[None]
    ang = torch.cat([ang, ang], dim=-1)
    cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    if pitch is not None:  # the tables as views of wider rows
        wide = torch.zeros((2, t, pitch), dtype=torch.bfloat16, device=dev)
        wide[0, :, :d], wide[1, :, :d] = cos, sin
        cos, sin = wide[0, :, :d], wide[1, :, :d]
    return cos, sin


def setup(t, nh, kv, shared, k, dev, seed):
    d = 256
    n = (nh if shared else nh + 2 * kv) * d
    gen = torch.Generator(device=dev).manual_seed(seed)
    x, sx = w8.quant_rows(torch.randn((t, k), device=dev, generator=gen, dtype=torch.bfloat16))
    wq, sw = w8.quant_rows(torch.randn((n, k), device=dev, generator=gen, dtype=torch.bfloat16) * 0.02)
    qw = (1 + 0.1 * torch.randn((d,), device=dev, generator=gen)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn((d,), device=dev, generator=gen)).to(torch.bfloat16)
    return x, sx, wq, sw, qw, kw


@pytest.mark.parametrize("t,nh,kv,shared,k", [(3658, 8, 1, False, 1536), (3658, 8, 1, True, 1536),
                                              (207, 8, 1, False, 1536), (1000, 4, 2, False, 2048),
                                              (129, 8, 1, False, 1536), (128, 8, 1, False, 1536),
                                              (100, 8, 1, False, 1536), (1, 2, 1, False, 256),
                                              (37, 3, 1, True, 112)])
def test_fused_equals_two_step_path(cuda, t, nh, kv, shared, k):
    x, sx, wq, sw, qw, kw = setup(t, nh, kv, shared, k, cuda, t + nh + k)
    cos, sin = rope_tables(t, 256, cuda, pitch=320 if t % 2 else None)
    eps = 1e-6
    want = w8.qkv_norm_rope(w8.gemm_dequant(x, wq, sx, sw), cos, sin, qw, kw, eps, nh, kv, 256, shared)
    per_tok = nh if shared else nh + 2 * kv
    big = torch.full((per_tok, t + 5, 256 + 64), float("nan"), dtype=torch.bfloat16, device=cuda)
    out = big[:, :t, :256]  # strided head-major output (token pitch 320, head pitch (t + 5) * 320)
    got = w8.gemm_qkv_norm_rope(x, wq, sx, sw, cos, sin, qw, kw, eps, nh, kv, 256, shared, out=out)
    torch.cuda.synchronize()
    for name, g, w_ in zip("qkv", got, want):
        assert torch.equal(g.view(torch.int16), w_.view(torch.int16)), name
    assert torch.isnan(big[:, t:].float()).all() and torch.isnan(big[:, :, 256:].float()).all()  # nothing outside
    # the same kernel reading cos / sin from the 8-column tiled tables: the same bits
    big.fill_(float("nan"))
    got = w8.gemm_qkv_norm_rope(x, wq, sx, sw, cos, sin, qw, kw, eps, nh, kv, 256, shared, out=out,
                                tiles=w8.rope_tiles(cos, sin))
    torch.cuda.synchronize()
    for name, g, w_ in zip("qkv", got, want):
        assert torch.equal(g.view(torch.int16), w_.view(torch.int16)), "tiled " + name
    assert torch.isnan(big[:, t:].float()).all() and torch.isnan(big[:, :, 256:].float()).all()


def test_fused_against_oracle(cuda):
    t, nh, kv, k = 300, 8, 1, 1536
    x, sx, wq, sw, qw, kw = setup(t, nh, kv, False, k, cuda, 5)
    cos, sin = rope_tables(t, 256, cuda)
    q, kk, v = w8.gemm_qkv_norm_rope(x, wq, sx, sw, cos, sin, qw, kw, 1e-6, nh, kv, 256)
    rows = np.array([0, 1, 17, 128, 255, 256, 299])
    acc = ref.int_mm(x[rows].cpu().numpy(), wq.t().cpu().numpy())
    f = lambda z: z.float().cpu().numpy()
    qr, kr, vr = ref.k_qkv(acc, f(sx[rows]), f(sw), f(cos[rows]), f(sin[rows]), f(qw), f(kw), 1e-6, nh, kv, 256,
                           False)
    for mine, theirs in ((q, qr), (kk, kr), (v, vr)):
        a = mine[:, rows].float().cpu().numpy()
        b = ref.bf16_bits_to_f32(ref.f32_to_bf16_bits(theirs))
        # within one bf16 step of the oracle (the norm sums run in another order than ATen's)
        step = np.maximum(np.abs(b), 2.0 ** -126) * 2.0 ** -7
        assert (np.abs(a - b) <= step * 1.01).all()


def test_fused_rejects_other_shapes(cuda):
    x, sx, wq, sw, qw, kw = setup(64, 2, 1, False, 256, cuda, 9)
    cos, sin = rope_tables(64, 256, cuda)
    with pytest.raises(ValueError):
        w8.gemm_qkv_norm_rope(x, wq[:-256], sx, sw[:-256], cos, sin, qw, kw, 1e-6, 2, 1, 256)
