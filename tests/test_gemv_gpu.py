"""Parity of the weight-only int8 GEMV and the fused LM head with the reference CPU path.

Tolerance: normwise max-rel <= 1e-2, i.e.
max|gpu - ref| <= 1e-2 * max|ref|, against gemma_npu.cpu_int8_linear
(torch._weight_int8pack_mm, gemma_npu.py:155-156) and Int8Head + softcap
(gemma_npu.py:170-172, pipeline.py:335-338).  The kernel holds the activation row as
16-bit fixed point (per 16-element piece) and sums exactly in int32, ATen accumulates in fp32, so bit equality is
not expected.
"""
import numpy as np
import pytest
import torch

import gemma_npu_b200 as w8
from oracle import cpu_int8, w8a8_numpy as ref

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2


def max_rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def bf16(bits, device):
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def test_golden_gemv(cuda, golden):
    w = golden("wquant")
    wq, s = torch.from_numpy(w["q"]).to(cuda), bf16(w["s"], cuda)
    for t in (1, 3):
        g = golden(f"gemv_t{t}")
        y = w8.int8_linear(bf16(g["x"], cuda), wq, s)
        assert max_rel(y.float().cpu().numpy(), ref.bf16_bits_to_f32(g["y"])) <= MAX_REL


def test_golden_head_softcap(cuda, golden):
    w, g = golden("wquant"), golden("head")
    logits = w8.lm_head_logits(bf16(g["h"], cuda), torch.from_numpy(w["q"]).to(cuda), bf16(w["s"], cuda),
                               float(g["cap"]))
    assert max_rel(logits.cpu().numpy(), g["logits"]) <= MAX_REL


# Every decode shape of BASELINE config 2 plus the K > 6144 team paths.
SHAPES = [(2560, 1536), (1536, 2048), (12288, 1536), (1536, 6144), (256, 1536), (1536, 256),
          (1024, 12288), (512, 16384), (1000, 48), (77, 4096), (333, 3072), (64, 8192),
          # the real E2B mix: double-wide MLP, head_dim-512 attention, q-only qkv
          (24576, 1536), (1536, 12288), (5120, 1536), (1536, 4096), (2048, 1536)]


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("t", [1, 2])
def test_gemv_matches_oracle(cuda, n, k, t):
    gen = torch.Generator().manual_seed(n * 3 + k)
    x = torch.randn(t, k, generator=gen).to(torch.bfloat16)
    wf = torch.randn(n, k, generator=gen) * 0.02
    q, s_f32, _, s = cpu_int8.weight_quant(wf)
    y = w8.int8_linear(x.to(cuda), q.to(cuda), s.to(cuda))
    exact = ref.int8_linear(x.view(torch.int16).numpy().view(np.uint16), q.numpy(),
                            s.view(torch.int16).numpy().view(np.uint16))
    assert max_rel(y.float().cpu().numpy(), exact) <= MAX_REL
    if t == 1:
        want = cpu_int8.int8_linear(x, q, s)  # the reference's CPU op itself
        assert max_rel(y.float().cpu().numpy(), want.float().numpy()) <= MAX_REL


def test_full_lm_head_262144(cuda):
    gen = torch.Generator(device=cuda).manual_seed(5)
    w = (torch.randn(262144, 1536, device=cuda, generator=gen) * 0.02).to(torch.bfloat16)
    wq, sw = w8.quant_rows(w)
    s = sw.to(torch.bfloat16)
    h = torch.randn(1536, device=cuda, generator=gen).to(torch.bfloat16)
    logits = w8.lm_head_logits(h, wq, s, 30.0)
    want = cpu_int8.lm_head_logits(h.cpu(), wq.cpu(), s.cpu(), 30.0)
    assert max_rel(logits.cpu().numpy(), want.numpy()) <= MAX_REL
    y = w8.int8_linear(h[None], wq, s)
    assert max_rel(y.float().cpu().numpy(), cpu_int8.int8_linear(h[None].cpu(), wq.cpu(), s.cpu()).float().numpy()) <= MAX_REL
    # The softcap is applied to the bf16 head output: same argmax as the unfused path.
    assert int(logits.argmax()) == int((torch.tanh(y[0].float() / 30.0) * 30.0).argmax())


@pytest.mark.parametrize("cap", [30.0, 0.0])
def test_lm_head_argmax_equals_torch_argmax(cuda, cap):
    """The greedy token folded inside the head GEMV equals torch.argmax of the same
    logits (gemma_npu.py:291), including the lowest-id rule on ties: rows 7 and 100 and
    200000 are copies of one row (equal logits)."""
    gen = torch.Generator(device=cuda).manual_seed(11)
    w = (torch.randn(262144, 1536, device=cuda, generator=gen) * 0.02).to(torch.bfloat16)
    h = torch.randn(1536, device=cuda, generator=gen).to(torch.bfloat16)
    wq, sw = w8.quant_rows(w)
    s = sw.to(torch.bfloat16)
    top = int(w8.lm_head_logits(h, wq, s, cap).argmax())
    for r in (7, 100, 200000):
        wq[r] = wq[top]
        s[r] = s[top]
    for _ in range(2):  # the key is cleared by every call
        logits, tok = w8.lm_head_logits(h, wq, s, cap, argmax=True)
        assert int(tok) == int(logits.argmax()) == 7
    # negated scales flip every logit's sign: the monotone key of negative floats
    logits, tok = w8.lm_head_logits(h, wq[:5000], s[:5000] * -1, cap, argmax=True)
    assert int(tok) == int(logits.argmax())

