"""The reference-facing linear surface on a B200: to_b200 (to_npu), B200Gemm (NPUGemm),
Slice, stage/launch_slot, gemm() requests and Int8Head, against the reference's
cpu-int8 path (oracle.cpu_int8) on a small decoder with the Gemma attribute layout."""
import numpy as np
import pytest
import torch

import gemma_npu_b200 as w8
from gemma_npu_b200 import gemm as g8
from oracle import cpu_int8

from fakes import fake_model

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2


def max_rel(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-30))


@pytest.fixture(scope="module")
def swapped(cuda):
    torch.manual_seed(0)
    m = fake_model(layers=2, d=256, inter=512, heads=(4, 1, 1), hd=64, ple=64).to(torch.bfloat16)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0, 0.02)
    lm = m.model.language_model
    before = [torch.cat([l.weight.detach().clone() for l in linears]) for _, _, linears in g8.layer_groups(lm)[0]]
    head_w = m.lm_head.weight.detach().clone()
    gemms = w8.to_b200(m, device=cuda)
    return m, gemms, before, head_w


def test_resident_weights_equal_reference_quant(swapped):
    _, gemms, before, _ = swapped
    for g, w in zip(gemms, before):
        q, sw, _, sw_bf16 = cpu_int8.weight_quant(w)
        assert torch.equal(g.w.cpu(), q)
        assert torch.equal(g.sw.cpu(), sw)
        assert torch.equal(g.sw_cpu.cpu(), sw_bf16)
        assert g.w_cpu is g.w and g.on_cpu is False


def test_matmul_prefill_bit_exact_and_decode_within_tolerance(swapped, cuda):
    _, gemms, before, _ = swapped
    gen = torch.Generator().manual_seed(1)
    for g, w in zip(gemms, before):
        q, sw, _, sw_bf16 = cpu_int8.weight_quant(w)
        x = torch.randn(40, g.K, generator=gen).to(torch.bfloat16)
        y = g.matmul(x.to(cuda))
        want = cpu_int8.linear_dequant(x, q, sw)  # NPUGemm.matmul on_cpu (gemma_npu.py:122-124)
        assert torch.equal(y.cpu().view(torch.int16), want.view(torch.int16)), g.name
        y1 = g.matmul(x[:3].to(cuda))  # T < 16: the decode GEMV
        assert max_rel(y1.float(), cpu_int8.int8_linear(x[:3], q, sw_bf16).float()) <= MAX_REL


def test_slices_fan_out_the_group(swapped, cuda):
    m, gemms, _, _ = swapped
    a = m.model.language_model.layers[0].self_attn
    x = torch.randn(2, 20, 256, device=cuda).to(torch.bfloat16)
    qv, kv, vv = a.q_proj(x), a.k_proj(x), a.v_proj(x)
    full = gemms[0].matmul(x.reshape(-1, 256))
    assert qv.shape == (2, 20, 256) and kv.shape == (2, 20, 64) and vv.shape == (2, 20, 64)
    assert torch.equal(torch.cat([qv, kv, vv], -1).reshape(40, -1), full)
    assert gemms[0].pending is None


def test_stage_and_launch_slot_exact(swapped, cuda):
    _, gemms, before, _ = swapped
    gen = torch.Generator().manual_seed(2)
    for slot, (g, w) in enumerate(zip(gemms[:6], before[:6])):
        q, _, w_kn, _ = cpu_int8.weight_quant(w)
        T = 100 + slot
        xq = torch.randint(-127, 128, (T, g.K), dtype=torch.int8, generator=gen)
        kind, thunk, name = g8.gemm(g, xq.to(cuda), None, slot % g8.N_SLOTS)
        assert kind == "npu" and name == g.name
        acc = thunk()
        assert acc.shape == (T, g.N)
        assert torch.equal(acc.cpu(), cpu_int8.int_mm(xq, w_kn))


def test_int8_head_and_softcap(swapped, cuda):
    m, _, _, head_w = swapped
    q, _, _, sw_bf16 = cpu_int8.weight_quant(head_w)
    assert torch.equal(m.lm_head.wq.cpu(), q)
    h = torch.randn(1, 1, 256).to(torch.bfloat16)
    y = m.lm_head(h.to(cuda))
    assert y.shape == (1, 1, 512)
    assert max_rel(y.float().reshape(-1), cpu_int8.int8_linear(h.reshape(1, -1), q, sw_bf16).float().reshape(-1)) <= MAX_REL
    logits = m.lm_head.logits(h.reshape(-1).to(cuda), cap=30.0)
    assert max_rel(logits, cpu_int8.lm_head_logits(h.reshape(-1), q, sw_bf16, 30.0)) <= MAX_REL


def test_device_status_clean(cuda):
    assert w8.device_status() == 0
