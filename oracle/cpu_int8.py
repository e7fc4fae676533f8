"""The reference's `--backend cpu-int8` W8A8 path, restated on torch CPU -- TEST INFRASTRUCTURE ONLY.

The reference runs this path when launched with `--backend cpu-int8`
(gemma_npu.py:254 -> to_npu(all_cpu=True)): every prefill GEMM is
`torch._int_mm(xq, w_kn)` (pipeline.py:235-239), quant/dequant are `_quant` /
`_deq` (pipeline.py:49-57), and decode plus the LM head are
`torch._weight_int8pack_mm` (gemma_npu.py:155-172).  The arithmetic lives in
ATen's CPU kernels, which are present wherever torch is, so this module calls
those same kernels with the reference's own operation order.  It is the
`cpu_baseline` / `--impl reference` arm of bench.py and a second oracle for
the tests; it is never called by the product path.
"""
import os

import torch


def set_threads(n=None):
    """Use all host cores (the reference sets torch.set_num_threads(--threads), gemma_npu.py:313)."""
    n = n or os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def quant(x):
    """pipeline.py:49-52 (_quant)."""
    x = x.float()
    s = x.abs().amax(dim=-1).clamp(min=1e-8) / 127
    return torch.round(x / s[:, None]).clamp(-127, 127).to(torch.int8), s


def deq(acc, sx, sw):
    """pipeline.py:55-57 (_deq)."""
    return (acc.float() * sx[:, None] * sw[None, :]).to(torch.bfloat16)


def weight_quant(w):
    """gemma_npu.py:62,68-69 (NPUGemm.__init__): per-output-channel int8 of a [N, K] weight.

    Returns (q [N,K] int8, sw fp32 [N], w_kn [K,N] int8 contiguous, sw bf16 [N]):
    the `w_cpu`, `sw`, `w_kn` and `sw_cpu` the reference keeps (gemma_npu.py:76-82).
    """
    w = w.detach().float()
    sw = w.abs().amax(dim=1).clamp(min=1e-8) / 127
    q = torch.round(w / sw[:, None]).clamp(-127, 127).to(torch.int8)
    return q.contiguous(), sw, q.t().contiguous(), sw.to(torch.bfloat16)


def int_mm(xq, w_kn):
    """pipeline.py:237: the cpu-int8 prefill GEMM, int8 [T,K] @ int8 [K,N] -> int32."""
    return torch._int_mm(xq, w_kn)


def _aligned(t):
    """A 64-byte-aligned contiguous tensor: ATen's CPU int8pack kernel faults on less
    (tensors wrapping numpy buffers, e.g. loaded from .npz, often are)."""
    t = t.contiguous()
    return t if t.data_ptr() % 64 == 0 else t.clone()


def int8_linear(x2d, wq, sw):
    """gemma_npu.py:155-156 (cpu_int8_linear)."""
    return torch._weight_int8pack_mm(_aligned(x2d.to(torch.bfloat16)), _aligned(wq), _aligned(sw))


def lm_head_logits(h, wq, sw, cap=None):
    """gemma_npu.py:170-172 (Int8Head.forward) on one row, then pipeline.py:335-338 (softcap)."""
    logits = int8_linear(h.reshape(1, -1), wq, sw)[0].float()
    if cap:
        logits = torch.tanh(logits / cap) * cap
    return logits


def linear_dequant(x, q, sw):
    """gemma_npu.py:122-124 (NPUGemm.matmul, on_cpu): quant -> _int_mm -> dequant, bf16 out."""
    xq, sx = quant(x)
    return deq(torch._int_mm(xq, q.t().contiguous()), sx, sw)
