"""Generate the golden vectors of the W8A8 path by running the REFERENCE's own code.

Imports `pipeline.py` and `gemma_npu.py` from a checkout of AyaSakura-comp/gemma-npu
(default: the REFERENCE environment variable, else ../reference next to the
repository) and records, on seeded inputs:

  quant     pipeline._quant (pipeline.py:49-52)            bf16 rows -> int8 + fp32 scale
  quant_c   gemma_npu._quant_rows (gemma_npu.py:37-42)     the torch.compile'd twin
  wquant    gemma_npu.Int8Head.__init__ (gemma_npu.py:164-167) = NPUGemm's weight quant (:68-69)
  int_mm    torch._int_mm as the cpu-int8 GEMM calls it (pipeline.py:237) and the exactness
            check of shape_bench.py:25-31 (randint(-128, 128) operands)
  deq       pipeline._deq (pipeline.py:55-57) and gemma_npu._dequant (gemma_npu.py:45-47)
  gemv      gemma_npu.cpu_int8_linear (gemma_npu.py:155-156), T = 1 and T = 3
  head      gemma_npu.Int8Head.forward + the softcap of pipeline.py:335-338
  gelu_up   pipeline.k_gelu (pipeline.py:102-107): dequant, gelu_tanh(gate) * up, int8 quant
  k_in, k_post_attn, k_post_ff, k_attn_out, k_qkv(_shared)
            the RMSNorm / residual / RoPE glue of pipeline.py:66-99, 110-114 (eager bodies)
  k_ple_gate, k_ple_out(_one)
            the per-layer-input glue of pipeline.py:117-127 (eager bodies)
  attn_sliding, attn_full
            pipeline.sliding_attention / full_attention (pipeline.py:139-180), q_start = 0

The weight of the GEMM, GEMV and head cases is the one stored in wquant.npz
(q [N,K] int8, s bf16 [N]); the GEMM's B operand is its transpose.  The outputs
are small .npz files beside this script; the tests read only those,
so neither the reference nor this script is needed where the tests run.

usage: python tests/golden/make_golden.py [REFERENCE_DIR]
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def bf16_bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main(ref_dir):
    sys.path.insert(0, ref_dir)
    import gemma_npu  # noqa: E402  (reference)
    import pipeline  # noqa: E402  (reference)

    torch.manual_seed(0)
    out = {}

    # ---- activation quant: N(0,1) rows as the pipeline's bf16 activations, plus edge rows
    x = torch.randn(48, 1536).to(torch.bfloat16)
    x[0] = 0                                            # all-zero row: scale floor 1e-8 / 127
    x[1] = torch.linspace(-3, 3, 1536).to(torch.bfloat16)
    x[2, :] = 1e-12                                     # tiny row below the scale floor
    x[3] = (torch.arange(1536) % 255 - 127).to(torch.bfloat16)  # exact-integer row (absmax 127)
    x[4] = torch.randn(1536).to(torch.bfloat16) * 3e4   # large magnitudes
    x[5, ::2] = 0.5
    x[5, 1::2] = -254.0                                  # ties at x/s = +-0.25 / -127
    q, s = pipeline._quant(x)
    out["quant"] = dict(x=bf16_bits(x), q=q.numpy(), s=s.numpy())
    try:
        qc, sc = gemma_npu._quant_rows(x)
        out["quant_c"] = dict(x=bf16_bits(x), q=qc.numpy(), s=sc.numpy())
    except Exception as e:  # torch.compile needs a working C++ toolchain
        print("skipping gemma_npu._quant_rows:", type(e).__name__, e)

    # ---- weight quant through the reference's Int8Head on an nn.Linear (N(0, 0.02), bf16)
    lin = torch.nn.Linear(1536, 384, bias=False)
    with torch.no_grad():
        lin.weight.normal_(0, 0.02)
        lin.weight[7] = 0
    lin = lin.to(torch.bfloat16)
    head = gemma_npu.Int8Head(lin)
    out["wquant"] = dict(w=bf16_bits(lin.weight.detach()), q=head.wq.numpy(), s=bf16_bits(head.sw))
    w32 = lin.weight.detach().float()
    sw32 = w32.abs().amax(dim=1).clamp(min=1e-8) / 127   # gemma_npu.py:68 (fp32 scales of NPUGemm)
    out["wquant"]["s_f32"] = sw32.numpy()

    # ---- int32 GEMM: quantised activations x quantised weights, and full-range random int8
    xq, sx = pipeline._quant(torch.randn(40, 1536).to(torch.bfloat16))
    wq = head.wq                                          # [N, K]
    w_kn = wq.t().contiguous()                            # the w_kn layout of gemma_npu.py:76
    acc = torch._int_mm(xq, w_kn)
    out["int_mm"] = dict(a=xq.numpy(), c=acc.numpy())  # b = wquant.q transposed
    a = torch.randint(-128, 128, (72, 256), dtype=torch.int8)
    b = torch.randint(-128, 128, (256, 160), dtype=torch.int8)
    out["int_mm_full"] = dict(a=a.numpy(), b=b.numpy(), c=torch._int_mm(a, b).numpy())
    assert torch.equal(torch._int_mm(a, b), a.int() @ b.int())

    # ---- dequant
    y = pipeline._deq(acc, sx, sw32)
    out["deq"] = dict(acc=acc.numpy(), sx=sx.numpy(), sw=sw32.numpy(), y=bf16_bits(y))
    try:
        yc = gemma_npu._dequant(acc, sx, sw32, torch.bfloat16)
        out["deq_c"] = dict(acc=acc.numpy(), sx=sx.numpy(), sw=sw32.numpy(), y=bf16_bits(yc))
    except Exception as e:
        print("skipping gemma_npu._dequant:", type(e).__name__, e)

    # ---- decode GEMV and LM head (+ softcap 30.0, Gemma's final_logit_softcapping)
    for t in (1, 3):
        xv = torch.randn(t, 1536).to(torch.bfloat16)
        yv = gemma_npu.cpu_int8_linear(xv, head.wq, head.sw)
        out[f"gemv_t{t}"] = dict(x=bf16_bits(xv), y=bf16_bits(yv))  # w, s = wquant.q, wquant.s
    h = torch.randn(1, 1, 1536).to(torch.bfloat16)
    logits = head(h)[0, -1].float()
    cap = 30.0
    logits = torch.tanh(logits / cap) * cap
    out["head"] = dict(h=bf16_bits(h.reshape(-1)), cap=np.float32(cap), logits=logits.numpy())

    # ---- gate/up epilogue glue (pipeline.py:102-107, k_gelu): dequant -> gelu_tanh(gate) * up
    # -> per-row int8 quant of the down projection's input.  k_gelu is torch.compile'd; its
    # eager function (the same Python body) is what runs here.
    k_gelu = getattr(pipeline.k_gelu, "_torchdynamo_orig_callable", pipeline.k_gelu)
    gi, gk, gt = 512, 256, 24
    gx, gsx = pipeline._quant(torch.randn(gt, gk).to(torch.bfloat16))
    gw = (torch.randn(2 * gi, gk) * 0.02).float()
    gsw = gw.abs().amax(dim=1).clamp(min=1e-8) / 127
    gwq = torch.round(gw / gsw[:, None]).clamp(-127, 127).to(torch.int8)
    gx[0] = 0                                             # zero row: the 1e-8 scale floor
    gacc = torch._int_mm(gx, gwq.t().contiguous())
    gq, gs = k_gelu(gacc, gsx, gsw, gi)
    out["gelu_up"] = dict(x=gx.numpy(), w=gwq.numpy(), acc=gacc.numpy(), sx=gsx.numpy(), sw=gsw.numpy(),
                          inter=np.int32(gi), q=gq.numpy(), s=gs.numpy())

    # ---- the norm / RoPE glue around the other GEMMs (pipeline.py:66-99, 110-114), eager
    def eager(f):
        return getattr(f, "_torchdynamo_orig_callable", f)

    eps = 1e-6
    nt, nn = 16, 512

    def norm_w(n):
        return (1.0 + 0.1 * torch.randn(n)).to(torch.bfloat16)

    def gemm_out(t, n, k=256):
        xq, sx_ = pipeline._quant(torch.randn(t, k).to(torch.bfloat16))
        wf = torch.randn(n, k) * 0.02
        sw_ = wf.abs().amax(dim=1).clamp(min=1e-8) / 127
        wq_ = torch.round(wf / sw_[:, None]).clamp(-127, 127).to(torch.int8)
        return torch._int_mm(xq, wq_.t().contiguous()), sx_, sw_

    hin = (torch.randn(nt, nn) * 2).to(torch.bfloat16)
    w_in = norm_w(nn)
    q_, s_ = eager(pipeline.k_in)(hin, w_in, eps)
    out["k_in"] = dict(h=bf16_bits(hin), w=bf16_bits(w_in), eps=np.float32(eps), q=q_.numpy(), s=s_.numpy())

    acc, sxa, swa = gemm_out(nt, nn)
    res = torch.randn(nt, nn).to(torch.bfloat16)
    w1, w2 = norm_w(nn), norm_w(nn)
    h_, q_, s_ = eager(pipeline.k_post_attn)(acc, sxa, swa, res, w1, w2, eps)
    out["k_post_attn"] = dict(acc=acc.numpy(), sx=sxa.numpy(), sw=swa.numpy(), res=bf16_bits(res), w1=bf16_bits(w1),
                              w2=bf16_bits(w2), eps=np.float32(eps), h=bf16_bits(h_), q=q_.numpy(), s=s_.numpy())
    h_, q_, s_ = eager(pipeline.k_post_ff)(acc, sxa, swa, res, w1, eps)
    out["k_post_ff"] = dict(acc=acc.numpy(), sx=sxa.numpy(), sw=swa.numpy(), res=bf16_bits(res), w1=bf16_bits(w1),
                            eps=np.float32(eps), h=bf16_bits(h_), q=q_.numpy(), s=s_.numpy())

    o = torch.randn(4, nt, 64).to(torch.bfloat16)
    q_, s_ = eager(pipeline.k_attn_out)(o)
    out["k_attn_out"] = dict(o=bf16_bits(o), q=q_.numpy(), s=s_.numpy())

    nh, kv, hd = 2, 1, 64
    acc, sxa, swa = gemm_out(nt, (nh + 2 * kv) * hd)
    ang = torch.arange(nt)[:, None].float() * (10000.0 ** (-torch.arange(0, hd, 2).float() / hd))[None]
    ang = torch.cat([ang, ang], dim=-1)
    cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    qw, kw = norm_w(hd), norm_w(hd)
    for shared in (False, True):
        qq, kk, vv = eager(pipeline.k_qkv)(acc, sxa, swa, cos, sin, qw, None if shared else kw, eps, nh, kv, hd, shared)
        out[f"k_qkv{'_shared' if shared else ''}"] = dict(
            acc=acc.numpy(), sx=sxa.numpy(), sw=swa.numpy(), cos=bf16_bits(cos), sin=bf16_bits(sin), qw=bf16_bits(qw),
            kw=bf16_bits(kw), eps=np.float32(eps), dims=np.array([nh, kv, hd, int(shared)], np.int32),
            q=bf16_bits(qq), k=bf16_bits(kk), v=bf16_bits(vv))

    # ---- prefill attention (pipeline.py:139-180), one prompt from position 0: sliding
    # window 512 (head_dim 256) and full causal (head_dim 512), 2 query heads on 1 KV head
    for name, (at, ad, win) in {"attn_sliding": (640, 256, 512), "attn_full": (200, 512, 0)}.items():
        aq = torch.randn(2, at, ad).to(torch.bfloat16)
        ak = torch.randn(1, at, ad).to(torch.bfloat16)
        av = torch.randn(1, at, ad).to(torch.bfloat16)
        scale = ad ** -0.25  # keep the logits O(1) at scale 1.0, as q_norm / k_norm do
        aq, ak = (aq.float() * scale).to(torch.bfloat16), (ak.float() * scale).to(torch.bfloat16)
        ao = pipeline.sliding_attention(aq, ak, av, 0, win) if win else pipeline.full_attention(aq, ak, av, 0)
        out[name] = dict(q=bf16_bits(aq), k=bf16_bits(ak), v=bf16_bits(av), window=np.int32(win), o=bf16_bits(ao))

    # ---- the per-layer-input glue (pipeline.py:117-127, k_ple_gate / k_ple_out), eager bodies:
    # the PLE gate GEMM output [T, 256] with this layer's per-layer input, and the projection
    # output [T, hidden] added into the residual stream and scaled by the layer scalar
    pn = 256
    acc, sxa, swa = gemm_out(nt, pn, k=nn)
    ple = torch.randn(nt, pn).to(torch.bfloat16)
    ple[0] = 0                                            # gated-off row: the 1e-8 scale floor
    q_, s_ = eager(pipeline.k_ple_gate)(acc, sxa, swa, ple)
    out["k_ple_gate"] = dict(acc=acc.numpy(), sx=sxa.numpy(), sw=swa.numpy(), ple=bf16_bits(ple), q=q_.numpy(),
                             s=s_.numpy())
    acc, sxa, swa = gemm_out(nt, nn, k=pn)
    res = torch.randn(nt, nn).to(torch.bfloat16)
    w1 = norm_w(nn)
    for tag, val in (("", 0.3), ("_one", 1.0)):
        scalar = torch.tensor([val]).to(torch.bfloat16)
        h_ = eager(pipeline.k_ple_out)(acc, sxa, swa, res, w1, scalar, eps)
        out[f"k_ple_out{tag}"] = dict(acc=acc.numpy(), sx=sxa.numpy(), sw=swa.numpy(), res=bf16_bits(res),
                                      w1=bf16_bits(w1), scalar=bf16_bits(scalar), eps=np.float32(eps),
                                      h=bf16_bits(h_))

    for name, arrays in out.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
        print("wrote", name, {k: getattr(v, "shape", ()) for k, v in arrays.items()})


if __name__ == "__main__":
    default = os.environ.get("REFERENCE", os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))),
                                                       "reference"))
    main(sys.argv[1] if len(sys.argv) > 1 else default)
