"""numpy restatement of the reference's W8A8 arithmetic -- TEST INFRASTRUCTURE ONLY.

Each function cites the reference line (file:line within AyaSakura-comp/gemma-npu)
it restates.  Integer results are exact; fp32 steps are done in np.float32 with
the reference's operation order, so quant and dequant are bit-exact, while the
GEMV (whose CPU accumulation order is ATen's) is returned in float64 for a
tolerance check.
"""
import numpy as np

SCALE_FLOOR = np.float32(1e-8)
QMAX = np.float32(127)


def bf16_bits_to_f32(bits):
    """uint16 bf16 bit patterns -> float32 values (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x):
    """float32 -> uint16 bf16 bit patterns, round to nearest even (torch's .to(bfloat16))."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def quant_rows(x):
    """Per-row symmetric int8 quant (pipeline.py:49-52; gemma_npu.py:37-42).

    s = max(absmax(row), 1e-8) / 127 in fp32; q = clamp(round_half_even(x / s), -127, 127).
    `x` is float32 (bf16 inputs are upcast exactly first, as `x.float()` does).
    """
    x = np.asarray(x, dtype=np.float32)
    s = np.maximum(np.abs(x).max(axis=1), SCALE_FLOOR) / QMAX
    s = s.astype(np.float32)
    q = np.rint(x / s[:, None]).clip(-127, 127).astype(np.int8)
    return q, s


def weight_quant(w):
    """Per-output-channel weight quant of a [N, K] weight (gemma_npu.py:62,68-69; :164-167).

    Identical arithmetic to quant_rows on the rows of W taken in fp32.
    """
    return quant_rows(np.asarray(w, dtype=np.float32))


def int_mm(a, b):
    """int32 C = A @ B for int8 A [M,K], B [K,N] (npu_kernels.py:40-56; torch._int_mm at pipeline.py:237).

    Exact: products and sums in int64, which cannot overflow int32 for K < 2^17.
    """
    return (np.asarray(a, dtype=np.int64) @ np.asarray(b, dtype=np.int64)).astype(np.int32)


def dequant(acc, sx, sw):
    """bf16 bits of (float(acc) * sx[:,None]) * sw[None,:] (pipeline.py:55-57; gemma_npu.py:45-47)."""
    y = np.asarray(acc).astype(np.float32) * np.asarray(sx, np.float32)[:, None]
    y = y.astype(np.float32) * np.asarray(sw, np.float32)[None, :]
    return f32_to_bf16_bits(y.astype(np.float32))


def int8_linear(x_bf16_bits, wq, s_bf16_bits):
    """Weight-only int8 GEMV (gemma_npu.py:155-156 = torch._weight_int8pack_mm), in float64.

    y[t,n] = float(s[n]) * sum_k float(x[t,k]) * w[n,k].  The result is returned
    unrounded (float64) so callers compare the bf16 kernel output within a tolerance.
    """
    x = bf16_bits_to_f32(x_bf16_bits).astype(np.float64)
    w = np.asarray(wq, dtype=np.float64)
    s = bf16_bits_to_f32(s_bf16_bits).astype(np.float64)
    return (x @ w.T) * s[None, :]


def softcap(logits, cap):
    """cap * tanh(logits / cap) (pipeline.py:336-338); identity when cap is falsy."""
    logits = np.asarray(logits, dtype=np.float64)
    return np.tanh(logits / cap) * cap if cap else logits


GELU_BETA = np.float32(np.sqrt(2.0) * (2.0 / np.sqrt(np.pi)) * 0.5)  # sqrt(2 / pi)
GELU_KAPPA = np.float32(0.044715)


def gelu_tanh_bf16(g):
    """F.gelu(g, approximate="tanh") of bf16 values g (float32 in, bf16-rounded float32 out).

    0.5 * g * (1 + tanh(sqrt(2/pi) * (g + 0.044715 * g^3))) in fp32, rounded once to bf16,
    the operation order of ATen's CPU kernel for reduced-precision inputs.
    """
    g = np.asarray(g, dtype=np.float32)
    inner = GELU_BETA * (g + GELU_KAPPA * (g * g * g))
    out = np.float32(0.5) * g * (np.float32(1) + np.tanh(inner).astype(np.float32))
    return bf16_bits_to_f32(f32_to_bf16_bits(out.astype(np.float32)))


def gelu_up_quant(acc, sx, sw, inter):
    """The gate/up epilogue glue k_gelu (pipeline.py:102-107).

    y = _deq(acc, sx, sw) (bf16 [T, 2I]); a = bf16(gelu_tanh(y[:, :I]) * y[:, I:]);
    returns _quant(a): int8 [T, I] and fp32 scales [T].
    """
    y = bf16_bits_to_f32(dequant(acc, sx, sw))
    g, u = y[:, :inter], y[:, inter:]
    a = bf16_bits_to_f32(f32_to_bf16_bits((gelu_tanh_bf16(g) * u).astype(np.float32)))
    return quant_rows(a)


def bf16_round(x):
    """float32 values rounded to bf16 (RNE) and returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


def rms(x, w, eps):
    """_rms (pipeline.py:43-46): x * (mean(x^2) + eps)^-0.5 [* w], fp32 out, unrounded to bf16.

    The mean is accumulated in float64 and rounded to fp32 (ATen's fp32 sum order is not
    reproduced: the last bit of the mean may differ), then pow(., -0.5) = rsqrt in fp32.
    """
    x = np.asarray(x, dtype=np.float32)
    ms = (x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True).astype(np.float32)
    r = (1.0 / np.sqrt((ms + np.float32(eps)).astype(np.float64))).astype(np.float32)
    y = (x * r).astype(np.float32)
    return (y * np.asarray(w, dtype=np.float32)).astype(np.float32) if w is not None else y


def rope(x, cos, sin):
    """_rope (pipeline.py:60-63) on bf16 values: x * cos + rotate_half(x) * sin, each bf16 op
    rounded to bf16 as eager torch does."""
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return bf16_round(bf16_round(x * cos) + bf16_round(rot * sin))


def k_in(h, w, eps):
    """k_in (pipeline.py:66-69): _quant(bf16(_rms(h, w)))."""
    return quant_rows(bf16_round(rms(h, w, eps)))


def k_post(y, res, w1, w2, eps):
    """k_post_attn (pipeline.py:95-99; w2 given) and k_post_ff (pipeline.py:110-114; w2 None)
    after the dequant: h = bf16(res + bf16(_rms(y, w1))); q, s = _quant(bf16(_rms(h, w2)) or h)."""
    h = bf16_round(np.asarray(res, np.float32) + bf16_round(rms(y, w1, eps)))
    t = bf16_round(rms(h, w2, eps)) if w2 is not None else h
    q, s = quant_rows(t)
    return h, q, s


def k_ple_gate(y, ple):
    """k_ple_gate (pipeline.py:117-121) after the dequant, y = _deq(acc) as bf16 values:
    g = bf16(bf16(gelu_tanh(y)) * ple); returns _quant(g)."""
    g = bf16_round(gelu_tanh_bf16(y) * np.asarray(ple, np.float32))
    return quant_rows(g)


def k_ple_out(y, h, w, scalar, eps):
    """k_ple_out (pipeline.py:124-127) after the dequant: bf16(bf16(h + bf16(_rms(y, w))) * scalar),
    `scalar` the bf16 layer scalar as a float."""
    hh = bf16_round(np.asarray(h, np.float32) + bf16_round(rms(y, w, eps)))
    return bf16_round(hh * np.float32(scalar))


def k_attn_out(o):
    """k_attn_out (pipeline.py:88-92): o [H, T, D] -> _quant of the [T, H*D] rows."""
    o = np.asarray(o, np.float32)
    nh, t, d = o.shape
    return quant_rows(o.transpose(1, 0, 2).reshape(t, nh * d))


def k_qkv(acc, sx, sw, cos, sin, qw, kw, eps, nh, kv, d, shared):
    """k_qkv (pipeline.py:72-86): dequant, per-head _rms with q_norm / k_norm (v: no
    weight), RoPE on q and k; returns q [H, T, D], k, v [KV, T, D] as bf16 values."""
    y = bf16_bits_to_f32(dequant(acc, sx, sw))
    t = y.shape[0]
    cos, sin = np.asarray(cos, np.float32)[:, None], np.asarray(sin, np.float32)[:, None]
    q = rope(bf16_round(rms(y[:, : nh * d].reshape(t, nh, d), qw, eps)), cos, sin).transpose(1, 0, 2)
    if shared:
        return q, q, q
    k = y[:, nh * d: (nh + kv) * d].reshape(t, kv, d)
    v = y[:, (nh + kv) * d:].reshape(t, kv, d)
    k = rope(bf16_round(rms(k, kw, eps)), cos, sin).transpose(1, 0, 2)
    v = bf16_round(rms(v, None, eps)).transpose(1, 0, 2)
    return q, k, v


def attention(q, k, v, window=0):
    """Prefill attention of one prompt (pipeline.py:139-180 with q_start = 0): scale 1.0,
    causal, and with window W > 0 each query sees only the W keys up to itself
    (sliding_attention's mask: key <= query, query - key < W).  q [H, T, D], k, v [KV, T, D]
    (grouped-query: head h reads KV head h // (H / KV)); float64 softmax, unrounded result."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    nh, t, _ = q.shape
    group = nh // k.shape[0]
    pos = np.arange(t)
    allowed = pos[None, :] <= pos[:, None]
    if window:
        allowed &= (pos[:, None] - pos[None, :]) < window
    out = np.empty_like(q)
    for h in range(nh):
        s = q[h] @ k[h // group].T
        s = np.where(allowed, s, -np.inf)
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        out[h] = (p / p.sum(axis=1, keepdims=True)) @ v[h // group]
    return out
