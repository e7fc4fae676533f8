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
