"""Pin the CPU oracle against the golden vectors made by the reference's own functions.

The golden vectors (tests/golden/*.npz) were produced by tests/golden/make_golden.py
calling pipeline._quant/_deq, gemma_npu.Int8Head/cpu_int8_linear and torch._int_mm
exactly as the reference does.  Both oracle restatements must reproduce them:
bit-exactly for quant, weight quant, the int32 GEMM and dequant; within the stated
tolerance for the GEMV and the softcapped head, whose fp32 accumulation order is
ATen's.
"""
import numpy as np
import torch

from oracle import cpu_int8, w8a8_numpy as ref

# Float tolerance of the GEMV / head: normwise max-rel <= 1e-2,
# i.e. max|a - b| <= 1e-2 * max|b|.
MAX_REL = 1e-2


def max_rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _bf16(bits):
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def test_quant_numpy_bit_exact(golden):
    g = golden("quant")
    q, s = ref.quant_rows(ref.bf16_bits_to_f32(g["x"]))
    np.testing.assert_array_equal(s.view(np.uint32), g["s"].view(np.uint32))
    np.testing.assert_array_equal(q, g["q"])


def test_quant_edge_rows(golden):
    g = golden("quant")
    # all-zero row: scale is the floor 1e-8/127 and every q is 0
    assert g["s"][0] == np.float32(np.float32(1e-8) / np.float32(127))
    assert not g["q"][0].any()
    # an exact-integer row with absmax 127 quantises to itself
    np.testing.assert_array_equal(g["q"][3], ref.bf16_bits_to_f32(g["x"][3]).astype(np.int8))
    # clamp range is [-127, 127] (never -128)
    assert g["q"].min() >= -127 and g["q"].max() <= 127


def test_quant_torch_restatement_bit_exact(golden):
    g = golden("quant")
    q, s = cpu_int8.quant(_bf16(g["x"]))
    np.testing.assert_array_equal(q.numpy(), g["q"])
    np.testing.assert_array_equal(s.numpy().view(np.uint32), g["s"].view(np.uint32))


def test_weight_quant_bit_exact(golden):
    g = golden("wquant")
    q, s = ref.weight_quant(ref.bf16_bits_to_f32(g["w"]))
    np.testing.assert_array_equal(q, g["q"])
    np.testing.assert_array_equal(s.view(np.uint32), g["s_f32"].view(np.uint32))
    np.testing.assert_array_equal(ref.f32_to_bf16_bits(s), g["s"])
    q2, s2, w_kn, s_bf16 = cpu_int8.weight_quant(_bf16(g["w"]))
    np.testing.assert_array_equal(q2.numpy(), g["q"])
    np.testing.assert_array_equal(w_kn.numpy(), g["q"].T)
    np.testing.assert_array_equal(s_bf16.view(torch.int16).numpy().view(np.uint16), g["s"])


def test_int_mm_exact(golden):
    g, w = golden("int_mm"), golden("wquant")
    np.testing.assert_array_equal(ref.int_mm(g["a"], w["q"].T), g["c"])
    full = golden("int_mm_full")
    np.testing.assert_array_equal(ref.int_mm(full["a"], full["b"]), full["c"])
    assert full["a"].min() == -128  # the full int8 range, as shape_bench.py draws it


def test_dequant_bit_exact(golden):
    g = golden("deq")
    np.testing.assert_array_equal(ref.dequant(g["acc"], g["sx"], g["sw"]), g["y"])
    y = cpu_int8.deq(torch.from_numpy(g["acc"]), torch.from_numpy(g["sx"]), torch.from_numpy(g["sw"]))
    np.testing.assert_array_equal(y.view(torch.int16).numpy().view(np.uint16), g["y"])


def test_gemv_within_tolerance(golden):
    w = golden("wquant")
    for t in (1, 3):
        g = golden(f"gemv_t{t}")
        y = ref.int8_linear(g["x"], w["q"], w["s"])
        assert max_rel(ref.bf16_bits_to_f32(g["y"]), y) <= MAX_REL


def test_head_softcap_within_tolerance(golden):
    w, g = golden("wquant"), golden("head")
    y = ref.int8_linear(g["h"][None], w["q"], w["s"])[0]
    y = ref.bf16_bits_to_f32(ref.f32_to_bf16_bits(y.astype(np.float32)))
    assert max_rel(ref.softcap(y, float(g["cap"])), g["logits"]) <= MAX_REL
    out = cpu_int8.lm_head_logits(_bf16(g["h"]), torch.from_numpy(w["q"]), _bf16(w["s"]), float(g["cap"]))
    np.testing.assert_allclose(out.numpy(), g["logits"], rtol=0, atol=1e-5)


def test_bf16_round_trip():
    x = np.array([1.0, -2.5, 3.14159, 1e-30, 65504.0, np.float32(1.00390625)], dtype=np.float32)
    t = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(ref.f32_to_bf16_bits(x), t)


def test_gelu_up_quant_bit_exact(golden):
    """k_gelu (pipeline.py:102-107): dequant, gelu_tanh(gate) * up, int8 quant."""
    g = golden("gelu_up")
    np.testing.assert_array_equal(ref.int_mm(g["x"], g["w"].T), g["acc"])
    q, s = ref.gelu_up_quant(g["acc"], g["sx"], g["sw"], int(g["inter"]))
    np.testing.assert_array_equal(q, g["q"])
    np.testing.assert_array_equal(s, g["s"])


# The norm glue reduces mean(x^2) in fp32 in ATen's order (and takes pow(., -0.5) as
# ATen's rsqrt); the oracle rounds an fp64 mean.  The last bit of the mean may differ,
# so a bf16 output may move by one bf16 step and an int8 code by one.
def _close_bf16(a_bits, b_bits, frac=1e-2):
    a, b = ref.bf16_bits_to_f32(a_bits), ref.bf16_bits_to_f32(b_bits)
    d = np.abs(a - b)
    assert np.all(d <= np.abs(b) * 2.0 ** -7 + 1e-30)
    assert (d != 0).mean() <= frac


def _close_q(q, q_ref, frac=1e-2):
    d = np.abs(q.astype(np.int32) - q_ref.astype(np.int32))
    assert d.max() <= 1 and (d != 0).mean() <= frac


def test_k_in(golden):
    g = golden("k_in")
    q, s = ref.k_in(ref.bf16_bits_to_f32(g["h"]), ref.bf16_bits_to_f32(g["w"]), float(g["eps"]))
    _close_q(q, g["q"])
    np.testing.assert_allclose(s, g["s"], rtol=2.0 ** -7)


def test_k_post_attn_and_ff(golden):
    for name in ("k_post_attn", "k_post_ff"):
        g = golden(name)
        y = ref.bf16_bits_to_f32(ref.dequant(g["acc"], g["sx"], g["sw"]))
        w2 = ref.bf16_bits_to_f32(g["w2"]) if "w2" in g else None
        h, q, s = ref.k_post(y, ref.bf16_bits_to_f32(g["res"]), ref.bf16_bits_to_f32(g["w1"]), w2, float(g["eps"]))
        _close_bf16(ref.f32_to_bf16_bits(h), g["h"])
        _close_q(q, g["q"])
        np.testing.assert_allclose(s, g["s"], rtol=2.0 ** -7)


def test_k_ple_gate_bit_exact(golden):
    """k_ple_gate (pipeline.py:117-121): dequant, bf16(gelu_tanh(y)) * ple, int8 quant."""
    g = golden("k_ple_gate")
    y = ref.bf16_bits_to_f32(ref.dequant(g["acc"], g["sx"], g["sw"]))
    q, s = ref.k_ple_gate(y, ref.bf16_bits_to_f32(g["ple"]))
    np.testing.assert_array_equal(q, g["q"])
    np.testing.assert_array_equal(s, g["s"])


def test_k_ple_out(golden):
    """k_ple_out (pipeline.py:124-127), with a layer scalar of 0.3 and of exactly 1."""
    for name in ("k_ple_out", "k_ple_out_one"):
        g = golden(name)
        y = ref.bf16_bits_to_f32(ref.dequant(g["acc"], g["sx"], g["sw"]))
        scalar = float(ref.bf16_bits_to_f32(g["scalar"])[0])
        h = ref.k_ple_out(y, ref.bf16_bits_to_f32(g["res"]), ref.bf16_bits_to_f32(g["w1"]), scalar,
                          float(g["eps"]))
        _close_bf16(ref.f32_to_bf16_bits(h), g["h"])


def test_k_attn_out_bit_exact(golden):
    g = golden("k_attn_out")
    q, s = ref.k_attn_out(ref.bf16_bits_to_f32(g["o"]))
    np.testing.assert_array_equal(q, g["q"])
    np.testing.assert_array_equal(s, g["s"])


def test_k_qkv(golden):
    for name in ("k_qkv", "k_qkv_shared"):
        g = golden(name)
        nh, kv, d, shared = (int(v) for v in g["dims"])
        f = ref.bf16_bits_to_f32
        q, k, v = ref.k_qkv(g["acc"], g["sx"], g["sw"], f(g["cos"]), f(g["sin"]), f(g["qw"]),
                            None if shared else f(g["kw"]), float(g["eps"]), nh, kv, d, bool(shared))
        for mine, theirs in ((q, g["q"]), (k, g["k"]), (v, g["v"])):
            _close_bf16(ref.f32_to_bf16_bits(mine), theirs)
