"""CPU oracle of the W8A8 linear hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, what the reference (AyaSakura-comp/gemma-npu)
computes on its W8A8 path, so that the CUDA kernels can be checked against it.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import it, and only as the checker or as the timed CPU baseline --
never as the product path, which has no CPU fallback.

    w8a8_numpy   independent numpy restatement (quant, int32 GEMM, dequant, GEMV,
                 softcap, weight quant), each function citing the reference line.
    cpu_int8     the reference's `--backend cpu-int8` path restated over the same
                 ATen CPU kernels it calls (torch._int_mm, torch._weight_int8pack_mm);
                 this is the CPU baseline that bench.py times.

Parity pinning: both are checked against golden vectors that
tests/golden/make_golden.py produced by importing the reference's own
pipeline.py / gemma_npu.py functions (tests/test_oracle.py).
"""
