"""B200 (sm_100a) W8A8 linear hot path of the Gemma E2B NPU pipeline.

Import with `importlib.import_module("gemma-npu_b200")`; after that the package
is also reachable as `gemma_npu_b200` (and its submodules as
`gemma_npu_b200.kernels`, ...), so ordinary `import` statements work.

Modules:
    kernels   mm_i8 / quant_rows / dequant / gemm_dequant / int8_linear / lm_head_logits /
              gelu_up_quant (k_gelu fused onto the gate/up GEMM) / pack_gelu_up
              over the C ABI (the reference's npu_kernels.py + quant glue)
    gemm      B200Gemm (NPUGemm), Slice, Int8Head, to_b200 (to_npu), gemm (Prefill.gemm)
    lm_head   ShardedInt8Head: column-sharded LM head with an NCCL all-gather
    npu_kernels  stand-in for the reference's top-level `npu_kernels` module (use_npu,
              mm_i8, BLOCK_*); npu_kernels.install() registers it under that name
    _lib      ctypes binding of libw8a8_b200.so (include/w8a8_b200.h)
    build     nvcc build of the library
"""
import sys as _sys

_sys.modules.setdefault("gemma_npu_b200", _sys.modules[__name__])

from . import _lib, build, kernels, gemm, lm_head, npu_kernels  # noqa: E402

for _m in (_lib, build, kernels, gemm, lm_head, npu_kernels):
    _sys.modules.setdefault("gemma_npu_b200." + _m.__name__.rsplit(".", 1)[-1], _m)

from .kernels import (  # noqa: E402,F401
    BLOCK_K, BLOCK_M, BLOCK_N, attention_prefill, attention_quant, attn_out_quant, dequant, gelu_up_quant, gemm_dequant, gemm_qkv_norm_rope, rope_tiles, int8_linear,
    lm_head_logits, mm_i8, mm_i8_nk, pack_gelu_up, ple_gate_quant, ple_out, post_norm_quant, qkv_norm_rope,
    quant_rows, rms_quant, use_device, use_npu)
from .gemm import (  # noqa: E402,F401
    BACKENDS, B200Gemm, Int8Head, NPUGemm, Slice, add_backend_argument, apply_backend, to_b200)
from .lm_head import ShardedInt8Head  # noqa: E402,F401
from ._lib import W8Error, device_status  # noqa: E402,F401

__all__ = ["mm_i8", "mm_i8_nk", "gemm_qkv_norm_rope", "rope_tiles", "gemm_dequant", "gelu_up_quant", "pack_gelu_up", "rms_quant", "post_norm_quant",
           "ple_gate_quant", "ple_out",
           "attn_out_quant", "attention_prefill", "attention_quant", "qkv_norm_rope", "quant_rows", "dequant",
           "int8_linear",
           "lm_head_logits", "use_device", "use_npu", "B200Gemm", "NPUGemm", "Slice", "Int8Head", "to_b200",
           "ShardedInt8Head", "BACKENDS", "add_backend_argument", "apply_backend", "W8Error",
           "device_status"]
