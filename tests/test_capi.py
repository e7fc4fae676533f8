"""The C-ABI library: it loads, exports every entry point the header declares, and its
host-side argument checks answer with status codes -- all without a GPU."""
import ctypes
import os
import re

import pytest
import torch

import gemma_npu_b200 as w8
from gemma_npu_b200 import _lib


def declared_functions():
    text = open(_lib.HEADER_PATH).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int64_t|int|const char\s*\*)\s*(w8_\w+)\s*\(", text, flags=re.M)))


def test_library_builds_and_loads():
    if not os.path.exists(_lib.LIB_PATH):
        w8.build.build(quiet=True)
    assert _lib.lib() is not None


def test_every_declared_symbol_is_exported():
    names = declared_functions()
    assert len(names) >= 13, names
    handle = ctypes.CDLL(_lib.LIB_PATH)
    for name in names:
        assert hasattr(handle, name), f"{name} is declared in w8a8_b200.h but not exported"


def test_binding_covers_the_header():
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_status_strings_and_version():
    lib = _lib.lib()
    for code in range(0, 6):
        assert lib.w8_status_string(code)
    assert lib.w8_abi_version() >> 16 == 1


def test_host_side_argument_checks_need_no_gpu():
    lib = _lib.lib()
    # negative size
    assert lib.w8_mm_i8(None, 16, None, 16, _lib.W8_B_NK, None, 16, -1, 16, 16, None) == _lib.W8_ERR_INVALID_ARG
    # unknown B layout
    assert lib.w8_mm_i8(None, 16, None, 16, 7, None, 16, 4, 4, 16, None) == _lib.W8_ERR_INVALID_ARG
    assert b"b_layout" in lib.w8_last_error()
    # empty problems are no-ops
    assert lib.w8_mm_i8(None, 16, None, 16, _lib.W8_B_NK, None, 16, 0, 16, 16, None) == _lib.W8_OK
    assert lib.w8_int8_linear_bf16(None, 16, None, 16, None, None, 16, 0, 16, 16, None) == _lib.W8_OK
    # null operands with real sizes
    assert lib.w8_gemm_dequant_bf16(None, 16, None, 16, _lib.W8_B_NK, None, None, None, 16, 4, 4, 16,
                                    None) == _lib.W8_ERR_INVALID_ARG
    assert lib.w8_quant_rows_bf16(None, 16, None, 16, None, 4, 16, None) == _lib.W8_ERR_INVALID_ARG
    assert lib.w8_dequant_bf16(None, 16, None, None, None, 16, 4, 16, None) == _lib.W8_ERR_INVALID_ARG
    assert lib.w8_lm_head_f32(None, None, None, 30.0, None, 8, 16, None) == _lib.W8_ERR_INVALID_ARG
    # gate/up glue: I must be a multiple of 128; the absmax scratch is required
    assert lib.w8_gemm_gelu_up_quant(None, 16, None, 16, None, None, 4, 100, 16, None, 128, None, None, 128,
                                     None, None) == _lib.W8_ERR_INVALID_ARG
    assert b"inter" in lib.w8_last_error()
    assert lib.w8_gemm_gelu_up_quant(None, 16, None, 16, None, None, 0, 128, 16, None, 128, None, None, 128,
                                     None, None) == _lib.W8_OK


def test_status_maps_to_exceptions():
    with pytest.raises(_lib.W8InvalidArgument):
        _lib.call("w8_mm_i8", None, 16, None, 16, 7, None, 16, 4, 4, 16, None)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_compute_without_gpu_fails_loudly():
    # Valid-looking arguments on a host without a device: an error status, never a CPU result.
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.addressof(buf)
    p16 = (p + 15) // 16 * 16
    st = _lib.lib().w8_quant_rows_f32(p16, 16, p16 + 1024, 16, p16 + 2048, 1, 16, None)
    assert st in (_lib.W8_ERR_CUDA, _lib.W8_ERR_UNSUPPORTED)
