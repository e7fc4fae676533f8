"""ctypes binding of `libw8a8_b200.so`, the C ABI declared in include/w8a8_b200.h.

The library is built in-tree by `build.py`.  Loading it needs no GPU (the
symbols resolve on any Linux host); calling a compute entry point needs an
sm_100 device.  There is no fallback: if the library is missing, `lib()` raises.
"""
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libw8a8_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "w8a8_b200.h")

# Status codes (w8a8_b200.h).
W8_OK = 0
W8_ERR_INVALID_ARG = 1
W8_ERR_ALIGNMENT = 2
W8_ERR_UNSUPPORTED = 3
W8_ERR_CUDA = 4
W8_ERR_DEVICE_TIMEOUT = 5

# Layout codes of the GEMM B operand.
W8_B_KN = 0  # [K, N] row-major, as npu_kernels.mm_i8 takes it
W8_B_NK = 1  # [N, K] row-major (K-major), the resident layout


class W8Error(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, status, fn, detail):
        self.status = status
        super().__init__(f"{fn}: {detail} (status {status})")


class W8InvalidArgument(W8Error, ValueError):
    pass


class W8AlignmentError(W8Error, ValueError):
    pass


class W8Unsupported(W8Error):
    pass


class W8CudaError(W8Error):
    pass


class W8DeviceTimeout(W8Error):
    pass


_EXC = {
    W8_ERR_INVALID_ARG: W8InvalidArgument,
    W8_ERR_ALIGNMENT: W8AlignmentError,
    W8_ERR_UNSUPPORTED: W8Unsupported,
    W8_ERR_CUDA: W8CudaError,
    W8_ERR_DEVICE_TIMEOUT: W8DeviceTimeout,
}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i = ctypes.c_int
_f = ctypes.c_float

# name -> (restype, argtypes); one entry per function the header declares.
SIGNATURES = {
    "w8_status_string": (ctypes.c_char_p, [_i]),
    "w8_last_error": (ctypes.c_char_p, []),
    "w8_device_status": (_i, [_i]),
    "w8_abi_version": (_i, []),
    "w8_gemm_last_schedule": (_i, [ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "w8_inject_stream_k_stall": (_i, [_i, ctypes.c_uint64]),
    "w8_mm_i8": (_i, [_p, _i64, _p, _i64, _i, _p, _i64, _i64, _i64, _i64, _p]),
    "w8_mm_i8_ws": (_i, [_p, _i64, _p, _i64, _i, _p, _i64, _i64, _i64, _i64, _p, _i64, _p]),
    "w8_mm_i8_workspace_bytes": (_i64, [_i64, _i64, _i64]),
    "w8_mm_i8_noalloc": (_i, [_p, _i64, _p, _i64, _i, _p, _i64, _i64, _i64, _i64, _p]),
    "w8_gemm_dequant_bf16": (_i, [_p, _i64, _p, _i64, _i, _p, _p, _p, _i64, _i64, _i64, _i64, _p]),
    "w8_rms_quant_bf16": (_i, [_p, _i64, _p, ctypes.c_float, _p, _i64, _p, _i64, _i64, _p]),
    "w8_post_norm_quant_bf16": (_i, [_p, _i64, _p, _i64, _p, _p, ctypes.c_float, _p, _i64, _p, _i64, _p, _i64,
                                     _i64, _p]),
    "w8_ple_gate_quant_bf16": (_i, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _i64, _p]),
    "w8_ple_out_bf16": (_i, [_p, _i64, _p, _i64, _p, ctypes.c_float, _p, ctypes.c_float, _p, _i64, _p, _i64, _p,
                             _i64, _i64, _p]),
    "w8_qkv_norm_rope_bf16": (_i, [_p, _i64, _p, _p, _i64, _p, _p, ctypes.c_float, _p, _i64, _i64, _i64, _i64,
                                   _i64, _i64, _i, _p]),
    "w8_attention_prefill_bf16": (_i, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64,
                                       _i64, _i64, _i64, _i64, _p]),
    "w8_attention_prefill_mma_bf16": (_i, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64,
                                           _i64, _i64, _i64, _i64, _i64, _p]),
    "w8_attn_out_quant_bf16": (_i, [_p, _i64, _i64, _p, _i64, _p, _i64, _i64, _i64, _p]),
    "w8_attention_prefill_quant": (_i, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _i64,
                                        _i64, _p, _i64, _p, _p]),
    "w8_gemm_qkv_norm_rope": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _i, _p, _p, _i64, _p, _p, _f, _p,
                                   _i64, _i64, _i64, _p]),
    "w8_gemm_qkv_norm_rope_tiled": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _i, _p, _p, _i64, _p, _p, _f, _p,
                                   _i64, _i64, _i64, _p]),
    "w8_gemm_gelu_up_quant": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _p, _i64, _p, _p, _i64, _p, _p]),
    "w8_quant_rows_bf16": (_i, [_p, _i64, _p, _i64, _p, _i64, _i64, _p]),
    "w8_quant_rows_f32": (_i, [_p, _i64, _p, _i64, _p, _i64, _i64, _p]),
    "w8_dequant_bf16": (_i, [_p, _i64, _p, _p, _p, _i64, _i64, _i64, _p]),
    "w8_int8_linear_bf16": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _i64, _p]),
    "w8_lm_head_f32": (_i, [_p, _p, _p, _f, _p, _i64, _i64, _p]),
    "w8_lm_head_argmax_f32": (_i, [_p, _p, _p, _f, _p, _i64, _i64, _p, _p]),
}

SIGNATURES.update({
    "w8_lm_head_peer_bytes": (_i64, [_i64]),
    "w8_peer_alloc": (_i, [_i64, ctypes.POINTER(ctypes.c_void_p), _p]),
    "w8_peer_open": (_i, [_p, ctypes.POINTER(ctypes.c_void_p)]),
    "w8_peer_close": (_i, [_p]),
    "w8_peer_free": (_i, [_p]),
    "w8_lm_head_peer_f32": (_i, [_p, _p, _p, _f, _i64, _i64, _i64, _i64, _i, _i, ctypes.POINTER(ctypes.c_void_p), _p,
                                 _p]),
    "w8_lm_head_peer_argmax": (_i, [_p, _p, _p, _f, _i64, _i64, _i64, _i64, _i, _i, ctypes.POINTER(ctypes.c_void_p), _p,
                                 _p]),
})

_lock = threading.Lock()
_lib = None


def lib():
    """The loaded library (loaded once per process)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is not built; run `python gemma-npu_b200/build.py` "
                        "(or __graft_entry__.build()) -- there is no CPU fallback")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def check(status, fn):
    """Raise the W8Error subclass matching a non-zero status."""
    if status == W8_OK:
        return
    detail = lib().w8_last_error().decode(errors="replace") or lib().w8_status_string(status).decode()
    raise _EXC.get(status, W8Error)(status, fn, detail)


def call(name, *args):
    """Call a status-returning entry point and raise on failure."""
    check(getattr(lib(), name)(*args), name)


def last_schedule():
    """Schedule of the last GEMM this thread launched: dict(pair, stream_k, workers, tile_n)."""
    sk, workers, tile_n = _i(), _i(), _i()
    pair = lib().w8_gemm_last_schedule(ctypes.byref(sk), ctypes.byref(workers), ctypes.byref(tile_n))
    return {"pair": bool(pair), "stream_k": bool(sk.value), "workers": workers.value, "tile_n": tile_n.value}


def device_status(clear=True):
    """Sticky device-side status (syncs the device); raises W8DeviceTimeout if a wait gave up."""
    st = lib().w8_device_status(1 if clear else 0)
    if st == W8_ERR_DEVICE_TIMEOUT:
        raise W8DeviceTimeout(st, "device", "a bounded device-side wait timed out")
    check(st, "w8_device_status")
    return st
