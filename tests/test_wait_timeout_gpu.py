"""A bounded device-side wait that runs out ends the kernel with an error status.

The stream-K GEMM splits ragged tiles between workers; the contributors of a split tile
wait, with a time limit, for the counter the tile's owner bumps once its partial sum
has landed.  Here the owner is told (w8_inject_stream_k_stall, a host-set flag) never to
bump it, with a 1 ms limit: the waiters give up, the kernel still ends, and
w8_device_status() reports W8_ERR_DEVICE_TIMEOUT.  Afterwards the context is still
usable: with the hook off, the same GEMM is exact again.  Nothing faults or hangs; the
wait that runs out is the same bounded wait every stream-K launch uses.
"""
import pytest
import torch

from gemma_npu_b200 import _lib

pytestmark = pytest.mark.gpu

M, N, K = 3658, 1536, 6144  # 90 tiles of 256 x 256 on 74 CTA pairs: a ragged wave, stream-K


def _gemm(a, w):
    c = torch.zeros((M, N), dtype=torch.int32, device=a.device)
    ws = torch.zeros(_lib.lib().w8_mm_i8_workspace_bytes(M, N, K) // 4, dtype=torch.int32, device=a.device)
    _lib.call("w8_mm_i8_ws", a.data_ptr(), K, w.data_ptr(), K, _lib.W8_B_NK, c.data_ptr(), N, M, N, K,
              ws.data_ptr(), ws.numel() * 4, torch.cuda.current_stream().cuda_stream or None)
    return c


def test_stream_k_wait_runs_out_and_reports_timeout(cuda):
    gen = torch.Generator(device=cuda).manual_seed(11)
    a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device=cuda, generator=gen)
    w = torch.randint(-128, 128, (N, K), dtype=torch.int8, device=cuda, generator=gen)
    want = torch._int_mm(a, w.t())
    assert _lib.lib().w8_device_status(1) == _lib.W8_OK
    try:
        _lib.call("w8_inject_stream_k_stall", 1, 1_000_000)  # owners never signal; 1 ms limit
        _gemm(a, w)
        assert _lib.last_schedule()["stream_k"]
        st = _lib.lib().w8_device_status(1)  # synchronises: the kernel ended
    finally:
        _lib.call("w8_inject_stream_k_stall", 0, 0)
    assert st == _lib.W8_ERR_DEVICE_TIMEOUT
    assert _lib.lib().w8_device_status(1) == _lib.W8_OK  # cleared
    got = _gemm(a, w)
    assert torch.equal(got, want)
    assert _lib.lib().w8_device_status(1) == _lib.W8_OK


def test_device_status_raises_timeout_in_python(cuda):
    gen = torch.Generator(device=cuda).manual_seed(12)
    a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device=cuda, generator=gen)
    w = torch.randint(-128, 128, (N, K), dtype=torch.int8, device=cuda, generator=gen)
    try:
        _lib.call("w8_inject_stream_k_stall", 1, 1_000_000)
        _gemm(a, w)
        with pytest.raises(_lib.W8DeviceTimeout):
            _lib.device_status()
    finally:
        _lib.call("w8_inject_stream_k_stall", 0, 0)
    assert _lib.device_status() == _lib.W8_OK
