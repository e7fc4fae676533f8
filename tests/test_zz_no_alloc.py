"""w8_mm_i8_noalloc, the GEMM entry point for callers that cannot allocate device memory.

Some callers of this library may not call cudaMalloc on their path (a plugin inside
another framework's execute callback that owns the device-memory budget, a serving loop
that must not synchronise the device).  This entry point takes only inputs and outputs:
its stream-K tile counters live in a static device array inside the library.  Its int32
result must equal, bit for bit (the tolerance of every int32 test here), torch._int_mm
(cuBLASLt, an independent implementation) and the workspace entry point w8_mm_i8_ws on
the same inputs, on two calls in a row that share the static array; the schedule must
really be stream-K (so the static counters are used), and oversized or invalid problems
must be rejected before anything is launched or cleared.

This file sorts last so that a run stopping at the first failure has run every other test.
"""
import pytest
import torch

from gemma_npu_b200 import _lib

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream or None


def with_workspace(a, w, k):
    m, n = a.shape[0], w.shape[0]
    c = torch.empty((m, n), dtype=torch.int32, device=a.device)
    ws = torch.zeros(_lib.lib().w8_mm_i8_workspace_bytes(m, n, k) // 4, dtype=torch.int32, device=a.device)
    _lib.call("w8_mm_i8_ws", a.data_ptr(), k, w.data_ptr(), k, _lib.W8_B_NK, c.data_ptr(), n, m, n, k,
              ws.data_ptr(), ws.numel() * 4, _stream())
    return c


def no_alloc(a, w, k):
    m, n = a.shape[0], w.shape[0]
    c = torch.full((m, n), -1, dtype=torch.int32, device=a.device)
    _lib.call("w8_mm_i8_noalloc", a.data_ptr(), k, w.data_ptr(), k, _lib.W8_B_NK, c.data_ptr(), n, m, n, k,
              _stream())
    return c


# Shapes whose schedule uses the counters (stream-K: ragged waves with long K), on the
# CTA-pair kernel (M > 128) and on the single-CTA kernel (M <= 128).
@pytest.mark.parametrize("m,n,k", [(3658, 1536, 6144), (100, 1536, 6144), (207, 2560, 4096)])
def test_no_alloc_matches_workspace_entry_point_twice(cuda, m, n, k):
    gen = torch.Generator(device=cuda).manual_seed(m + n + k)
    for call in range(2):  # two calls in a row share the static counters
        a = torch.randint(-128, 128, (m, k), dtype=torch.int8, device=cuda, generator=gen)
        w = torch.randint(-128, 128, (n, k), dtype=torch.int8, device=cuda, generator=gen)
        got = no_alloc(a, w, k)
        sched = _lib.last_schedule()
        assert sched["stream_k"], f"call {call}: {sched} (the static counters went unused)"
        want = with_workspace(a, w, k)
        ref = torch._int_mm(a, w.t())
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {call}: differs from torch._int_mm"
        assert torch.equal(got, want), f"call {call}: differs from w8_mm_i8_ws"
    assert _lib.lib().w8_device_status(1) == _lib.W8_OK


def test_no_alloc_rejects_more_tiles_than_its_scratch_holds(cuda):
    m, n, k = 4096 + 1, 131072, 16  # ceil(4097/128) * 512 = 16896 > 16384 counters
    st = _lib.lib().w8_mm_i8_noalloc(None, k, None, k, _lib.W8_B_NK, None, n, m, n, k, _stream())
    assert st == _lib.W8_ERR_INVALID_ARG
    assert b"static scratch" in _lib.lib().w8_last_error()


def test_no_alloc_rejects_bad_arguments_without_launching(cuda):
    m, n, k = 3658, 1536, 6144
    a = torch.zeros((m, k), dtype=torch.int8, device=cuda)
    w = torch.zeros((n, k), dtype=torch.int8, device=cuda)
    c = torch.zeros((m, n), dtype=torch.int32, device=cuda)
    # k not a multiple of 16, then an unknown layout code: rejected by the argument checks,
    # which run before the shared counters are cleared
    st = _lib.lib().w8_mm_i8_noalloc(a.data_ptr(), k, w.data_ptr(), k, _lib.W8_B_NK, c.data_ptr(), n, m, n, k - 8,
                                     _stream())
    assert st == _lib.W8_ERR_INVALID_ARG
    st = _lib.lib().w8_mm_i8_noalloc(a.data_ptr(), k, w.data_ptr(), k, 7, c.data_ptr(), n, m, n, k, _stream())
    assert st == _lib.W8_ERR_INVALID_ARG
    # and the next valid call is still exact
    gen = torch.Generator(device=cuda).manual_seed(5)
    a = torch.randint(-128, 128, (m, k), dtype=torch.int8, device=cuda, generator=gen)
    w = torch.randint(-128, 128, (n, k), dtype=torch.int8, device=cuda, generator=gen)
    got = no_alloc(a, w, k)
    assert torch.equal(got, torch._int_mm(a, w.t()))
