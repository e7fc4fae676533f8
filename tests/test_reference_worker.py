"""The reference's own scheduler plumbing runs unchanged over this library (no GPU).

The reference's worker thread starts with `import npu_kernels; npu_kernels.use_npu()`
(pipeline.py:203-204) and then runs the thunks `Prefill.gemm` returns (pipeline.py:233-242,
206-216).  Here the reference's real `pipeline.Worker` and `Prefill.gemm` are imported
from a checkout of the reference (skipped when none is present: REFERENCE, else
../reference next to this repository), `npu_kernels` is this library's stand-in, and
the groups are host_io B200Gemm objects.  Without a GPU the device-side pieces are
replaced by recorders: device selection records the thread that asked, and the GEMM
launch is `torch._int_mm` on the host rows (a fake device).  What is checked is the
plumbing the reference relies on: the import, use_npu on the worker thread, stage() rows
reaching launch_slot(), the int32 result coming back through the reference's Job, and
exceptions forwarded to the waiter.  The GPU test of the same flow with real kernels is
tests/test_host_io_gpu.py.
"""
import importlib
import os
import sys
import threading
import types

import pytest
import torch

import gemma_npu_b200 as w8
from gemma_npu_b200 import gemm as g8
from gemma_npu_b200 import kernels
from gemma_npu_b200 import npu_kernels as nk

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))


@pytest.fixture()
def reference_pipeline(monkeypatch):
    if not os.path.exists(os.path.join(REF, "pipeline.py")):
        pytest.skip("no reference checkout")
    monkeypatch.syspath_prepend(REF)
    saved = sys.modules.get("npu_kernels")
    try:
        pipeline = importlib.import_module("pipeline")
    except Exception as e:  # noqa: BLE001 -- an incomplete environment for the reference
        pytest.skip(f"reference pipeline does not import here: {e}")
    yield pipeline
    if saved is None:
        sys.modules.pop("npu_kernels", None)
    else:
        sys.modules["npu_kernels"] = saved


def _host_gemm(n, k, seed):
    """A host_io B200Gemm built without a GPU: host slots, int8 weight rows [N, K]."""
    g = object.__new__(g8.B200Gemm)
    gen = torch.Generator().manual_seed(seed)
    g.w = torch.randint(-127, 128, (n, k), dtype=torch.int8, generator=gen)
    g.N, g.K, g.n_pad, g.name, g.host_io, g.on_cpu = n, k, -(-n // 16) * 16, f"g{seed}", True, False
    g.device = torch.device("cpu")
    return g


def test_reference_worker_runs_b200_thunks(reference_pipeline, monkeypatch):
    pipeline = reference_pipeline
    asked = []
    monkeypatch.setattr(kernels, "use_device", lambda dev: asked.append((threading.current_thread().name, dev)))
    # fake device: the launch is an int32 product of the host rows; the stream sync a no-op
    monkeypatch.setattr(kernels, "mm_i8_nk", lambda a, w, c: c.copy_(torch._int_mm(a, w.t())))
    monkeypatch.setattr(torch.cuda, "current_stream", lambda dev=None: types.SimpleNamespace(synchronize=lambda: None))
    nk.install(device=0)
    assert sys.modules["npu_kernels"] is nk

    slots = 2
    monkeypatch.setattr(g8.B200Gemm, "slots", [(torch.empty(g8.SLOT_ROWS * 512, dtype=torch.int8),
                                                 torch.empty(g8.SLOT_ROWS * 512, dtype=torch.int32))
                                                for _ in range(slots)])
    monkeypatch.setattr(g8.B200Gemm, "host_slots", [(torch.empty(g8.SLOT_ROWS * 512, dtype=torch.int8),
                                                      torch.empty(g8.SLOT_ROWS * 512, dtype=torch.int32))
                                                     for _ in range(slots)])
    worker = pipeline.Worker()
    prefill = object.__new__(pipeline.Prefill)  # Prefill.gemm reads nothing but its arguments
    gen = torch.Generator().manual_seed(3)
    for i, (n, k, T) in enumerate([(96, 64, 40), (200, 128, 7), (48, 256, 512)]):
        g = _host_gemm(n, k, i)
        xq = torch.randint(-127, 128, (T, k), dtype=torch.int8, generator=gen)
        kind, fn, name = pipeline.Prefill.gemm(prefill, g, xq, None, i % slots)
        assert (kind, name) == ("npu", g.name)
        job = worker.submit(fn, 0, name)
        with worker.done:
            while not job.done:
                worker.done.wait(10)
        assert not isinstance(job.value, BaseException), job.value
        assert job.value.device.type == "cpu" and job.value.shape == (T, n)
        assert torch.equal(job.value, torch._int_mm(xq, g.w.t()))
    assert len(asked) == 1 and asked[0][0] == worker.t.name and asked[0][1] == torch.device("cuda", 0)

    def boom():
        raise w8.W8Error(1, "w8_mm_i8_ws", "bad shape")

    job = worker.submit(boom, 0, "boom")  # forwarded to the waiter (pipeline.py:212-216)
    with worker.done:
        while not job.done:
            worker.done.wait(10)
    assert isinstance(job.value, w8.W8Error)


def test_npu_kernels_surface():
    for name in ("use_npu", "mm_i8", "BLOCK_M", "BLOCK_N", "BLOCK_K", "install"):
        assert hasattr(nk, name), name
    assert nk.BLOCK_K % 16 == 0
    assert w8.use_npu is kernels.use_device
