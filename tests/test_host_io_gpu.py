"""The reference's unchanged CPU pipeline over the B200 GEMMs (host_io slots), on a GPU.

pipeline.py keeps its glue on the CPU (torch.compile'd `k_*`, pipeline.py:66-127), so a
drop-in for it must hand back host int32 results, as the reference's host-visible NPU
buffers do.  This test restates the two pieces of the reference that touch the GEMMs --
the worker thread (pipeline.py:196-216: `import npu_kernels; npu_kernels.use_npu()`, then
run each thunk) and Prefill.gemm (pipeline.py:233-242: fill `g.stage(slot, T)`, return
`("npu", lambda: g.launch_slot(T, slot), g.name)`) -- over `to_b200(model,
host_io=True)`, with this library's `npu_kernels` stand-in installed under the
reference's module name.  Results are checked bit for bit against the reference's
cpu-int8 path (torch._int_mm on the host, pipeline.py:237).
"""
import queue
import sys
import threading

import pytest
import torch

import gemma_npu_b200 as w8
from gemma_npu_b200 import gemm as g8
from gemma_npu_b200 import npu_kernels as nk
from oracle import cpu_int8

from fakes import fake_model

pytestmark = pytest.mark.gpu


class RefWorker:
    """pipeline.Worker's thread body (pipeline.py:202-216), restated."""

    def __init__(self):
        self.q = queue.Queue()
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        import npu_kernels
        npu_kernels.use_npu()
        while True:
            fn, out = self.q.get()
            if fn is None:
                return
            try:
                value = fn()
            except BaseException as e:  # noqa: BLE001 -- handed to the waiter
                value = e
            out.put(value)

    def run(self, fn):
        out = queue.Queue()
        self.q.put((fn, out))
        return out.get(timeout=60)


def ref_prefill_gemm(g, xq, sx, slot):
    """pipeline.Prefill.gemm's NPU branch (pipeline.py:240-242), restated."""
    T = xq.shape[0]
    g.stage(slot, T).copy_(xq)
    return ("npu", lambda: g.launch_slot(T, slot), g.name)


@pytest.fixture(scope="module")
def host_model(cuda):
    torch.manual_seed(0)
    m = fake_model(layers=2, d=256, inter=512, heads=(4, 1, 1), hd=64, ple=64).to(torch.bfloat16)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0, 0.02)
    before = [torch.cat([l.weight.detach().clone() for l in linears])
              for _, _, linears in g8.layer_groups(m.model.language_model)[0]]
    nk.install(device=cuda.index)
    gemms = w8.to_b200(m, device=cuda, host_io=True)
    yield m, gemms, before
    sys.modules.pop("npu_kernels", None)


def test_worker_thread_runs_host_io_gemms_exactly(host_model, cuda):
    _, gemms, before = host_model
    worker = RefWorker()
    gen = torch.Generator().manual_seed(7)
    for i, (g, w) in enumerate(zip(gemms, before)):
        q, sw, w_kn, _ = cpu_int8.weight_quant(w)
        assert g.sw.device.type == "cpu" and torch.equal(g.sw, sw)  # the CPU glue's scales
        T = [512, 37, 300, 1][i % 4]
        xq = torch.randint(-127, 128, (T, g.K), dtype=torch.int8, generator=gen)
        kind, fn, name = ref_prefill_gemm(g, xq, None, i % g8.N_SLOTS)
        assert kind == "npu" and name == g.name
        acc = worker.run(fn)
        assert not isinstance(acc, BaseException), acc
        assert acc.device.type == "cpu" and acc.shape == (T, g.N)
        assert torch.equal(acc, cpu_int8.int_mm(xq, w_kn)), g.name
    worker.q.put((None, None))


def test_host_rows_in_host_rows_out(host_model):
    m, gemms, before = host_model
    gen = torch.Generator().manual_seed(8)
    g, w = gemms[2], before[2]
    q, sw, _, sw_bf16 = cpu_int8.weight_quant(w)
    x = torch.randn(40, g.K, generator=gen).to(torch.bfloat16)
    y = g.matmul(x)  # host rows: quant + GEMM + dequant on the GPU, host result
    assert y.device.type == "cpu"
    assert torch.equal(y.view(torch.int16), cpu_int8.linear_dequant(x, q, sw).view(torch.int16))
    h = torch.randn(1, 256, generator=gen).to(torch.bfloat16)
    logits = m.lm_head(h)
    assert logits.device.type == "cpu" and logits.shape == (1, 512)


def test_npu_kernels_mm_i8_host_and_device(cuda):
    nk.install(device=cuda.index)
    nk.use_npu()
    gen = torch.Generator().manual_seed(9)
    a = torch.randint(-128, 128, (300, 1536), dtype=torch.int8, generator=gen)
    b = torch.randint(-128, 128, (1536, 2560), dtype=torch.int8, generator=gen)
    want = torch._int_mm(a, b)
    c = torch.zeros((300, 2560), dtype=torch.int32)
    assert nk.mm_i8(a, b, c) is c and torch.equal(c, want)  # host buffers, GEMM on the GPU
    cd = torch.zeros((300, 2560), dtype=torch.int32, device=cuda)
    nk.mm_i8(a.to(cuda), b.to(cuda), cd)
    assert torch.equal(cd.cpu(), want)
    with pytest.raises(ValueError):
        nk.mm_i8(a, b.to(cuda), c)
