"""Stand-in for the reference's `npu_kernels` module, backed by the sm_100a GEMM.

The reference's modules import it by its top-level name: the scheduler's worker thread
runs `import npu_kernels; npu_kernels.use_npu()` before its first job
(pipeline.py:203-204), `serve.py:67` does the same, NPUGemm reads `BLOCK_K` / `BLOCK_N`
(gemma_npu.py:65-67) and the benches call `mm_i8` (shape_bench.py:29,
bucket_bench.py:14).  `install()` registers this module under that name, so those
imports find it without any change to the reference:

    import gemma_npu_b200.npu_kernels as nk
    nk.install(device=0)          # sys.modules["npu_kernels"] is now this module

Surface (npu_kernels.py:25-64):
    use_npu()         selects, for the calling thread, the CUDA device the B200 GEMMs run
                      on (the reference selects Triton's NPU driver per thread,
                      npu_kernels.py:20-26)
    mm_i8(a, b, c)    c[M,N] int32 = a[M,K] int8 @ b[K,N] int8, written in place and
                      returned.  CUDA tensors run in place on their device.  Host tensors
                      (the reference's host-visible NPU buffers) are copied to the selected
                      device, multiplied there and the result copied back into c before the
                      call returns -- the GEMM itself always runs on the GPU.
    BLOCK_M/N/K       the sm_100a tile; informational, nothing needs padding to it.
"""
import sys
import threading

import torch

from . import kernels

BLOCK_M = kernels.BLOCK_M
BLOCK_N = kernels.BLOCK_N
BLOCK_K = kernels.BLOCK_K

_state = threading.local()
DEVICE = None  # the device use_npu() selects; set by install() (default: the current device)


def _device():
    if DEVICE is not None:
        return torch.device(DEVICE)
    return torch.device("cuda", torch.cuda.current_device())


def use_npu():
    """Select this thread's CUDA device (npu_kernels.py:25-26's per-thread driver choice).

    CUDA's current device is per thread, like Triton's active driver in the reference:
    the thread that launches GEMMs calls this once before its first job.
    """
    dev = _device()
    kernels.use_device(dev)
    _state.device = dev
    return dev


def mm_i8(a, b, c):
    """c = a @ b (int8 x int8 -> exact int32), the reference's mm_i8 (npu_kernels.py:59-64).

    Without its preconditions (M, N multiples of 512, K of 128): any M and N, K % 16 == 0.
    """
    if a.is_cuda and b.is_cuda and c.is_cuda:
        return kernels.mm_i8(a, b, c)
    if a.is_cuda or b.is_cuda or c.is_cuda:
        raise ValueError("mm_i8: a, b and c must all be CUDA tensors or all be host tensors")
    dev = getattr(_state, "device", None) or _device()
    with torch.cuda.device(dev):
        ad = a.to(dev, non_blocking=True)
        bd = b.to(dev, non_blocking=True)
        cd = torch.empty(c.shape, dtype=torch.int32, device=dev)
        kernels.mm_i8(ad, bd, cd)
        c.copy_(cd)  # synchronous device-to-host copy: c holds the result on return
    return c


def install(device=None):
    """Register this module as the top-level `npu_kernels` the reference imports.

    `device` (index or torch.device) is what use_npu() selects; default: the device that
    is current when use_npu() runs.  Returns the module.
    """
    global DEVICE
    if device is not None:
        DEVICE = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
    mod = sys.modules[__name__]
    sys.modules["npu_kernels"] = mod
    return mod
