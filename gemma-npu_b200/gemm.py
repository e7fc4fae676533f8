"""HBM-resident W8A8 linears: the B200 counterpart of the reference's L2 layer.

Mirrors, name for name, the surface of `gemma_npu.py` that the reference's
pipeline and HF forward call:

    B200Gemm      NPUGemm (gemma_npu.py:50-152): .K .N .n_pad .sw .sw_cpu .w_cpu
                  .sizes .name .on_cpu .pending, allocate / stage / launch_slot / matmul
    Slice         Slice (gemma_npu.py:175-193)
    Int8Head      Int8Head (gemma_npu.py:159-172), plus .logits() with the softcap fused
    int8_linear   cpu_int8_linear (gemma_npu.py:155-156)
    to_b200       to_npu (gemma_npu.py:207-241)
    gemm          Prefill.gemm (pipeline.py:233-242), same (kind, value, name) protocol
    BACKENDS / add_backend_argument / apply_backend   the --backend choice (gemma_npu.py:244-266,305)

What changes on B200:
  * one resident int8 copy per group, [N, K] K-major, quantised on the GPU; the
    prefill GEMM reads it as a K-major B operand through TMA and the decode GEMV
    streams its rows, so the reference's three copies (`wt` [K,N_pad] on the NPU,
    `w_kn` and `w_cpu` on the host) become one;
  * no 512-row padding: launch_slot runs one GEMM over exactly T rows, and N needs
    no padding to the tile (n_pad only rounds the slot pitch to 16 columns);
  * the PLE gate (N=256) and projection (K=256) run on the GPU like every other
    group: a launch costs microseconds here, so nothing stays on the CPU
    (`on_cpu` is always False and kept only as an attribute);
  * the dequant of `matmul` is fused into the GEMM epilogue.
Launches are stream-ordered on torch's current stream, so a returned view is
ready for any later work on that stream.

Where results live.  By default the slots are in HBM and `launch_slot` returns a CUDA
int32 view: the caller's glue must then run on the GPU too (the `kernels` row kernels),
because the reference's `k_*` glue is torch.compile'd for the CPU (pipeline.py:66-127)
and handed CUDA tensors Inductor would generate GPU code of its own.  With
`host_io=True` (to_b200(model, host_io=True)) the slots the caller reads and writes are
pinned host memory, like the reference's host-visible NPU buffers: `stage` returns host
rows, `launch_slot` copies them to HBM, runs the GEMM there, copies the int32 result
back and returns it once it has landed, and `.sw` is a host fp32 tensor.  The
reference's unchanged Prefill / Worker (pipeline.py:196-242) and its CPU glue then run
as they are, with every GEMM on the GPU.  `matmul` and `Int8Head` follow the input:
host rows in, host rows out.
"""
import os
import time

import torch

from . import kernels

MAX_ROWS = 4096
TIMES = {"gpu": 0.0, "quant": 0.0, "dequant": 0.0, "launches": 0}
BY_SHAPE = {}  # (N, K) -> [launches, host seconds]

# Rows per pipelined micro-batch slot (the reference's SLOT_ROWS / GEMMA_NPU_ROWS).
SLOT_ROWS = int(os.environ.get("GEMMA_NPU_ROWS", "512"))
MAX_PROMPT = int(os.environ.get("GEMMA_NPU_MAX_PROMPT", "4096"))
N_SLOTS = -(-MAX_PROMPT // SLOT_ROWS)
GEMV_ROWS = 16  # matmul() below this many rows is decode: weight-only GEMV (gemma_npu.py:120)

BACKENDS = ("b200", "npu", "cpu-int8", "cpu")


def _round_up(v, m):
    return -(-v // m) * m


def partition_rows(total, world, rank):
    """Rows [r0, r1) of `total` that `rank` of `world` owns: an even split of concatenated
    prompt rows, for running independent prompts' linears data-parallel over GPUs.

    Every W8A8 linear is row-independent (per-token quant, per-row dequant), so the rows of
    several prompts can be concatenated and cut anywhere; shares differ by at most one row.
    The reference cuts one prompt into 512-row micro-batches instead (pipeline.py:328).
    """
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad partition: total={total} world={world} rank={rank}")
    return total * rank // world, total * (rank + 1) // world


def int8_linear(x2d, wq, sw):
    """Weight-only int8 linear on the GPU: the reference's cpu_int8_linear (gemma_npu.py:155-156)."""
    return kernels.int8_linear(x2d, wq, sw)


def quantize_weight(w, device=None):
    """Per-output-channel int8 quant of a [N, K] weight on the GPU -> (q int8 [N,K], sw fp32 [N]).

    The reference's NPUGemm weight quant (gemma_npu.py:62,68-69): the weight is
    taken in fp32, sw = max(absmax_row, 1e-8) / 127, q = clamp(round(w / sw), -127, 127).
    A bf16 weight is quantised from its bf16 values (its fp32 upcast is exact).
    """
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    w = w.detach()
    if w.dtype not in (torch.bfloat16, torch.float32):
        w = w.float()
    w = w.to(device).contiguous()
    return kernels.quant_rows(w)


class B200Gemm:
    """Linears sharing one input, as a single HBM-resident W8A8 GEMM (NPUGemm on B200)."""

    a_flat = None  # int8 activations, MAX_ROWS x max K
    c_flat = None  # int32 results, MAX_ROWS x max N
    slots = []     # per pipelined micro-batch: (int8 activations, int32 results), SLOT_ROWS each
    host_slots = []  # host_io: the same pairs in pinned host memory (what stage/launch_slot expose)

    def __init__(self, linears, on_cpu=False, device=None, host_io=False):
        ws = [l.weight.detach() for l in linears]
        dt = torch.bfloat16 if all(w.dtype == torch.bfloat16 for w in ws) else torch.float32
        w = torch.cat([x.to(dt) for x in ws])
        self.sizes = [l.out_features for l in linears]
        self.N, self.K = w.shape
        if self.K % 16:
            raise ValueError(f"K = {self.K} must be a multiple of 16 (TMA row alignment)")
        self.n_pad = _round_up(self.N, 16)
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.w, self.sw_dev = quantize_weight(w, self.device)  # int8 [N, K], fp32 [N] in HBM
        self.sw_gemv = self.sw_dev.to(torch.bfloat16)           # bf16 scales of the decode GEMV
        self.host_io = bool(host_io)
        # The scales where the caller's glue reads them (pipeline.py:262-308 passes G[..].sw).
        self.sw = self.sw_dev.cpu() if self.host_io else self.sw_dev
        self.sw_cpu = self.sw_gemv.cpu() if self.host_io else self.sw_gemv
        self.on_cpu = False                                   # everything runs on the GPU
        self.w_kn = None                                      # no separate [K, N] copy
        self.dtype = linears[0].weight.dtype
        self.pending = None
        self.name = ""  # set by to_b200

    @property
    def w_cpu(self):
        """The [N, K] int8 weight the decode GEMV reads (the same resident buffer)."""
        return self.w

    @classmethod
    def allocate(cls, max_k, max_n, device=None, host_io=False):
        """Resident staging buffers: one flat pair plus one (A, C) pair per micro-batch slot
        (with host_io, also a pinned host pair per slot)."""
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        max_n = _round_up(max_n, 16)
        cls.a_flat = torch.empty(MAX_ROWS * max_k, dtype=torch.int8, device=dev)
        cls.c_flat = torch.empty(MAX_ROWS * max_n, dtype=torch.int32, device=dev)
        cls.slots = [(torch.empty(SLOT_ROWS * max_k, dtype=torch.int8, device=dev),
                      torch.empty(SLOT_ROWS * max_n, dtype=torch.int32, device=dev)) for _ in range(N_SLOTS)]
        cls.host_slots = [(torch.empty(SLOT_ROWS * max_k, dtype=torch.int8).pin_memory(),
                           torch.empty(SLOT_ROWS * max_n, dtype=torch.int32).pin_memory())
                          for _ in range(N_SLOTS)] if host_io else []

    def stage(self, slot, T):
        """The slot's int8 activation rows [T, K], to be filled before launch_slot (host rows
        with host_io)."""
        assert T <= SLOT_ROWS, f"micro-batch of {T} rows > {SLOT_ROWS}"
        slots = self.host_slots if self.host_io else self.slots
        return slots[slot][0][: T * self.K].view(T, self.K)

    def launch_slot(self, T, slot):
        """One GEMM over the slot's T staged rows; int32 [T, N], a view of the slot's results.

        With host_io the staged host rows are copied to HBM first and the view is of the
        pinned host results, complete when this returns (the reference's launch is
        synchronous from its worker's view, pipeline.py:206-209)."""
        t = time.perf_counter()
        a_flat, c_flat = self.slots[slot]
        a = a_flat[: T * self.K].view(T, self.K)
        c = c_flat[: T * self.n_pad].view(T, self.n_pad)[:, : self.N]
        if self.host_io:
            ha, hc = self.host_slots[slot]
            a.copy_(ha[: T * self.K].view(T, self.K), non_blocking=True)
            kernels.mm_i8_nk(a, self.w, c)
            out = hc[: T * self.n_pad].view(T, self.n_pad)
            out.copy_(c_flat[: T * self.n_pad].view(T, self.n_pad), non_blocking=True)
            torch.cuda.current_stream(self.device).synchronize()
            c = out[:, : self.N]
        else:
            kernels.mm_i8_nk(a, self.w, c)
        dt = time.perf_counter() - t
        TIMES["launches"] += 1
        TIMES["gpu"] += dt
        st = BY_SHAPE.setdefault((self.N, self.K), [0, 0.0])
        st[0] += 1
        st[1] += dt
        return c

    def matmul(self, x2d):
        """x2d [T, K] -> [T, N] in the layer dtype (NPUGemm.matmul, gemma_npu.py:117-152).

        T < 16 is decode: the weight-only GEMV over the same int8 weights.  Otherwise
        per-token quant, then one GEMM with the dequant fused into its epilogue.
        """
        T = x2d.shape[0]
        on_host = not x2d.is_cuda  # host rows in, host rows out; the work runs in HBM
        if on_host:
            x2d = x2d.to(self.device, non_blocking=True)
        if T < GEMV_ROWS:
            y = int8_linear(x2d, self.w, self.sw_gemv).to(self.dtype)
            return y.cpu() if on_host else y
        t = time.perf_counter()
        xq, sx = kernels.quant_rows(x2d.contiguous())
        t1 = time.perf_counter()
        TIMES["quant"] += t1 - t
        y = kernels.gemm_dequant(xq, self.w, sx, self.sw_dev)
        TIMES["launches"] += 1
        TIMES["gpu"] += time.perf_counter() - t1
        st = BY_SHAPE.setdefault((self.N, self.K), [0, 0.0])
        st[0] += 1
        y = y if self.dtype == torch.bfloat16 else y.to(self.dtype)
        return y.cpu() if on_host else y


# Kept for callers that import the reference's class name.
NPUGemm = B200Gemm


class Int8Head(torch.nn.Module):
    """The LM head as a weight-only int8 GEMV on the GPU (Int8Head, gemma_npu.py:159-172)."""

    def __init__(self, linear, device=None, rows=None):
        super().__init__()
        w = linear.weight.detach()
        if rows is not None:  # a column shard of the head: rows [r0, r1) of the [V, K] weight
            w = w[rows[0]: rows[1]]
        self.wq, sw = quantize_weight(w, device)
        self.sw = sw.to(torch.bfloat16)
        self.in_features = linear.in_features
        self.out_features = w.shape[0]

    def forward(self, x):
        shape = x.shape[:-1]
        on_host = not x.is_cuda  # host rows in, host logits out; the GEMV runs in HBM
        xd = x.to(self.wq.device, non_blocking=True) if on_host else x
        y = int8_linear(xd.reshape(-1, x.shape[-1]), self.wq, self.sw).reshape(*shape, -1)
        return y.cpu() if on_host else y

    def logits(self, h, cap=None, out=None):
        """fp32 logits of one hidden row with the final softcap fused (pipeline.py:335-338)."""
        return kernels.lm_head_logits(h, self.wq, self.sw, cap or 0.0, out=out)


class Slice(torch.nn.Module):
    """Stands in for one linear of a B200Gemm group (Slice, gemma_npu.py:175-193)."""

    def __init__(self, gemm, index, in_features, out_features):
        super().__init__()
        self.gemm, self.index = gemm, index
        self.in_features, self.out_features = in_features, out_features

    def forward(self, x):
        g = self.gemm
        shape = x.shape[:-1]
        if self.index == 0 or g.pending is None or g.pending[0] is not x:
            y = g.matmul(x.reshape(-1, x.shape[-1]))
            parts = torch.split(y, g.sizes, dim=-1) if len(g.sizes) > 1 else (y,)
            g.pending = (x, parts)
        out = g.pending[1][self.index]
        if self.index == len(g.sizes) - 1:
            g.pending = None
        return out.reshape(*shape, -1)


def layer_groups(lm):
    """The reference's per-layer linear grouping (gemma_npu.py:209-224).

    Returns (groups, per_layer_keys): groups is a list of (parent, attribute names,
    linears) and per_layer_keys the 6 group keys of every decoder layer.
    """
    groups, per_layer = [], []
    for layer in lm.layers:
        a, mlp = layer.self_attn, layer.mlp
        qkv = [a.q_proj]
        if not getattr(a, "is_kv_shared_layer", False):
            qkv += [a.k_proj] + ([a.v_proj] if getattr(a, "v_proj", None) is not None else [])
        groups += [(a, ["q_proj", "k_proj", "v_proj"][: len(qkv)], qkv),
                   (a, ["o_proj"], [a.o_proj]),
                   (mlp, ["gate_proj", "up_proj"], [mlp.gate_proj, mlp.up_proj]),
                   (mlp, ["down_proj"], [mlp.down_proj]),
                   (layer, ["per_layer_input_gate"], [layer.per_layer_input_gate]),
                   (layer, ["per_layer_projection"], [layer.per_layer_projection])]
        per_layer.append(["qkv", "o", "gate_up", "down", "ple_gate", "ple_proj"])
    groups.append((lm, ["per_layer_model_projection"], [lm.per_layer_model_projection]))
    return groups, per_layer


def to_b200(model, device=None, host_io=False):
    """Swap the text decoder's linears for resident W8A8 GEMMs on a B200 (to_npu, gemma_npu.py:207-241).

    Every group, the PLE gate/projection included, becomes a B200Gemm; the tied LM
    head gets a separate int8 copy (Int8Head).  Returns the list of groups and sets
    model.layer_gemms like the reference.  host_io=True keeps the slots the caller reads
    and writes in pinned host memory, for the reference's unchanged CPU pipeline.
    """
    lm = model.model.language_model
    groups, per_layer = layer_groups(lm)
    gemms = []
    for parent, names, linears in groups:
        g = B200Gemm(linears, device=device, host_io=host_io)
        g.name = "+".join(names)
        gemms.append(g)
        for i, (name, l) in enumerate(zip(names, linears)):
            setattr(parent, name, Slice(g, i, l.in_features, l.out_features))
    model.layer_gemms = [dict(zip(keys, gemms[6 * i: 6 * i + 6])) for i, keys in enumerate(per_layer)]
    B200Gemm.allocate(max(g.K for g in gemms), max(g.n_pad for g in gemms), device=device, host_io=host_io)
    model.lm_head = Int8Head(model.lm_head, device=device)
    return gemms


def gemm(g, xq, sx, slot):
    """Yieldable GEMM request (Prefill.gemm, pipeline.py:233-242): stage now, run on resume.

    Returns ("npu", thunk, name) so the reference's scheduler hands the thunk to its
    worker thread unchanged; the thunk launches one stream-ordered GEMM and returns
    the int32 [T, N] view of the slot.
    """
    T = xq.shape[0]
    g.stage(slot, T).copy_(xq, non_blocking=True)
    return ("npu", lambda: g.launch_slot(T, slot), g.name)


def add_backend_argument(parser):
    """The reference's --backend flag (gemma_npu.py:305) with the b200 choice added (the default)."""
    parser.add_argument("--backend", default="b200", choices=list(BACKENDS))
    return parser


def apply_backend(model, backend, device=None, host_io=False):
    """What load(backend) does to the model (gemma_npu.py:254) for the b200 backend.

    Returns the groups.  The npu / cpu-int8 / cpu backends are the reference's own
    code paths and are not part of this library.
    """
    if backend != "b200":
        raise ValueError(f"backend {backend!r} is served by the reference pipeline, not by this library")
    return to_b200(model, device=device, host_io=host_io)
