#!/usr/bin/env python
"""Benchmark of the B200 W8A8 linear hot path (BASELINE.json configs 1 and 2).

A step is one pass of the prefill linear set of a 35-layer Gemma E2B-class decoder over
one prompt of M = 3658 tokens (config 1): per layer the qkv (1536->2560), o (2048->1536),
gate_up (1536->12288) and down (6144->1536) W8A8 GEMMs, plus the PLE model projection
(1536->8960), each int8 x int8 -> exact int32 as the reference's mm_i8 / torch._int_mm
produce it.  Weights are random N(0, 0.02) quantised per channel and activations random
N(0, 1) quantised per token, seeded per layer, distinct buffers per layer (synthetic data:
no checkpoint is available).  The step is captured once into a CUDA graph and replayed.

`value` is whole-job TOPS with inputs resident in HBM; `e2e` is the same metric through
the reference-facing API with host buffers (pinned int8 activations and row scales copied
in, the fused-dequant GEMM, bf16 results copied out every step; `e2e_int32` copies the
int32 results out instead, as pipeline.py's CPU glue consumes them).  The decode
weight-only GEMV chain (config 2: the same 140 layer weights + the 262144-wide LM head
with the softcap fused) is reported beside it in GB/s.

With torchrun (N > 1) every rank runs its own prompt (weak scaling, no collective on the
data path); time is the max over ranks.  `--impl reference` times the reference's own
CPU implementation of the path (its `cpu-int8` backend: torch._int_mm) on the host cores.

usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

LAYERS = 35
M_TOKENS = 3658
LAYER_SHAPES = [("qkv", 2560, 1536), ("o", 1536, 2048), ("gate_up", 12288, 1536), ("down", 1536, 6144)]
PLE_SHAPE = ("ple_model", 8960, 1536)
VOCAB, HIDDEN, SOFTCAP = 262144, 1536, 30.0
INT8_PER_BF16 = 2.0  # dense int8 tensor rate / dense bf16 rate on B200 (4.5 / 2.25 PFLOP/s nominal)
NOMINAL_INT8_TOPS = 4500.0
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "gemm_traffic_config1.txt")
SUSTAINED_REGION_S = 1.0  # timed regions at least this long are judged against the sustained peak


def macs_per_token():
    return LAYERS * sum(n * k for _, n, k in LAYER_SHAPES) + PLE_SHAPE[1] * PLE_SHAPE[2]


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ----------------------------------------------------------------------------- setup
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if world == 1 and args.gpus > 1:
        raise SystemExit("--gpus > 1 needs torchrun (one process per GPU)")
    return world, rank, local


def peaks():
    """Roofline denominators: the driver's measurements on this pool, else the recipe's fallback."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    return dict(FALLBACK, source="fallback")


def gemm_traffic_per_launch(layers, m):
    """Memory traffic per GEMM launch of one step, averaged over the step's launches, from
    the committed ncu capture of each config-1 shape (one launch each, M = 3658): DRAM
    bytes read plus every byte the kernel wrote into L2 (L2 write sectors x 32).  DRAM
    write counters miss output still in L2 when a kernel ends, so writes are counted where
    they enter L2.  None when the capture is absent or was taken at another M."""
    if not os.path.exists(TRAFFIC_FILE) or m != M_TOKENS:
        return None
    per = {}
    with open(TRAFFIC_FILE) as f:
        for line in f:
            parts = line.split()
            if len(parts) == 7 and not line.startswith("#"):
                per[parts[0]] = int(parts[4]) + 32 * int(parts[6])
    if not all(name in per for name, _, _ in LAYER_SHAPES + [PLE_SHAPE]):
        return None
    total = layers * sum(per[name] for name, _, _ in LAYER_SHAPES) + per[PLE_SHAPE[0]]
    return {"bytes": total / (layers * len(LAYER_SHAPES) + 1),
            "note": "per GEMM launch, averaged over one step: dram__bytes_read.sum + 32 x "
                    "lts__t_sectors_srcunit_tex_op_write.sum of each shape's single-launch ncu capture "
                    f"({os.path.relpath(TRAFFIC_FILE, ROOT)})"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.proc, self.path = None, None
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            self.fh = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(index), "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) == 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------------------- workloads
def build_prefill(w8, dev, m, only=None, seed=0, layers=LAYERS):
    """Per layer: resident int8 [N,K] weights and int8 [M,K] activations; shared int32 outputs."""
    shapes = [s for s in LAYER_SHAPES if only in (None, s[0])]
    calls, weights = [], []
    outs = {name: torch.empty((m, n), dtype=torch.int32, device=dev) for name, n, _ in shapes + [PLE_SHAPE]}
    acts = []
    for layer in range(layers):
        g = torch.Generator(device=dev).manual_seed(seed * 1000 + layer)
        per = {}
        for name, n, k in shapes:
            wq, _ = w8.quant_rows(torch.randn((n, k), device=dev, generator=g, dtype=torch.bfloat16) * 0.02)
            xq, _ = w8.quant_rows(torch.randn((m, k), device=dev, generator=g, dtype=torch.bfloat16))
            calls.append((xq, wq, outs[name], name))
            per[name] = wq
            acts.append(xq)
        weights.append(per)
    if only in (None, PLE_SHAPE[0]):
        g = torch.Generator(device=dev).manual_seed(seed * 1000 + 999)
        name, n, k = PLE_SHAPE
        wq, _ = w8.quant_rows(torch.randn((n, k), device=dev, generator=g, dtype=torch.bfloat16) * 0.02)
        xq, _ = w8.quant_rows(torch.randn((m, k), device=dev, generator=g, dtype=torch.bfloat16))
        calls.append((xq, wq, outs[name], name))
    torch.cuda.synchronize()
    ops = sum(2 * xq.shape[0] * wq.shape[0] * wq.shape[1] for xq, wq, _, _ in calls)
    # algorithmic bytes: A and B read once, the int32 C written once
    nbytes = sum(xq.numel() + wq.numel() + 4 * xq.shape[0] * wq.shape[0] for xq, wq, _, _ in calls)
    return {"calls": calls, "weights": weights, "ops": ops, "outs": outs, "bytes": nbytes}


def capture(fn, stream):
    """Run fn once eagerly (sets kernel attributes), then capture it into a CUDA graph."""
    with torch.cuda.stream(stream):
        fn()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        fn()
    return graph


def timed(replay, steps, warmup, stream, world):
    """Warm up, then time exactly `steps` replays with CUDA events; max over ranks (ms)."""
    import torch.distributed as dist

    with torch.cuda.stream(stream):  # replays and events on the same stream
        for _ in range(warmup):
            replay()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            replay()
        end.record(stream)
        end.synchronize()
    ms = start.elapsed_time(end)
    torch.cuda.synchronize()
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def e2e_prefill(w8, work, dev, steps, warmup, world, dequant=True):
    """Host-buffer path of the config-1 step through the reference-facing calls: per GEMM,
    pinned host int8 activations (and, with dequant, their fp32 row scales) -> HBM, the
    GEMM, the result -> pinned host (one host buffer per projection; every GEMM has its own
    device output, so no copy out waits for a later GEMM).  dequant=True runs `gemm_dequant` (int32 accumulate
    plus the _deq epilogue, bf16 out: config 0's full operation); dequant=False runs
    `mm_i8_nk` (int32 out, the data flow of pipeline.py's Prefill.gemm).  Copies in, GEMMs
    and copies out run on three streams ordered by events, so PCIe traffic in both
    directions overlaps the GEMMs."""
    import torch.distributed as dist

    calls = work["calls"]
    g = torch.Generator(device=dev).manual_seed(7)
    out_dtype = torch.bfloat16 if dequant else torch.int32
    host_in, host_sx, host_out, scales, outs = {}, {}, {}, [], []
    for xq, wq, _, name in calls:
        if name not in host_in:  # host buffers per projection (each layer's result overwrites the last)
            host_in[name] = xq.cpu().pin_memory()
            host_sx[name] = (torch.rand((xq.shape[0],), generator=None) * 1e-2 + 1e-3).pin_memory()
            host_out[name] = torch.empty((xq.shape[0], wq.shape[0]), dtype=out_dtype).pin_memory()
        sx = torch.empty((xq.shape[0],), dtype=torch.float32, device=dev)
        sw = torch.rand((wq.shape[0],), device=dev, generator=g) * 1e-3 + 1e-4
        scales.append((sx, sw))
        outs.append(torch.empty((xq.shape[0], wq.shape[0]), dtype=out_dtype, device=dev))
    bi = sum(xq.numel() + (4 * xq.shape[0] if dequant else 0) for xq, _, _, _ in calls)
    bo = sum(o.numel() * o.element_size() for o in outs)
    s_in, s_mm, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def step():
        for i, (xq, wq, _, name) in enumerate(calls):
            sx, sw = scales[i]
            with torch.cuda.stream(s_in):
                xq.copy_(host_in[name], non_blocking=True)
                if dequant:
                    sx.copy_(host_sx[name], non_blocking=True)
                e_in = torch.cuda.Event()
                e_in.record(s_in)
            with torch.cuda.stream(s_mm):
                s_mm.wait_event(e_in)
                if dequant:
                    w8.gemm_dequant(xq, wq, sx, sw, out=outs[i])
                else:
                    w8.mm_i8_nk(xq, wq, outs[i])
                e_mm = torch.cuda.Event()
                e_mm.record(s_mm)
            with torch.cuda.stream(s_out):
                s_out.wait_event(e_mm)
                host_out[name].copy_(outs[i], non_blocking=True)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_in)
    s_mm.wait_stream(s_in)
    s_out.wait_stream(s_in)
    for _ in range(steps):
        step()
        torch.cuda.synchronize()  # the results are on the host when the step ends
    s_in.wait_stream(s_out)
    end.record(s_in)
    end.synchronize()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del outs, host_out
    return ms / steps, bi, bo


def build_decode(w8, work, dev):
    """The decode GEMV chain over the prefill's resident weights + an int8 LM head.

    Each GEMV reads the previous one's output as its activation row (its first K values:
    every config-2 output is at least as wide as the next input), and the head reads the
    last one, so the chain is dependent through its data as a decode step is, and every
    activation row is the freshly written output of the kernel before.  The independent
    variant gives each GEMV a row of its own."""
    g = torch.Generator(device=dev).manual_seed(4242)
    chain, indep, nbytes = [], [], 0
    prev = torch.randn((1, HIDDEN), device=dev, generator=g).to(torch.bfloat16)
    for per in work["weights"]:
        for name, n, k in LAYER_SHAPES:
            wq = per[name]
            s = (torch.rand((n,), device=dev, generator=g) * 1e-3 + 1e-4).to(torch.bfloat16)
            y = torch.empty((1, n), dtype=torch.bfloat16, device=dev)
            chain.append((prev[:, :k], wq, s, y))
            indep.append((torch.randn((1, k), device=dev, generator=g).to(torch.bfloat16), wq, s,
                          torch.empty((1, n), dtype=torch.bfloat16, device=dev)))
            prev = y
            nbytes += n * k + 2 * n + 2 * k + 2 * n
    hw, hs = w8.quant_rows(torch.randn((VOCAB, HIDDEN), device=dev, generator=g, dtype=torch.bfloat16) * 0.02)
    head = (prev[0, :HIDDEN], hw, hs.to(torch.bfloat16), torch.empty((VOCAB,), dtype=torch.float32, device=dev))
    nbytes += VOCAB * HIDDEN + 2 * VOCAB + 2 * HIDDEN + 4 * VOCAB
    torch.cuda.synchronize()

    def step():
        for x, wq, s, y in chain:
            w8.int8_linear(x, wq, s, out=y)
        h, hq, hsc, logits = head
        w8.lm_head_logits(h, hq, hsc, SOFTCAP, out=logits, argmax=True)  # + the greedy token


    hq16 = head[1][:, :16].contiguous()

    def step_floor():
        """The same dependent chain (same launches, grids, activation hand-offs and output
        rows) with every GEMV cut to its first 16 columns of K: what a dependent step costs
        without its weight stream."""
        for x, wq, s, y in chain:
            w8.int8_linear(x[:, :16], wq[:, :16], s, out=y)
        h, hq, hsc, logits = head
        w8.lm_head_logits(h[:16], hq16, hsc, SOFTCAP, out=logits, argmax=True)

    side = [torch.cuda.Stream(device=dev) for _ in range(4)]
    layer_bytes = sum(wq.numel() + 2 * wq.shape[0] + 2 * x.numel() + 2 * y.numel() for x, wq, _, y in indep)

    def step_independent():
        """The same layer GEMVs with no order between them: round-robin on 4 streams that
        fork from and join the capturing stream, so consecutive GEMVs overlap."""
        cur = torch.cuda.current_stream()
        fork = torch.cuda.Event()
        fork.record(cur)
        joins = []
        for j, sj in enumerate(side):
            sj.wait_event(fork)
            with torch.cuda.stream(sj):
                for x, wq, sc, y in indep[j::len(side)]:
                    w8.int8_linear(x, wq, sc, out=y)
            ev = torch.cuda.Event()
            ev.record(sj)
            joins.append(ev)
        for ev in joins:
            cur.wait_event(ev)

    return step, nbytes, len(chain) + 1, head, (step_independent, layer_bytes, len(chain)), step_floor


def prompt_lengths(count=8, seed=0, lo=200, hi=3700):
    """Config 4: prompt lengths uniform in [lo, hi], seeded."""
    g = torch.Generator().manual_seed(seed)
    return [int(v) for v in torch.randint(lo, hi + 1, (count,), generator=g)]


def prompts_dp(w8, dev, stream, world, rank, steps, warmup):
    """Config 4: 8 independent prompts through the 35-layer prefill linear set, partitioned
    across the ranks by rows.  Every linear of the set is row-independent, so the prompts'
    rows are concatenated (12851 rows for the seeded lengths) and rank r runs one GEMM per
    weight over its even share [r R / N, (r + 1) R / N) -- no collective, and the same
    rows per GPU whatever the prompt lengths.  Aggregate TOPS over the max-over-ranks time."""
    lengths = prompt_lengths()
    total = sum(lengths)
    r0, r1 = w8.gemm.partition_rows(total, world, rank)
    rows = r1 - r0
    work = build_prefill(w8, dev, rows, seed=100 + rank)

    def step():
        for xq, wq, c, _ in work["calls"]:
            w8.mm_i8_nk(xq, wq, c)

    graph = capture(step, stream)
    ops_all = 2 * total * macs_per_token()
    ms = timed(lambda: graph.replay(), steps, warmup, stream, world) / steps
    del graph, work
    return {"workload": "config 4: 8 prompts, lengths uniform in [200, 3700] (seed 0), their rows concatenated "
                        "and split evenly over the N ranks (rank r: rows [r R/N, (r+1) R/N)), 35-layer prefill "
                        "linear set + PLE projection on each rank's rows, no collective",
            "lengths": lengths, "rows_total": total, "rows_per_rank_max": -(-total // world),
            "value": ops_all / (ms * 1e-3) / 1e12, "unit": "TOPS", "ms_per_pass": ms, "steps": steps,
            "partition": "rows"}


def _head_weight(dev):
    """The config-4 LM head weight (seeded, the same on every rank)."""
    g = torch.Generator(device=dev).manual_seed(77)
    return torch.randn((VOCAB, HIDDEN), device=dev, generator=g, dtype=torch.bfloat16) * 0.02


def sharded_head(w8, dev, stream, world, steps, warmup, pk):
    """Config 4: the 262144-wide LM head column-sharded over the N ranks (local int8 GEMV
    with the softcap + NCCL all-gather of the fp32 logits), time per token, max over ranks.

    Each path is captured once into a CUDA graph (the GEMV and the NCCL all-gather in one
    graph) and replayed; the all-gather alone is timed the same way, so the collective's
    share of a token is measured, not inferred.  The eager path is reported beside it."""
    import torch.distributed as dist

    head = w8.ShardedInt8Head(_head_weight(dev), device=dev, cap=SOFTCAP)
    h = torch.randn((HIDDEN,), device=dev, generator=torch.Generator(device=dev).manual_seed(78)).to(torch.bfloat16)
    eager_ms = timed(lambda: head(h), steps, warmup, stream, world) / steps
    graph = capture(lambda: head(h), stream)
    ms = timed(lambda: graph.replay(), steps, warmup, stream, world) / steps
    del graph
    ggraph = capture(lambda: head.greedy(h), stream)
    gms = timed(lambda: ggraph.replay(), steps, warmup, stream, world) / steps
    del ggraph
    local_graph = capture(lambda: head.local_logits(h), stream)
    lms = timed(lambda: local_graph.replay(), steps, warmup, stream, world) / steps
    del local_graph
    ag_ms = None
    if world > 1:
        agraph = capture(lambda: dist.all_gather_into_tensor(head.full, head.local), stream)
        ag_ms = timed(lambda: agraph.replay(), steps, warmup, stream, world) / steps
        del agraph
    peer = {}
    if world > 1:
        # the all-gather inside the GEMV: every logit stored into every rank's buffer over NVLink
        head_p = w8.ShardedInt8Head(_head_weight(dev), device=dev, cap=SOFTCAP, transport="peer")
        pgraph = capture(lambda: head_p(h), stream)
        pms = timed(lambda: pgraph.replay(), steps, warmup, stream, world) / steps
        del pgraph
        pggraph = capture(lambda: head_p.greedy(h), stream)
        pgms = timed(lambda: pggraph.replay(), steps, warmup, stream, world) / steps
        del pggraph
        torch.cuda.synchronize()
        peer = {"us_per_token_peer": pms * 1e3, "us_per_token_peer_greedy": pgms * 1e3,
                "peer_note": "w8_lm_head_peer_f32: one kernel per rank, each logit stored into every rank's gathered "
                             "buffer through CUDA IPC peer pointers, ready/done flags in the same buffers; no NCCL. "
                             "The greedy path (w8_lm_head_peer_argmax) sends only the 8-byte keys"}
        head_p.close()
    shard_bytes = (head.r1 - head.r0) * (HIDDEN + 2)
    return {"workload": f"config 4: LM head {VOCAB}x{HIDDEN} int8 split by rows over {world} GPU(s), "
                        "fused softcap, NCCL all-gather of fp32 logits" + (" (no collective at N=1)" if world == 1 else ""),
            **peer,
            "us_per_token": ms * 1e3, "us_per_token_eager": eager_ms * 1e3, "us_per_token_greedy": gms * 1e3,
            "us_local_gemv": lms * 1e3, "us_allgather": None if ag_ms is None else ag_ms * 1e3,
            "shard_rows": head.r1 - head.r0, "local_gemv_gbs": shard_bytes / (lms * 1e-3) / 1e9,
            "allgather_bytes": 4 * world * head.per, "graph": "GEMV + NCCL all-gather captured in one CUDA graph",
            "steps": steps}


def fused_gelu_up(w8, work, dev, stream, steps, warmup, world):
    """Fused epilogue chain: the gate/up GEMM with the k_gelu glue (pipeline.py:102-107)
    fused into its epilogue, against the same work unfused on the GPU (int32 GEMM, then
    dequant, gelu(gate) * up and quant as separate kernels), 35 layers each."""
    name, n, k = LAYER_SHAPES[2]
    inter = n // 2
    g = torch.Generator(device=dev).manual_seed(31)
    xs = [xq for xq, _, _, nm in work["calls"] if nm == name]
    m = xs[0].shape[0]
    layers = []
    for per, xq in zip(work["weights"], xs):
        sx = torch.rand((m,), device=dev, generator=g) * 0.03 + 0.01
        sw = torch.rand((n,), device=dev, generator=g) * 1e-3 + 1e-4
        wp, swp = w8.pack_gelu_up(per[name], sw)
        layers.append((xq, sx, per[name], sw, wp, swp))
    q = torch.empty((m, inter), dtype=torch.int8, device=dev)
    s = torch.empty((m,), dtype=torch.float32, device=dev)
    y = torch.empty((m, inter), dtype=torch.bfloat16, device=dev)
    acc = torch.empty((m, n), dtype=torch.int32, device=dev)

    def fused():
        for xq, sx, _, _, wp, swp in layers:
            w8.gelu_up_quant(xq, sx, wp, swp, q=q, s=s, y=y)

    def unfused():
        for xq, sx, wq, sw, _, _ in layers:
            w8.mm_i8_nk(xq, wq, acc)
            d = w8.dequant(acc, sx, sw)
            a = (torch.nn.functional.gelu(d[:, :inter], approximate="tanh") * d[:, inter:]).to(torch.bfloat16)
            w8.quant_rows(a, q=q, s=s)

    res = {}
    for label, fn in (("fused", fused), ("unfused", unfused)):
        gr = capture(fn, stream)
        res[label] = timed(lambda: gr.replay(), steps, warmup, stream, world) / steps / len(layers)
        del gr
    ops = 2 * m * n * k
    return {"workload": f"config-1 gate/up (M={m}, 2I={n}, K={k}) x {len(layers)} layers, k_gelu glue "
                        "(dequant, gelu_tanh(gate) * up, int8 quant) fused into the GEMM epilogue",
            "us_per_layer_fused": res["fused"] * 1e3, "us_per_layer_unfused": res["unfused"] * 1e3,
            "tops_fused": ops / (res["fused"] * 1e-3) / 1e12, "speedup": res["unfused"] / res["fused"],
            "unfused": "int32 GEMM + dequant kernel + torch gelu/mul + quant kernel on the same GPU",
            "hbm_bytes_avoided_per_layer": 4 * m * n * 2 + 2 * m * n * 2}


def _torch_rms(x, w, eps):
    x = x.float()
    y = x * torch.pow(x.pow(2).mean(-1, keepdim=True) + eps, -0.5)
    return y * w.float() if w is not None else y


def _torch_rope(x, cos, sin):
    half = x.shape[-1] // 2
    return x * cos + torch.cat((-x[..., half:], x[..., :half]), dim=-1) * sin


def glue_rows(w8, dev, stream, m, steps, warmup, world, pk):
    """The warp-per-row glue kernels one at a time at M tokens (pipeline.py:66-127, config-1
    widths: hidden 1536, 8 query heads on 1 KV head of 256, PLE width 256).  Each kernel runs
    over 8 sets of distinct buffers in one graph (> 126 MB of L2 per pass, except the
    256-wide k_ple_gate), so it streams from HBM; us per call, algorithmic GB/s (bytes read + written
    once) and the fraction of the measured HBM copy bandwidth.  `floor_us` is the same kernel
    over 8 rows in the same graph (its launch, its wait for the previous kernel and one row's
    round trip); `remainder_frac` is the HBM fraction of the time the other rows add."""
    eps, hid, nh, kv, d, pw, sets, few = 1e-6, 1536, 8, 1, 256, 256, 8, 8
    g = torch.Generator(device=dev).manual_seed(91)

    def bf(*shape, scale=1.0):
        return (torch.randn(shape, device=dev, generator=g) * scale).to(torch.bfloat16)

    w1, w2, qn, kn = bf(hid, scale=0.1) + 1, bf(hid, scale=0.1) + 1, bf(d, scale=0.1) + 1, bf(d, scale=0.1) + 1
    cos_all, sin_all = bf(m, d), bf(m, d)

    def make_cases(t):
        cos, sin = cos_all[:t], sin_all[:t]
        return {
            "k_in": (lambda i, b: w8.rms_quant(b[0], w1, eps), lambda: [bf(t, hid)], 3 * t * hid + 4 * t),
            "k_qkv_d256": (lambda i, b: w8.qkv_norm_rope(b[0], cos, sin, qn, kn, eps, nh, kv, d, out=b[1]),
                           lambda: [bf(t, (nh + 2 * kv) * d),
                                    torch.empty(((nh + 2 * kv), t, d), dtype=torch.bfloat16, device=dev)],
                           4 * t * (nh + 2 * kv) * d + 4 * t * d),
            "k_attn_out": (lambda i, b: w8.attn_out_quant(b[0]), lambda: [bf(nh, t, d)], 3 * t * nh * d + 4 * t),
            "k_post_attn": (lambda i, b: w8.post_norm_quant(b[0], b[1], w1, w2, eps, h=b[2]),
                            lambda: [bf(t, hid), bf(t, hid), torch.empty((t, hid), dtype=torch.bfloat16, device=dev)],
                            7 * t * hid + 4 * t),
            "k_post_ff": (lambda i, b: w8.post_norm_quant(b[0], b[1], w1, None, eps, h=b[2]),
                          lambda: [bf(t, hid), bf(t, hid), torch.empty((t, hid), dtype=torch.bfloat16, device=dev)],
                          7 * t * hid + 4 * t),
            "k_ple_gate": (lambda i, b: w8.ple_gate_quant(b[0], b[1]), lambda: [bf(t, pw), bf(t, pw)],
                           5 * t * pw + 4 * t),
            "k_ple_out+k_in": (lambda i, b: w8.ple_out(b[0], b[1], w1, 0.75, eps, w_next=w2, h=b[2]),
                               lambda: [bf(t, hid), bf(t, hid), torch.empty((t, hid), dtype=torch.bfloat16, device=dev)],
                               7 * t * hid + 4 * t),
        }

    def run(call, make):
        bufs = [make() for _ in range(sets)]
        graph = capture(lambda: [call(i, b) for i, b in enumerate(bufs)], stream)
        us = timed(lambda: graph.replay(), steps, warmup, stream, world) / (steps * sets) * 1e3
        del graph, bufs
        return us

    out = {}
    full, small = make_cases(m), make_cases(few)
    for name, (call, make, nbytes) in full.items():
        us = run(call, make)
        floor = run(*small[name][:2])
        gbs = nbytes / (us * 1e-6) / 1e9
        rest = nbytes / ((us - floor) * 1e-6) / 1e9 if us > floor else None
        out[name] = {"us": us, "bytes": nbytes, "gbs": gbs, "frac_hbm": gbs / pk["hbm_gbs"], "floor_us": floor,
                     "remainder_frac": None if rest is None else rest / pk["hbm_gbs"]}
    torch.cuda.synchronize()
    return {"workload": f"glue row kernels at M={m} (hidden 1536, H=8 / KV=1 / D=256, PLE 256), 8 buffer sets "
                        "rotated per graph so each call streams from HBM",
            "kernels": out,
            "note": "each call pays a floor (launch, wait for the previous kernel, one row's DRAM round trip: "
                    "floor_us, the same kernel over 8 rows) before its rows stream; one row per warp, one wave"}


def fused_layer(w8, dev, stream, m, steps, warmup, world, layers=35):
    """The fused epilogue chain across a whole decoder layer: the linear set with all of its glue
    on the GPU (k_in, qkv + k_qkv, k_attn_out, o + k_post_attn, gate_up + k_gelu,
    down + k_post_ff; pipeline.py:66-114), attention excluded (a synthetic o of the right
    shape stands in).  Fused: dequant / gelu in the GEMM epilogues plus warp-per-row glue
    kernels (k_qkv as the row kernel: inside the dependent layer chain it measured as fast
    as the qkv GEMM with k_qkv in its epilogue, 180 against 181 us per layer).  Unfused: int32 GEMMs, then the reference's glue expressions as torch ops on
    the same GPU."""
    eps, nh, kv, d, hid = 1e-6, 8, 1, 256, 1536
    g = torch.Generator(device=dev).manual_seed(57)

    def wq(n, k):
        w, s_ = w8.quant_rows(torch.randn((n, k), device=dev, generator=g, dtype=torch.bfloat16) * 0.02)
        return w, s_

    def nw(n):
        return (1 + 0.1 * torch.randn((n,), device=dev, generator=g)).to(torch.bfloat16)

    L = []
    for _ in range(layers):
        qkv, o, gu, dn = wq((nh + 2 * kv) * d, hid), wq(hid, nh * d), wq(12288, hid), wq(hid, 6144)
        gup = w8.pack_gelu_up(*gu)
        L.append(dict(qkv=qkv, o=o, gu=gu, gup=gup, dn=dn, w_in=nw(hid), qn=nw(d), kn=nw(d), w_post=nw(hid),
                      w_pre=nw(hid), w_pff=nw(hid)))
    h0 = torch.randn((m, hid), device=dev, generator=g).to(torch.bfloat16)
    ang = torch.arange(m, device=dev)[:, None].float() * (1e6 ** (-torch.arange(0, d, 2, device=dev).float() / d))[None]
    ang = torch.cat([ang, ang], dim=-1)
    cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    attn = torch.randn((nh, m, d), device=dev, generator=g).to(torch.bfloat16)  # stands in for attention
    h = torch.empty_like(h0)
    c_qkv = torch.empty((m, (nh + 2 * kv) * d), dtype=torch.int32, device=dev)
    c_o = torch.empty((m, hid), dtype=torch.int32, device=dev)
    c_gu = torch.empty((m, 12288), dtype=torch.int32, device=dev)
    c_dn = torch.empty((m, hid), dtype=torch.int32, device=dev)

    def fused():
        h.copy_(h0)
        for l in L:
            xq, sx = w8.rms_quant(h, l["w_in"], eps)
            y = w8.gemm_dequant(xq, l["qkv"][0], sx, l["qkv"][1])
            w8.qkv_norm_rope(y, cos, sin, l["qn"], l["kn"], eps, nh, kv, d)
            xq, sx = w8.attn_out_quant(attn)
            y = w8.gemm_dequant(xq, l["o"][0], sx, l["o"][1])
            _, xq, sx = w8.post_norm_quant(y, h, l["w_post"], l["w_pre"], eps, h=h)
            xq, sx = w8.gelu_up_quant(xq, sx, *l["gup"])
            y = w8.gemm_dequant(xq, l["dn"][0], sx, l["dn"][1])
            w8.post_norm_quant(y, h, l["w_pff"], None, eps, h=h)

    def unfused():
        hh = h0
        for l in L:
            xq, sx = w8.quant_rows(_torch_rms(hh, l["w_in"], eps).to(torch.bfloat16))
            w8.mm_i8_nk(xq, l["qkv"][0], c_qkv)
            yq = w8.dequant(c_qkv, sx, l["qkv"][1])
            q = yq[:, : nh * d].reshape(m, nh, d)
            q = _torch_rope(_torch_rms(q, l["qn"], eps).to(torch.bfloat16), cos[:, None], sin[:, None]).transpose(0, 1)
            k_ = yq[:, nh * d: (nh + kv) * d].reshape(m, kv, d)
            k_ = _torch_rope(_torch_rms(k_, l["kn"], eps).to(torch.bfloat16), cos[:, None], sin[:, None]).transpose(0, 1)
            v_ = _torch_rms(yq[:, (nh + kv) * d:].reshape(m, kv, d), None, eps).to(torch.bfloat16).transpose(0, 1)
            xq, sx = w8.quant_rows(attn.transpose(0, 1).reshape(m, nh * d).contiguous())
            w8.mm_i8_nk(xq, l["o"][0], c_o)
            hh = hh + _torch_rms(w8.dequant(c_o, sx, l["o"][1]), l["w_post"], eps).to(torch.bfloat16)
            xq, sx = w8.quant_rows(_torch_rms(hh, l["w_pre"], eps).to(torch.bfloat16))
            w8.mm_i8_nk(xq, l["gu"][0], c_gu)
            yg = w8.dequant(c_gu, sx, l["gu"][1])
            a = (torch.nn.functional.gelu(yg[:, :6144], approximate="tanh") * yg[:, 6144:]).to(torch.bfloat16)
            xq, sx = w8.quant_rows(a)
            w8.mm_i8_nk(xq, l["dn"][0], c_dn)
            hh = hh + _torch_rms(w8.dequant(c_dn, sx, l["dn"][1]), l["w_pff"], eps).to(torch.bfloat16)
            del q, k_, v_

    res = {}
    for label, fn in (("fused", fused), ("unfused", unfused)):
        gr = capture(fn, stream)
        res[label] = timed(lambda: gr.replay(), steps, warmup, stream, world) / steps / layers
        del gr
    ops = 2 * m * sum(n * k for _, n, k in LAYER_SHAPES)
    return {"workload": f"{layers} decoder layers at M={m}: k_in, qkv + k_qkv (H=8, KV=1, D=256, RoPE), "
                        "k_attn_out, o + k_post_attn, gate_up + k_gelu, down + k_post_ff (attention excluded)",
            "us_per_layer_fused": res["fused"] * 1e3, "us_per_layer_unfused": res["unfused"] * 1e3,
            "tops_fused": ops / (res["fused"] * 1e-3) / 1e12, "speedup": res["unfused"] / res["fused"],
            "unfused": "int32 GEMMs + dequant / quant kernels + the reference's glue as torch ops on the same GPU"}


def prefill_gpu(w8, dev, stream, m, steps, warmup, world, layers=35, kv_shared=0):
    """One prompt through every decoder layer's linear set, glue and attention on the GPU,
    the layer body of pipeline.py:262-310: k_in, qkv GEMM + k_qkv, attention, k_attn_out, o GEMM + k_post_attn, gate/up GEMM + k_gelu, down GEMM +
    k_post_ff, PLE gate GEMM (1536 -> 256) + k_ple_gate, PLE projection GEMM (256 -> 1536) +
    k_ple_out.  Gemma E2B attention layout: every 5th layer full causal with head_dim 512
    (qkv 5120 x 1536, o 1536 x 4096), the others sliding window 512 with head_dim 256; 8
    query heads on 1 KV head.  The last `kv_shared` layers are KV-shared as the reference
    groups them (gemma_npu.py:214-216, pipeline.py:258-281): a q-only qkv GEMM, the keys and
    values of the last unshared layer of the same attention type, and a double-wide MLP
    (gate/up 24576 x 1536, down 1536 x 12288).  Random weights and per-layer inputs; the
    residual stream is carried from layer to layer, and k_ple_out shares its row pass with
    the next k_in."""
    eps, nh, kv, hid = 1e-6, 8, 1, 1536
    g = torch.Generator(device=dev).manual_seed(91)

    def wq(n, k):
        return w8.quant_rows(torch.randn((n, k), device=dev, generator=g, dtype=torch.bfloat16) * 0.02)

    def nw(n):
        return (1 + 0.1 * torch.randn((n,), device=dev, generator=g)).to(torch.bfloat16)

    def rope(d, base):
        ang = torch.arange(m, device=dev)[:, None].float() * (base ** (-torch.arange(0, d, 2, device=dev).float() / d))[None]
        ang = torch.cat([ang, ang], dim=-1)
        return ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)

    tables = {256: rope(256, 1e4), 512: rope(512, 1e6)}
    L = []
    first_shared = layers - kv_shared
    for i in range(layers):
        d, win = (512, 0) if i % 5 == 4 else (256, 512)
        shared = i >= first_shared
        inter = 12288 if shared else 6144  # the double-wide MLP of KV-shared layers
        L.append(dict(d=d, win=win, shared=shared, qkv=wq((nh if shared else nh + 2 * kv) * d, hid), o=wq(hid, nh * d),
                      gup=w8.pack_gelu_up(*wq(2 * inter, hid)), dn=wq(hid, inter), w_in=nw(hid), qn=nw(d), kn=nw(d),
                      w_post=nw(hid), w_pre=nw(hid), w_pff=nw(hid), pg=wq(256, hid), pp=wq(hid, 256),
                      w_ple=nw(hid), scalar=float((0.5 + torch.rand((1,), device=dev, generator=g)).to(torch.bfloat16))))
    ple = torch.randn((m, layers, 256), device=dev, generator=g).to(torch.bfloat16)  # per-layer inputs
    h0 = torch.randn((m, hid), device=dev, generator=g).to(torch.bfloat16)
    h = torch.empty_like(h0)

    # keys / values of the last unshared layer of each attention type, for the shared layers
    kv_store = {d: torch.empty((2 * kv, m, d), dtype=torch.bfloat16, device=dev) for d in tables}

    def qkv(xq, sx, l, shared):
        """The qkv GEMM (dequant fused), then the k_qkv row kernel.  The GEMM with k_qkv in its
        epilogue (w8_gemm_qkv_norm_rope_tiled) is faster alone (bench qkv_paths) but measured
        9.43 against 9.40 ms per prefill inside this dependent chain."""
        d = l["d"]
        y = w8.gemm_dequant(xq, l["qkv"][0], sx, l["qkv"][1])
        return w8.qkv_norm_rope(y, *tables[d], l["qn"], None if shared else l["kn"], eps, nh, kv, d, shared=shared)

    def step():
        h.copy_(h0)
        xq, sx = w8.rms_quant(h, L[0]["w_in"], eps)
        for i, l in enumerate(L):
            d = l["d"]
            if l["shared"]:
                q, _, _ = qkv(xq, sx, l, True)
                k, v = kv_store[d][:kv], kv_store[d][kv:]
            else:
                q, k, v = qkv(xq, sx, l, False)
                if i < first_shared and any(x["d"] == d for x in L[first_shared:]) and \
                        all(x["d"] != d for x in L[i + 1: first_shared]):
                    kv_store[d][:kv].copy_(k)  # the last unshared layer of this type stores its K / V
                    kv_store[d][kv:].copy_(v)
            xq, sx = w8.attention_quant(q, k, v, l["win"])  # attention + k_attn_out
            y = w8.gemm_dequant(xq, l["o"][0], sx, l["o"][1])
            _, xq, sx = w8.post_norm_quant(y, h, l["w_post"], l["w_pre"], eps, h=h)
            xq, sx = w8.gelu_up_quant(xq, sx, *l["gup"])
            y = w8.gemm_dequant(xq, l["dn"][0], sx, l["dn"][1])
            _, xq, sx = w8.post_norm_quant(y, h, l["w_pff"], None, eps, h=h)  # k_post_ff
            y = w8.gemm_dequant(xq, l["pg"][0], sx, l["pg"][1])
            xq, sx = w8.ple_gate_quant(y, ple[:, i])
            y = w8.gemm_dequant(xq, l["pp"][0], sx, l["pp"][1])
            # k_ple_out and the next layer's k_in in one row pass
            nxt = L[i + 1]["w_in"] if i + 1 < len(L) else None
            r = w8.ple_out(y, h, l["w_ple"], l["scalar"], eps, w_next=nxt, h=h)
            if nxt is not None:
                _, xq, sx = r

    gr = capture(step, stream)
    ms = timed(lambda: gr.replay(), steps, warmup, stream, world) / steps
    del gr
    assert torch.isfinite(h.float()).all()
    linear_ops = sum(2 * m * (l["qkv"][0].numel() + l["o"][0].numel() + l["gup"][0].numel() + l["dn"][0].numel()
                              + l["pg"][0].numel() + l["pp"][0].numel()) for l in L)
    return {"workload": f"{layers} decoder layers of one {m}-token prompt on the GPU (linear set + glue + attention; "
                        "every 5th layer full attention with head_dim 512, others sliding window 512 / head_dim 256; "
                        "PLE branch per layer (gate 1536->256 + k_ple_gate, projection 256->1536 + k_ple_out); "
                        + (f"the last {kv_shared} layers KV-shared: q-only qkv, shared K/V, double-wide MLP)"
                           if kv_shared else "no KV sharing)"),
            "ms_per_prefill": ms, "linear_tops": linear_ops / (ms * 1e-3) / 1e12,
            "reference": "the reference keeps its NPU busy 2.38 s per 3658-token prefill (README.md:61-62), its CPU "
                         "attention on top"}


def qkv_paths(w8, dev, stream, m, steps, warmup, world):
    """The qkv GEMM + k_qkv at head_dim 256 (8 q heads, 1 KV head, M tokens), both ways:
    the GEMM with the dequant fused then the k_qkv row kernel, and the one kernel with
    k_qkv in the GEMM epilogue (w8_gemm_qkv_norm_rope); 8 rotated weights, us per call."""
    nh, kv, d, k = 8, 1, 256, 1536
    g = torch.Generator(device=dev).manual_seed(33)
    xq, sx = w8.quant_rows(torch.randn((m, k), device=dev, generator=g, dtype=torch.bfloat16))
    ws = [w8.quant_rows(torch.randn(((nh + 2 * kv) * d, k), device=dev, generator=g, dtype=torch.bfloat16) * 0.02)
          for _ in range(8)]
    ang = torch.arange(m, device=dev)[:, None].float() * (1e4 ** (-torch.arange(0, d, 2, device=dev).float() / d))[None]
    ang = torch.cat([ang, ang], dim=-1)
    cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    qn = torch.ones((d,), dtype=torch.bfloat16, device=dev)
    out = torch.empty(((nh + 2 * kv), m, d), dtype=torch.bfloat16, device=dev)
    y = torch.empty((m, (nh + 2 * kv) * d), dtype=torch.bfloat16, device=dev)

    def two_step():
        for wq, sw in ws:
            w8.gemm_dequant(xq, wq, sx, sw, out=y)
            w8.qkv_norm_rope(y, cos, sin, qn, qn, 1e-6, nh, kv, d, out=out)

    def fused():
        for wq, sw in ws:
            w8.gemm_qkv_norm_rope(xq, wq, sx, sw, cos, sin, qn, qn, 1e-6, nh, kv, d, out=out)

    tiles = w8.rope_tiles(cos, sin)  # once per prompt

    def fused_tiled():
        for wq, sw in ws:
            w8.gemm_qkv_norm_rope(xq, wq, sx, sw, cos, sin, qn, qn, 1e-6, nh, kv, d, out=out, tiles=tiles)

    res = {}
    for label, fn in (("gemm_then_row_kernel", two_step), ("fused_epilogue", fused),
                      ("fused_epilogue_tiled_rope", fused_tiled)):
        gr = capture(fn, stream)
        res[label + "_us"] = timed(lambda: gr.replay(), steps, warmup, stream, world) / steps * 1e3 / len(ws)
        del gr
    res["workload"] = f"qkv {(nh + 2 * kv) * d}x{k} at M={m} + k_qkv (D 256, H 8, KV 1)"
    return res


def attention_bench(w8, dev, stream, m, steps, warmup, world):
    """GPU attention: prefill attention of one prompt on the GPU (pipeline.py:139-180),
    Gemma E2B layer types: sliding window 512 with head_dim 256 (28 of 35 layers) and full
    causal with head_dim 512 (7 layers), 8 query heads on 1 KV head.  TFLOP/s counts the
    useful products (keys each query may see), 4 * H * D per (query, key)."""
    out = {}
    g = torch.Generator(device=dev).manual_seed(3)
    for name, d, win in (("sliding_w512_d256", 256, 512), ("full_d512", 512, 0)):
        sc = d ** -0.25
        q = (torch.randn((8, m, d), device=dev, generator=g) * sc).to(torch.bfloat16)
        k = (torch.randn((1, m, d), device=dev, generator=g) * sc).to(torch.bfloat16)
        v = torch.randn((1, m, d), device=dev, generator=g).to(torch.bfloat16)
        o = torch.empty_like(q)
        pos = torch.arange(m, dtype=torch.float64)
        pairs = float(torch.clamp(pos + 1, max=win).sum()) if win else m * (m + 1) / 2
        for sched in ("tc", "mma"):
            gr = capture(lambda: w8.attention_prefill(q, k, v, win, out=o, schedule=sched), stream)
            ms = timed(lambda: gr.replay(), steps, warmup, stream, world) / steps
            del gr
            key = name if sched == "tc" else name + "_mma"
            out[key] = {"us": ms * 1e3, "tflops": 4 * 8 * d * pairs / (ms * 1e-3) / 1e12}
    out["per_prefill_ms"] = (28 * out["sliding_w512_d256"]["us"] + 7 * out["full_d512"]["us"]) / 1e3
    out["per_prefill_ms_mma"] = (28 * out["sliding_w512_d256_mma"]["us"] + 7 * out["full_d512_mma"]["us"]) / 1e3
    out["workload"] = (f"one prompt of {m} tokens, 8 query heads on 1 KV head; per_prefill_ms = 28 sliding + "
                       "7 full layers; tcgen05 flash attention (the *_mma keys: the mma.sync schedule)")
    return out


def sweep(w8, dev, stream, steps, warmup):
    """Config 3: each projection shape over 35 layers at M in {207, 858, 1878, 3658}, with
    and without the reference's 512-row padding (TOPS on the unpadded rows); plus the real
    E2B shape mix at M = 3658."""
    out = {}
    for m in (207, 858, 1878, 3658):
        mp = -(-m // 512) * 512
        work = build_prefill(w8, dev, mp)
        row = {}
        for name, n, k in LAYER_SHAPES + [PLE_SHAPE]:
            calls = [(xq, wq, c) for xq, wq, c, nm in work["calls"] if nm == name]
            res = {}
            for label, rows in (("unpadded", m), ("padded", mp)):
                cs = [(xq[:rows], wq, c[:rows]) for xq, wq, c in calls]

                def step(cs=cs):
                    for xq, wq, c in cs:
                        w8.mm_i8_nk(xq, wq, c)

                gr = capture(step, stream)
                ms = timed(lambda: gr.replay(), steps, warmup, stream, 1) / steps
                del gr
                res[label] = {"us_per_gemm": ms * 1e3 / len(cs),
                              "tops": 2 * m * n * k * len(cs) / (ms * 1e-3) / 1e12}
            row[name] = res
        out[str(m)] = row
        del work
    # The real E2B shape mix at M = 3658, 8 distinct weights per shape.
    e2b = {"gate_up_x2 24576x1536": (24576, 1536), "down_x2 1536x12288": (1536, 12288),
           "qkv_global 5120x1536": (5120, 1536), "o_global 1536x4096": (1536, 4096),
           "q_only 2048x1536": (2048, 1536), "ple_gate 256x1536": (256, 1536), "ple_proj 1536x256": (1536, 256)}
    m = 3658
    g = torch.Generator(device=dev).manual_seed(5)
    mix = {}
    for name, (n, k) in e2b.items():
        xq = torch.randint(-127, 128, (m, k), dtype=torch.int8, device=dev, generator=g)
        ws = [torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev, generator=g) for _ in range(8)]
        c = torch.empty((m, n), dtype=torch.int32, device=dev)

        def step(xq=xq, ws=ws, c=c):
            for w in ws:
                w8.mm_i8_nk(xq, w, c)

        gr = capture(step, stream)
        ms = timed(lambda: gr.replay(), steps, warmup, stream, 1) / steps
        del gr
        mix[name] = {"us_per_gemm": ms * 1e3 / len(ws), "tops": 2 * m * n * k * len(ws) / (ms * 1e-3) / 1e12}
    out["e2b_mix_m3658"] = mix
    return out


def gemm_table(w8, dev, stream, steps, warmup):
    """Each config-1 shape at M = 3658 with this library's GEMM (w8_mm_i8_ws) and with
    cuBLASLt (torch._int_mm, the library GEMM the kernel replaces), int32 out, both over
    the same 4 rotating (activation, weight, output) sets so that every launch streams from
    HBM; the results are compared bit for bit.  us per GEMM and TOPS per side."""
    m = M_TOKENS
    g = torch.Generator(device=dev).manual_seed(17)
    out = {}
    for name, n, k in LAYER_SHAPES + [PLE_SHAPE]:
        sets = [(torch.randint(-128, 128, (m, k), dtype=torch.int8, device=dev, generator=g),
                 torch.randint(-128, 128, (n, k), dtype=torch.int8, device=dev, generator=g),
                 torch.empty((m, n), dtype=torch.int32, device=dev)) for _ in range(4)]
        refs = [torch.empty((m, n), dtype=torch.int32, device=dev) for _ in range(4)]

        def ours():
            for a, w, c in sets:
                w8.mm_i8_nk(a, w, c)

        def cublas():
            for (a, w, _), r in zip(sets, refs):
                torch._int_mm(a, w.t(), out=r)

        res = {}
        for label, fn in (("b200", ours), ("cublaslt", cublas)):
            gr = capture(fn, stream)
            ms = timed(lambda: gr.replay(), steps, warmup, stream, 1) / steps
            del gr
            us = ms * 1e3 / len(sets)
            res[label] = {"us": us, "tops": 2 * m * n * k / (us * 1e-6) / 1e12}
        res["bit_exact"] = all(torch.equal(c, r) for (_, _, c), r in zip(sets, refs))
        res["ratio_b200_over_cublaslt"] = res["cublaslt"]["us"] / res["b200"]["us"]
        out[f"{name} {m}x{n}x{k}"] = res
        del sets, refs
    return out


# ----------------------------------------------------------------------------- CPU reference
def cpu_reference_step(m, layers, seed=0):
    """The reference's cpu-int8 prefill GEMMs (torch._int_mm) over `layers` layers plus the
    PLE model projection, the same GEMM mix as the GPU step; returns (run, ops)."""
    from oracle import cpu_int8

    g = torch.Generator().manual_seed(seed)
    data = []
    for _, n, k in [s for _ in range(layers) for s in LAYER_SHAPES] + [PLE_SHAPE]:
        xq, _ = cpu_int8.quant(torch.randn(m, k, generator=g).to(torch.bfloat16))
        w_kn = cpu_int8.weight_quant(torch.randn(n, k, generator=g) * 0.02)[2]
        data.append((xq, w_kn))
    ops = sum(2 * m * w.shape[1] * w.shape[0] for _, w in data)

    def run():
        for xq, w_kn in data:
            cpu_int8.int_mm(xq, w_kn)

    return run, ops


def cpu_reference_rate(m, target_s=10.0, max_layers=35):
    """TOPS of the reference CPU path on a bounded sample of config 1, sized to ~target_s."""
    from oracle import cpu_int8

    cores = cpu_int8.set_threads()
    run1, _ = cpu_reference_step(m, 1)
    run1()
    t = time.perf_counter()
    run1()
    per_layer = time.perf_counter() - t
    layers = max(1, min(int(target_s / 4 / max(per_layer, 1e-6)), max_layers))
    run, ops = cpu_reference_step(m, layers, seed=1)
    run()  # warm-up
    times = []
    t_end = time.perf_counter() + target_s
    while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 50):
        t = time.perf_counter()
        run()
        times.append(time.perf_counter() - t)
    dt = statistics.median(times)
    return {"value": ops / dt / 1e12, "unit": "TOPS", "cores": cores, "kind": "port",
            "sample": f"{layers} of {LAYERS} layers x 4 GEMMs + the PLE model projection (torch._int_mm, M={m}); "
                      f"median of {len(times)} passes, {sum(times):.1f} s of CPU time"}


def run_reference_arm(args, world, rank):
    if rank != 0:
        return
    from oracle import cpu_int8

    cores = cpu_int8.set_threads()
    run1, _ = cpu_reference_step(args.m, 1)
    run1()
    t = time.perf_counter()
    run1()
    per_layer = time.perf_counter() - t
    # each step a bounded sample of the layer set so the whole run stays within minutes
    layers = max(1, min(LAYERS, int(args.ref_step_s / max(per_layer, 1e-6))))
    run, ops = cpu_reference_step(args.m, layers, seed=1)
    for _ in range(args.warmup):
        run()
    t = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = (time.perf_counter() - t) / args.steps
    tops = ops / dt / 1e12
    step_ms_full = dt * 1e3 * macs_per_token() * 2 * args.m / ops  # projected to the full layer set
    sample = (f"{layers} of {LAYERS} layers x 4 GEMMs + the PLE model projection per step "
              f"(torch._int_mm, M={args.m})")
    line = {"metric": "W8A8 GEMM TOPS, prefill linear set @3658 tok (config 1)", "value": tops, "unit": "TOPS",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
            "ms_full_layer_set": step_ms_full, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
            "config": {"workload": f"config 1: 35-layer prefill linear set, M={args.m} (sampled)",
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": tops, "unit": "TOPS", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": tops, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--m", type=int, default=M_TOKENS, help="tokens per prompt (rows of every GEMM)")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="decoder layers per step (fewer only for profiling captures; the metric is quoted at 35)")
    ap.add_argument("--only", default=None, help="profile one projection shape only (qkv/o/gate_up/down/ple_model)")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--decode-steps", type=int, default=200)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-step-s", type=float, default=4.0, help="CPU seconds per reference-arm step")
    ap.add_argument("--sweep", action="store_true", help="config 3: per-shape M sweep, padded vs unpadded (own JSON line)")
    ap.add_argument("--gemm-table", action="store_true",
                    help="each config-1 shape against cuBLASLt (torch._int_mm), bit-exact check (own JSON line)")
    ap.add_argument("--no-config4", action="store_true", help="skip the config-4 prompts / sharded LM head objects")
    ap.add_argument("--no-fused", action="store_true", help="skip the fused gate/up glue object")
    ap.add_argument("--no-attention", action="store_true", help="skip the prefill attention object")
    ap.add_argument("--only-attention", action="store_true",
                    help="time only the prefill attention object (--steps / --warmup replays; profiling captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    world, rank, local = dist_setup(args)

    if args.impl == "reference":
        run_reference_arm(args, world, rank)
        return

    import importlib
    import torch.distributed as dist

    w8 = importlib.import_module("gemma-npu_b200")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        pk = peaks()
        stream = torch.cuda.Stream(device=dev)
        if args.only_attention:
            att = attention_bench(w8, dev, stream, args.m, args.steps, args.warmup, world)
            if rank == 0:
                print(json.dumps({"attention": att}), flush=True)
            return
        if args.gemm_table:
            table = gemm_table(w8, dev, stream, args.steps, args.warmup)
            if rank == 0:
                print(json.dumps({"metric": "W8A8 GEMM us per launch vs cuBLASLt, config-1 shapes @M=3658",
                                  "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                                  "dtype": "int8", "data": "synthetic", "table": table}), flush=True)
            return
        if args.sweep:
            table = sweep(w8, dev, stream, args.steps, args.warmup)
            if rank == 0:
                print(json.dumps({"metric": "W8A8 GEMM TOPS sweep (config 3)", "unit": "TOPS", "n_gpus": 1,
                                  "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                                  "dtype": "int8", "data": "synthetic", "sweep": table}), flush=True)
            return
        work = build_prefill(w8, dev, args.m, only=args.only, seed=rank, layers=args.layers)

        def prefill_step():
            for xq, wq, c, _ in work["calls"]:
                w8.mm_i8_nk(xq, wq, c)

        graph = capture(prefill_step, stream)
        sampler = ClockSampler(local) if rank == 0 else None
        ms = timed(lambda: graph.replay(), args.steps, args.warmup, stream, world)
        clocks = sampler.stop() if sampler else None
        ms_step = ms / args.steps
        tops_rank = work["ops"] / (ms_step * 1e-3) / 1e12
        value = world * tops_rank  # each rank processed one prompt per step
        # Denominator by the length of the timed region: a region under a second runs at
        # the burst clock (the measured burst cuBLAS rate), a longer one settles at the
        # power-capped clock (the measured sustained rate).  Both are reported.
        region_s = ms / 1e3
        sustained = region_s >= SUSTAINED_REGION_S
        int8_burst = INT8_PER_BF16 * pk["bf16_tflops"]
        int8_sustained = INT8_PER_BF16 * pk["bf16_tflops_sustained"]
        int8_peak = int8_sustained if sustained else int8_burst
        traffic = gemm_traffic_per_launch(args.layers, args.m) if args.only is None else None
        line = {
            "metric": "W8A8 GEMM TOPS, prefill linear set @3658 tok (config 1)"
            if args.only is None else f"W8A8 GEMM TOPS, {args.only} @M={args.m}",
            "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic (seeded N(0,1) activations / N(0,0.02) weights, W8A8-quantised)",
            "config": {"workload": f"config 1: {args.layers} layers x (qkv, o, gate_up, down) + PLE model projection, "
                                   f"M={args.m} tokens per rank", "m_tokens": args.m,
                       "gemms_per_step": len(work["calls"]), "parallelism": f"dp{world} (one prompt per GPU)",
                       "l2": "no flush: every step streams 1.24 GB of weights, 1.45 GB of activations and "
                             "9.3 GB of int32 outputs (>> 126 MB L2)"},
            "pct_int8_peak": 100.0 * tops_rank / int8_peak,
            "pct_int8_peak_burst": 100.0 * tops_rank / int8_burst,
            "pct_int8_peak_sustained": 100.0 * tops_rank / int8_sustained,
            "pct_int8_nominal": 100.0 * tops_rank / NOMINAL_INT8_TOPS,
            "gpu_launches": args.steps * len(work["calls"]),
            "roofline": {"bound": "tensor", "achieved": tops_rank, "peak": int8_peak, "unit": "TOP/s",
                         "frac": tops_rank / int8_peak, "traffic": None if traffic is None else traffic["bytes"],
                         "peak_kind": "sustained" if sustained else "burst", "timed_region_s": region_s,
                         "peak_note": f"2 x {pk['source']} dense bf16 cuBLAS rate (B200 dense int8 = 2 x bf16): "
                                      f"burst 2 x {pk['bf16_tflops']}, sustained 2 x {pk['bf16_tflops_sustained']} "
                                      f"TFLOP/s; burst when the timed region is under {SUSTAINED_REGION_S:.0f} s",
                         "algorithmic_bytes_per_launch": work["bytes"] / len(work["calls"]),
                         "traffic_note": None if traffic is None else traffic["note"]},
            "clocks": clocks,
        }
        del graph
        if not args.no_e2e and args.only is None:
            e_ms, bi, bo = e2e_prefill(w8, work, dev, args.e2e_steps, 1, world, dequant=True)
            line["e2e"] = {"value": world * work["ops"] / (e_ms * 1e-3) / 1e12, "unit": "TOPS",
                           "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo, "ms_per_step": e_ms,
                           "steps": args.e2e_steps,
                           "path": "gemma_npu_b200.gemm_dequant per GEMM (int32 accumulate + the _deq epilogue, "
                                   "config 0's operation): pinned int8 activations + fp32 row scales H2D, bf16 "
                                   "results D2H; copies in, GEMMs and copies out on three streams"}
            e_ms, bi, bo = e2e_prefill(w8, work, dev, args.e2e_steps, 1, world, dequant=False)
            line["e2e_int32"] = {"value": world * work["ops"] / (e_ms * 1e-3) / 1e12, "unit": "TOPS",
                                 "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo, "ms_per_step": e_ms,
                                 "steps": args.e2e_steps,
                                 "path": "gemma_npu_b200.mm_i8_nk per GEMM: pinned int8 activations H2D, int32 results "
                                         "D2H (pipeline.py's Prefill.gemm data flow); same three-stream pipeline"}
        if not args.no_decode and args.only is None:
            step, nbytes, launches, head, (istep, ibytes, ilaunches), fstep = build_decode(w8, work, dev)
            dgraph = capture(step, stream)
            dms = timed(lambda: dgraph.replay(), args.decode_steps, args.warmup, stream, world)
            per = dms / args.decode_steps
            gbs = nbytes / (per * 1e-3) / 1e9
            del dgraph
            hx, hq, hsc, hlog = head
            hgraph = capture(lambda: w8.lm_head_logits(hx, hq, hsc, SOFTCAP, out=hlog), stream)
            hms = timed(lambda: hgraph.replay(), args.decode_steps, args.warmup, stream, world) / args.decode_steps
            del hgraph
            head_bytes = VOCAB * HIDDEN + 2 * VOCAB + 2 * HIDDEN + 4 * VOCAB
            head_gbs = head_bytes / (hms * 1e-3) / 1e9
            igraph = capture(istep, stream)
            ims = timed(lambda: igraph.replay(), args.decode_steps, args.warmup, stream, world) / args.decode_steps
            del igraph
            igbs = ibytes / (ims * 1e-3) / 1e9
            fgraph = capture(fstep, stream)
            fms = timed(lambda: fgraph.replay(), args.decode_steps, args.warmup, stream, world) / args.decode_steps
            del fgraph
            rest_gbs = nbytes / ((per - fms) * 1e-3) / 1e9 if per > fms else None
            line["decode_gemv"] = {
                "metric": "int8 GEMV GB/s, decode chain (config 2: 140 layer GEMVs + LM head 262144x1536, "
                          "softcap and greedy argmax fused, one CUDA graph, each GEMV ordered after the previous one)",
                "value": world * gbs, "unit": "GB/s", "ms_per_token": per, "bytes_per_token": nbytes,
                "launches_per_token": launches,
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                             "frac": gbs / pk["hbm_gbs"], "traffic": None,
                             "peak_note": f"{pk['source']} HBM copy bandwidth"},
                "lm_head": {"us": hms * 1e3, "bytes": head_bytes, "gbs": head_gbs,
                            "frac": head_gbs / pk["hbm_gbs"],
                            "note": "the 262144x1536 head GEMV alone (402.7 MB int8): the chain's per-layer "
                                    "GEMVs (3.1-18.9 MB) are bound by the dependent step's latency, not bandwidth"},
                "dependent_step_floor": {
                    "us": fms * 1e3, "us_per_launch": fms * 1e3 / launches,
                    "remainder_us": (per - fms) * 1e3, "remainder_gbs": rest_gbs,
                    "remainder_frac": None if rest_gbs is None else rest_gbs / pk["hbm_gbs"],
                    "note": "the same 141-launch dependent chain with every GEMV cut to K = 16 (same grids, "
                            "activation hand-offs and outputs, no weight stream): the latency floor of a "
                            "dependent batch-1 step; remainder = chain - floor, the time the weight bytes add "
                            "(a remainder_frac above 1 means part of the weight stream is hidden under the "
                            "steps' latency: each GEMV issues its first weight loads before waiting for the "
                            "previous one)"},
                "layer_gemvs_independent": {"us": ims * 1e3, "bytes": ibytes, "gbs": igbs,
                                            "frac": igbs / pk["hbm_gbs"], "launches": ilaunches,
                                            "note": "the chain's 140 layer GEMVs with no dependence between them, "
                                                    "round-robin on 4 streams inside one graph so that they overlap"}}
        if not args.no_fused and args.only is None:
            line["fused_gelu_up"] = fused_gelu_up(w8, work, dev, stream, 10, 3, world)
            line["fused_layer"] = fused_layer(w8, dev, stream, args.m, 5, 3, world)
            line["glue_rows"] = glue_rows(w8, dev, stream, args.m, 10, 3, world, pk)
            line["qkv_paths"] = qkv_paths(w8, dev, stream, args.m, 10, 3, world)
        if not args.no_attention and args.only is None:
            line["attention"] = attention_bench(w8, dev, stream, args.m, 10, 3, world)
            line["prefill_gpu"] = prefill_gpu(w8, dev, stream, args.m, 3, 3, world)
            # Gemma E2B's count of KV-shared layers comes from its config.json, absent here:
            # 20 of 35 is an assumption that exercises the shared-layer path at scale.
            line["prefill_gpu_kv_shared"] = prefill_gpu(w8, dev, stream, args.m, 3, 3, world, kv_shared=20)
        if not args.no_config4 and args.only is None:
            line["config4"] = {"prompts_dp": prompts_dp(w8, dev, stream, world, rank, 3, 3),
                               "lm_head_sharded": sharded_head(w8, dev, stream, world, 50, 5, pk)}
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_reference_rate(args.m)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
