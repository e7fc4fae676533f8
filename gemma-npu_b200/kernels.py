"""Torch-facing wrappers of the sm_100a W8A8 kernels.

B200 counterpart of the reference's kernel module `npu_kernels.py` plus the
quant/dequant glue of `pipeline.py` / `gemma_npu.py`:

    mm_i8(a, b, c) -> c          npu_kernels.py:59-64   (int8 [M,K] @ int8 [K,N] -> int32)
    use_device() / use_npu()     npu_kernels.py:25-26   (per-thread device selection)
    quant_rows(x) -> (q, s)      pipeline.py:49-52, gemma_npu.py:37-42
    dequant(acc, sx, sw)         pipeline.py:55-57, gemma_npu.py:45-47
    int8_linear(x, wq, sw)       gemma_npu.py:155-156   (torch._weight_int8pack_mm)
    gelu_up_quant(x, sx, w, sw)  pipeline.py:102-107   (k_gelu fused onto the gate/up GEMM)
    rms_quant(h, w, eps)         pipeline.py:66-69     (k_in)
    post_norm_quant(y, res, ..)  pipeline.py:95-99, 110-114 (k_post_attn / k_post_ff)
    attn_out_quant(o)            pipeline.py:88-92     (k_attn_out)
    qkv_norm_rope(y, cos, sin,..)pipeline.py:72-86     (k_qkv)
    attention_prefill(q, k, v, W)pipeline.py:139-180   (full / sliding-window attention)

Every function validates dtype/shape/layout on the host, passes raw device
pointers and torch's current CUDA stream to the C ABI, and raises a W8Error
subclass on a non-zero status.  Inputs must already live on a CUDA device:
nothing here copies to or from the host, and nothing falls back to the CPU.
Unlike the reference kernel, no shape needs padding to the tile (M, N any;
K a multiple of 16).
"""
import torch

from . import _lib
from ._lib import W8_B_KN, W8_B_NK

# Tile of the tcgen05 GEMM (rows x columns x K per pipeline stage).  Informational:
# callers need not pad to it (the reference's BLOCK_M = BLOCK_N = 512, BLOCK_K = 128).
BLOCK_M = 128
BLOCK_N = 256
BLOCK_K = 128


def use_device(device=None):
    """Select the CUDA device for the calling thread (the reference's use_npu()).

    CUDA's current device is per thread, like Triton's active driver in the
    reference: a worker thread that launches GEMMs calls this first.
    """
    if device is None:
        device = torch.cuda.current_device()
    torch.cuda.set_device(device)


# The reference's name for the same per-thread selection (npu_kernels.py:25-26).
use_npu = use_device


def _stream(t):
    return ctypes_ptr(torch.cuda.current_stream(t.device).cuda_stream)


def ctypes_ptr(v):
    return v if v else None


def _need(cond, msg):
    if not cond:
        raise ValueError(msg)


def _check_matrix(t, name, dtype):
    _need(isinstance(t, torch.Tensor), f"{name} must be a tensor")
    _need(t.is_cuda, f"{name} must be on a CUDA device (got {t.device}); there is no CPU path")
    _need(t.dtype == dtype, f"{name} must be {dtype} (got {t.dtype})")
    _need(t.dim() == 2, f"{name} must be 2-D (got shape {tuple(t.shape)})")
    _need(t.stride(1) == 1 or t.shape[1] <= 1, f"{name} must be row-major with unit column stride")


def _ld(t):
    return t.stride(0) if t.shape[0] > 1 else max(t.shape[1], t.stride(0))


# Stream-K counters for the GEMMs, one zero-filled buffer per (device, stream): the
# kernel leaves it zero after every call, and calls on one stream never overlap.
_WORKSPACES = {}
_MIN_WORKSPACE_WORDS = 1 << 16


def _workspace(device, stream, nbytes):
    key = (device.index, stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() * 4 < nbytes:
        words = max(_MIN_WORKSPACE_WORDS, -(-nbytes // 4))
        ws = torch.zeros(words, dtype=torch.int32, device=device)
        _WORKSPACES[key] = ws
    return ws


def _mm(a, b, layout, c, M, N, K):
    stream = _stream(a)
    nbytes = _lib.lib().w8_mm_i8_workspace_bytes(M, N, K)
    ws = _workspace(a.device, stream, nbytes)
    _lib.call("w8_mm_i8_ws", a.data_ptr(), _ld(a), b.data_ptr(), _ld(b), layout, c.data_ptr(), _ld(c),
              M, N, K, ws.data_ptr(), ws.numel() * 4, stream)


def _check_vector(t, name, dtype, n):
    _need(isinstance(t, torch.Tensor) and t.is_cuda, f"{name} must be a CUDA tensor")
    _need(t.dtype == dtype, f"{name} must be {dtype} (got {t.dtype})")
    _need(t.dim() == 1 and t.shape[0] == n, f"{name} must have shape ({n},) (got {tuple(t.shape)})")
    _need(t.is_contiguous(), f"{name} must be contiguous")


def mm_i8(a, b, c):
    """c[M,N] (int32) = a[M,K] (int8) @ b[K,N] (int8), exact; writes into c and returns it.

    Same contract as the reference's mm_i8 (npu_kernels.py:59-64) without its
    multiple-of-512 precondition.  b is the reference layout [K,N]; see
    mm_i8_nk for the resident [N,K] layout.
    """
    _check_matrix(a, "a", torch.int8)
    _check_matrix(b, "b", torch.int8)
    _check_matrix(c, "c", torch.int32)
    M, K = a.shape
    _need(b.shape[0] == K, f"inner sizes differ: a {tuple(a.shape)}, b {tuple(b.shape)}")
    N = b.shape[1]
    _need(tuple(c.shape) == (M, N), f"c must be ({M}, {N}) (got {tuple(c.shape)})")
    _need(a.device == b.device == c.device, "a, b, c must be on one device")
    _mm(a, b, W8_B_KN, c, M, N, K)
    return c


def mm_i8_nk(a, w, c):
    """c[M,N] (int32) = a[M,K] @ w[N,K]^T: the GEMM over a resident K-major weight."""
    _check_matrix(a, "a", torch.int8)
    _check_matrix(w, "w", torch.int8)
    _check_matrix(c, "c", torch.int32)
    M, K = a.shape
    N = w.shape[0]
    _need(w.shape[1] == K, f"inner sizes differ: a {tuple(a.shape)}, w {tuple(w.shape)}")
    _need(tuple(c.shape) == (M, N), f"c must be ({M}, {N}) (got {tuple(c.shape)})")
    _need(a.device == w.device == c.device, "a, w, c must be on one device")
    _mm(a, w, W8_B_NK, c, M, N, K)
    return c


def gemm_dequant(a, w, sx, sw, out=None):
    """bf16 [M,N] = dequant(a @ w^T) with the dequant fused into the GEMM epilogue.

    a int8 [M,K] with per-row scales sx fp32 [M]; w int8 [N,K] with per-channel
    scales sw fp32 [N].  Bit-identical to dequant(mm_i8_nk(a, w, c), sx, sw).
    """
    _check_matrix(a, "a", torch.int8)
    _check_matrix(w, "w", torch.int8)
    M, K = a.shape
    N = w.shape[0]
    _need(w.shape[1] == K, f"inner sizes differ: a {tuple(a.shape)}, w {tuple(w.shape)}")
    _check_vector(sx, "sx", torch.float32, M)
    _check_vector(sw, "sw", torch.float32, N)
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    _check_matrix(out, "out", torch.bfloat16)
    _need(tuple(out.shape) == (M, N), f"out must be ({M}, {N})")
    _lib.call("w8_gemm_dequant_bf16", a.data_ptr(), _ld(a), w.data_ptr(), _ld(w), W8_B_NK,
              sx.data_ptr(), sw.data_ptr(), out.data_ptr(), _ld(out), M, N, K, _stream(a))
    return out


def pack_gelu_up(w, sw):
    """Reorder a gate/up weight [2I, K] (gate rows, then up rows) and its scales [2I] for
    gelu_up_quant: packed row 256t + j = gate row 128t + j, packed row 256t + 128 + j =
    up row I + 128t + j (j < 128), so each 256-column GEMM tile holds matching gate and
    up columns.  Done once, when the resident weight is built.  I % 128 == 0."""
    two_i = w.shape[0]
    _need(two_i % 256 == 0, f"2 * I = {two_i} must be a multiple of 256")
    _need(sw.shape == (two_i,), f"sw must have shape ({two_i},)")
    inter = two_i // 2
    blk = torch.arange(inter // 128, device=w.device)[:, None] * 128 + torch.arange(128, device=w.device)
    idx = torch.stack([blk, blk + inter], dim=1).reshape(-1)
    return w.index_select(0, idx).contiguous(), sw.index_select(0, idx).contiguous()


# Row-absmax scratch of the gate/up glue, zero between calls, one per (device, stream).
_ABSMAX = {}


def _absmax_scratch(device, stream, rows):
    key = (device.index, stream)
    buf = _ABSMAX.get(key)
    if buf is None or buf.numel() < rows:
        buf = torch.zeros(max(rows, 4096), dtype=torch.float32, device=device)
        _ABSMAX[key] = buf
    return buf


def gelu_up_quant(x, sx, w_packed, sw_packed, q=None, s=None, y=None):
    """k_gelu (pipeline.py:102-107) fused onto the gate/up GEMM.

    x int8 [T, K] with per-row scales sx fp32 [T]; w_packed int8 [2I, K] and sw_packed
    fp32 [2I] from pack_gelu_up.  Returns (q int8 [T, I], s fp32 [T]) =
    _quant(bf16(gelu_tanh(_deq(gate)) * _deq(up))).  `y` (bf16 [T, I]) receives the
    pre-quant activation; it is allocated when not given.
    """
    _check_matrix(x, "x", torch.int8)
    _check_matrix(w_packed, "w_packed", torch.int8)
    T, K = x.shape
    two_i = w_packed.shape[0]
    _need(w_packed.shape[1] == K, f"inner sizes differ: x {tuple(x.shape)}, w {tuple(w_packed.shape)}")
    _need(two_i % 256 == 0, f"2 * I = {two_i} must be a multiple of 256")
    inter = two_i // 2
    _check_vector(sx, "sx", torch.float32, T)
    _check_vector(sw_packed, "sw_packed", torch.float32, two_i)
    if q is None:
        q = torch.empty((T, inter), dtype=torch.int8, device=x.device)
    if s is None:
        s = torch.empty((T,), dtype=torch.float32, device=x.device)
    if y is None:
        y = torch.empty((T, inter), dtype=torch.bfloat16, device=x.device)
    _check_matrix(q, "q", torch.int8)
    _check_matrix(y, "y", torch.bfloat16)
    _need(tuple(q.shape) == (T, inter) and tuple(y.shape) == (T, inter), f"q and y must be ({T}, {inter})")
    _check_vector(s, "s", torch.float32, T)
    stream = _stream(x)
    absmax = _absmax_scratch(x.device, stream, T)
    _lib.call("w8_gemm_gelu_up_quant", x.data_ptr(), _ld(x), w_packed.data_ptr(), _ld(w_packed),
              sx.data_ptr(), sw_packed.data_ptr(), T, inter, K, y.data_ptr(), _ld(y), absmax.data_ptr(),
              q.data_ptr(), _ld(q), s.data_ptr(), stream)
    return q, s


def _bf16_rows(t, name, n=None):
    _check_matrix(t, name, torch.bfloat16)
    if n is not None:
        _need(t.shape[1] == n, f"{name} must have {n} columns (got {t.shape[1]})")


def _bf16_vec(t, name, n):
    _check_vector(t, name, torch.bfloat16, n)


def rms_quant(h, w, eps, q=None, s=None):
    """k_in (pipeline.py:66-69): (q int8 [T, N], s fp32 [T]) = _quant(bf16(_rms(h, w, eps))).

    h bf16 [T, N] (N <= 2048, N % 8 == 0), w bf16 [N] (the input_layernorm weight)."""
    _bf16_rows(h, "h")
    T, N = h.shape
    _bf16_vec(w, "w", N)
    q = torch.empty((T, N), dtype=torch.int8, device=h.device) if q is None else q
    s = torch.empty((T,), dtype=torch.float32, device=h.device) if s is None else s
    _check_matrix(q, "q", torch.int8)
    _check_vector(s, "s", torch.float32, T)
    _lib.call("w8_rms_quant_bf16", h.data_ptr(), _ld(h), w.data_ptr(), float(eps), q.data_ptr(), _ld(q),
              s.data_ptr(), T, N, _stream(h))
    return q, s


def post_norm_quant(y, res, w1, w2, eps, h=None, q=None, s=None):
    """The glue after the o / down GEMMs, on y = the GEMM's dequantised bf16 output:
    h = bf16(res + bf16(_rms(y, w1))); with w2 (k_post_attn, pipeline.py:95-99)
    q, s = _quant(bf16(_rms(h, w2))), without (k_post_ff, pipeline.py:110-114) q, s = _quant(h).
    Returns (h, q, s); `h` may be `res` itself (in-place residual update)."""
    _bf16_rows(y, "y")
    T, N = y.shape
    _bf16_rows(res, "res", N)
    _need(res.shape[0] == T, "res must have the rows of y")
    _bf16_vec(w1, "w1", N)
    if w2 is not None:
        _bf16_vec(w2, "w2", N)
    h = torch.empty((T, N), dtype=torch.bfloat16, device=y.device) if h is None else h
    q = torch.empty((T, N), dtype=torch.int8, device=y.device) if q is None else q
    s = torch.empty((T,), dtype=torch.float32, device=y.device) if s is None else s
    _bf16_rows(h, "h", N)
    _check_matrix(q, "q", torch.int8)
    _check_vector(s, "s", torch.float32, T)
    _lib.call("w8_post_norm_quant_bf16", y.data_ptr(), _ld(y), res.data_ptr(), _ld(res), w1.data_ptr(),
              None if w2 is None else w2.data_ptr(), float(eps), h.data_ptr(), _ld(h), q.data_ptr(), _ld(q),
              s.data_ptr(), T, N, _stream(y))
    return h, q, s


def ple_gate_quant(y, ple, q=None, s=None):
    """k_ple_gate (pipeline.py:117-121) on y = the PLE gate GEMM's dequantised bf16 output
    [T, n] and this layer's per-layer input `ple` [T, n] (bf16, any row pitch, e.g. a
    [:, layer] slice of the [T, layers, n] per-layer inputs):
    q, s = _quant(bf16(bf16(gelu_tanh(y)) * ple)).  Returns (q, s)."""
    _bf16_rows(y, "y")
    T, N = y.shape
    _bf16_rows(ple, "ple", N)
    _need(ple.shape[0] == T, "ple must have the rows of y")
    q = torch.empty((T, N), dtype=torch.int8, device=y.device) if q is None else q
    s = torch.empty((T,), dtype=torch.float32, device=y.device) if s is None else s
    _check_matrix(q, "q", torch.int8)
    _check_vector(s, "s", torch.float32, T)
    _lib.call("w8_ple_gate_quant_bf16", y.data_ptr(), _ld(y), ple.data_ptr(), _ld(ple), q.data_ptr(), _ld(q),
              s.data_ptr(), T, N, _stream(y))
    return q, s


def ple_out(y, res, w_post, scalar, eps, w_next=None, h=None, q=None, s=None):
    """k_ple_out (pipeline.py:124-127) on y = the PLE projection GEMM's dequantised bf16
    output: h = bf16(bf16(res + bf16(_rms(y, w_post))) * scalar), `scalar` the layer's bf16
    layer_scalar (a 1-element tensor or a float; pass a float inside a CUDA graph capture,
    where reading a device tensor is not allowed).  Returns h; with `w_next` (the next
    layer's input norm weight) the next layer's k_in runs in the same pass and
    (h, q, s) is returned, q, s = _quant(bf16(_rms(h, w_next))).  `h` may be `res`."""
    _bf16_rows(y, "y")
    T, N = y.shape
    _bf16_rows(res, "res", N)
    _need(res.shape[0] == T, "res must have the rows of y")
    _bf16_vec(w_post, "w_post", N)
    h = torch.empty((T, N), dtype=torch.bfloat16, device=y.device) if h is None else h
    _bf16_rows(h, "h", N)
    qp = sp = None
    if w_next is not None:
        _bf16_vec(w_next, "w_next", N)
        q = torch.empty((T, N), dtype=torch.int8, device=y.device) if q is None else q
        s = torch.empty((T,), dtype=torch.float32, device=y.device) if s is None else s
        _check_matrix(q, "q", torch.int8)
        _check_vector(s, "s", torch.float32, T)
        qp, sp = q.data_ptr(), s.data_ptr()
    _lib.call("w8_ple_out_bf16", y.data_ptr(), _ld(y), res.data_ptr(), _ld(res), w_post.data_ptr(),
              float(scalar), None if w_next is None else w_next.data_ptr(), float(eps), h.data_ptr(), _ld(h), qp,
              _ld(q) if q is not None else 0, sp, T, N, _stream(y))
    return h if w_next is None else (h, q, s)


def qkv_norm_rope(y, cos, sin, qw, kw, eps, heads, kv_heads, head_dim, shared=False, out=None):
    """k_qkv (pipeline.py:72-86) on y = the qkv GEMM's dequantised bf16 output [T, (H+2KV)*D]
    (or [T, H*D] when shared): returns (q [H, T, D], k [KV, T, D], v [KV, T, D]) bf16, slices of
    one head-major buffer `out` [H + 2KV, T, D]; a KV-shared layer returns (q, q, q)."""
    _bf16_rows(y, "y")
    T = y.shape[0]
    per_tok = heads if shared else heads + 2 * kv_heads
    _need(y.shape[1] == per_tok * head_dim, f"y must have {per_tok * head_dim} columns")
    _bf16_rows(cos, "cos", head_dim)
    _bf16_rows(sin, "sin", head_dim)
    _need(cos.shape[0] == T and sin.shape[0] == T and cos.stride(0) == sin.stride(0),
          "cos and sin must be [T, D] with the same pitch")
    _bf16_vec(qw, "qw", head_dim)
    if not shared and kv_heads:
        _bf16_vec(kw, "kw", head_dim)
    if out is None:
        out = torch.empty((per_tok, T, head_dim), dtype=torch.bfloat16, device=y.device)
    _need(out.dtype == torch.bfloat16 and out.is_cuda and tuple(out.shape) == (per_tok, T, head_dim)
          and out.stride(2) == 1, f"out must be bf16 ({per_tok}, {T}, {head_dim}) with unit stride along D")
    _lib.call("w8_qkv_norm_rope_bf16", y.data_ptr(), _ld(y), cos.data_ptr(), sin.data_ptr(), cos.stride(0),
              qw.data_ptr(), None if (shared or not kv_heads) else kw.data_ptr(), float(eps), out.data_ptr(),
              out.stride(0), out.stride(1), T, heads, kv_heads, head_dim, int(bool(shared)), _stream(y))
    q = out[:heads]
    if shared:
        return q, q, q
    return q, out[heads: heads + kv_heads], out[heads + kv_heads:]


def rope_tiles(cos, sin):
    """cos / sin [T, D] bf16 -> the 8-column tiled tables (cos_t, sin_t), each [D / 8, T, 8],
    that gemm_qkv_norm_rope(..., tiles=) reads with coalesced loads.  The tables depend only
    on the positions, so a prefill lays them out once and every layer with the same RoPE
    reuses them."""
    _need(isinstance(cos, torch.Tensor) and isinstance(sin, torch.Tensor) and cos.shape == sin.shape,
          "cos and sin must be tensors of one shape")
    T, D = cos.shape
    _need(D % 8 == 0, f"head_dim {D} must be a multiple of 8")
    return tuple(t.contiguous().reshape(T, D // 8, 8).transpose(0, 1).contiguous() for t in (cos, sin))


def gemm_qkv_norm_rope(xq, w, sx, sw, cos, sin, qw, kw, eps, heads, kv_heads, head_dim, shared=False, out=None,
                       tiles=None):
    """The qkv GEMM and k_qkv (pipeline.py:233-242 + :72-86): xq int8 [T, K] with row scales
    sx, the resident qkv weight w [N, K] with channel scales sw -> (q [H, T, D], k, v), the
    same bits as qkv_norm_rope(gemm_dequant(xq, w, sx, sw), ...).  head_dim 256 runs as one
    kernel (the glue in the GEMM's epilogue, one head per 256-column tile, no bf16 [T, N]
    intermediate); other head dims run the two kernels.  `tiles`: rope_tiles(cos, sin),
    the same tables laid out for the fused kernel's loads (same result bits)."""
    T = xq.shape[0]
    per_tok = heads if shared else heads + 2 * kv_heads
    _need(w.shape[0] == per_tok * head_dim, f"w must have {per_tok * head_dim} rows")
    if head_dim != 256:
        return qkv_norm_rope(gemm_dequant(xq, w, sx, sw), cos, sin, qw, kw, eps, heads, kv_heads, head_dim,
                             shared=shared, out=out)
    _check_matrix(xq, "xq", torch.int8)
    _check_matrix(w, "w", torch.int8)
    K = xq.shape[1]
    _need(w.shape[1] == K, f"inner sizes differ: xq {tuple(xq.shape)}, w {tuple(w.shape)}")
    _check_vector(sx, "sx", torch.float32, T)
    _check_vector(sw, "sw", torch.float32, w.shape[0])
    _bf16_rows(cos, "cos", head_dim)
    _bf16_rows(sin, "sin", head_dim)
    _need(cos.shape[0] == T and sin.shape[0] == T and cos.stride(0) == sin.stride(0),
          "cos and sin must be [T, D] with the same pitch")
    _bf16_vec(qw, "qw", head_dim)
    if not shared and kv_heads:
        _bf16_vec(kw, "kw", head_dim)
    if out is None:
        out = torch.empty((per_tok, T, head_dim), dtype=torch.bfloat16, device=xq.device)
    _need(out.dtype == torch.bfloat16 and out.is_cuda and tuple(out.shape) == (per_tok, T, head_dim)
          and out.stride(2) == 1, f"out must be bf16 ({per_tok}, {T}, {head_dim}) with unit stride along D")
    kw_ptr = None if (shared or not kv_heads) else kw.data_ptr()
    if tiles is None:
        _lib.call("w8_gemm_qkv_norm_rope", xq.data_ptr(), _ld(xq), w.data_ptr(), _ld(w), sx.data_ptr(),
                  sw.data_ptr(), T, heads, kv_heads, int(bool(shared)), cos.data_ptr(), sin.data_ptr(), cos.stride(0),
                  qw.data_ptr(), kw_ptr, float(eps), out.data_ptr(), out.stride(0), out.stride(1), K, _stream(xq))
    else:
        ct, st = tiles
        for t_, name in ((ct, "cos tiles"), (st, "sin tiles")):
            _need(isinstance(t_, torch.Tensor) and t_.is_cuda and t_.dtype == torch.bfloat16
                  and tuple(t_.shape) == (head_dim // 8, T, 8) and t_.stride(2) == 1 and (T == 1 or t_.stride(1) == 8),
                  f"{name} must be bf16 [{head_dim // 8}, {T}, 8] as rope_tiles returns them")
        _need(ct.stride(0) == st.stride(0), "cos and sin tiles must have the same pitch")
        _lib.call("w8_gemm_qkv_norm_rope_tiled", xq.data_ptr(), _ld(xq), w.data_ptr(), _ld(w), sx.data_ptr(),
                  sw.data_ptr(), T, heads, kv_heads, int(bool(shared)), ct.data_ptr(), st.data_ptr(), ct.stride(0),
                  qw.data_ptr(), kw_ptr, float(eps), out.data_ptr(), out.stride(0), out.stride(1), K, _stream(xq))
    q = out[:heads]
    if shared:
        return q, q, q
    return q, out[heads: heads + kv_heads], out[heads + kv_heads:]


def attention_prefill(q, k, v, window=0, out=None, schedule="tc"):
    """Prefill attention of one prompt from position 0 (pipeline.py:139-180): causal, with
    a sliding window when window > 0, scale 1.0, grouped-query heads.  q bf16 [H, T, D],
    k, v [KV, T, D] (unit stride along D; any head / token pitch); returns o [H, T, D].
    schedule "tc" runs the tcgen05 kernel, "mma" the warp-level mma.sync one."""
    _need(schedule in ("tc", "mma"), "schedule must be 'tc' or 'mma'")
    for t_, name in ((q, "q"), (k, "k"), (v, "v")):
        _need(isinstance(t_, torch.Tensor) and t_.is_cuda and t_.dtype == torch.bfloat16 and t_.dim() == 3
              and t_.stride(2) == 1, f"{name} must be a bf16 CUDA tensor [heads, T, D] with unit stride along D")
    H, T, D = q.shape
    KV = k.shape[0]
    _need(tuple(k.shape) == (KV, T, D) and tuple(v.shape) == (KV, T, D), "k and v must be [KV, T, D]")
    if out is None:
        out = torch.empty((H, T, D), dtype=torch.bfloat16, device=q.device)
    _need(out.dtype == torch.bfloat16 and tuple(out.shape) == (H, T, D) and out.stride(2) == 1,
          f"out must be bf16 ({H}, {T}, {D})")
    entry = "w8_attention_prefill_bf16" if schedule == "tc" else "w8_attention_prefill_mma_bf16"
    _lib.call(entry, q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0),
              k.stride(1), v.data_ptr(), v.stride(0), v.stride(1), out.data_ptr(), out.stride(0), out.stride(1),
              T, H, KV, D, int(window), _stream(q))
    return out


def attention_quant(q, k, v, window=0, xq=None, xs=None):
    """Prefill attention followed by k_attn_out (pipeline.py:139-180 then :88-92): returns
    the per-token _quant of the attention output, (xq int8 [T, H*D], xs fp32 [T]),
    bit-identical to attn_out_quant(attention_prefill(q, k, v, window)).  One kernel when
    head_dim is 256 with one KV head and a power-of-two head count <= 16 (the Gemma E2B
    sliding layers); the two-step path otherwise."""
    for t_, name in ((q, "q"), (k, "k"), (v, "v")):
        _need(isinstance(t_, torch.Tensor) and t_.is_cuda and t_.dtype == torch.bfloat16 and t_.dim() == 3
              and t_.stride(2) == 1, f"{name} must be a bf16 CUDA tensor [heads, T, D] with unit stride along D")
    H, T, D = q.shape
    KV = k.shape[0]
    _need(tuple(k.shape) == (KV, T, D) and tuple(v.shape) == (KV, T, D), "k and v must be [KV, T, D]")
    xq = torch.empty((T, H * D), dtype=torch.int8, device=q.device) if xq is None else xq
    xs = torch.empty((T,), dtype=torch.float32, device=q.device) if xs is None else xs
    _check_matrix(xq, "xq", torch.int8)
    _check_vector(xs, "xs", torch.float32, T)
    if D == 256 and KV == 1 and 1 <= H <= 16 and H & (H - 1) == 0:
        _lib.call("w8_attention_prefill_quant", q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0),
                  k.stride(1), v.data_ptr(), v.stride(0), v.stride(1), T, H, KV, D, int(window), xq.data_ptr(),
                  _ld(xq), xs.data_ptr(), _stream(q))
        return xq, xs
    return attn_out_quant(attention_prefill(q, k, v, window), xq, xs)


def attn_out_quant(o, q=None, s=None):
    """k_attn_out (pipeline.py:88-92): o bf16 [H, T, D] -> _quant of its [T, H*D] rows."""
    _need(isinstance(o, torch.Tensor) and o.is_cuda and o.dtype == torch.bfloat16 and o.dim() == 3,
          "o must be a bf16 CUDA tensor [H, T, D]")
    _need(o.stride(2) == 1, "o must have unit stride along D")
    H, T, D = o.shape
    q = torch.empty((T, H * D), dtype=torch.int8, device=o.device) if q is None else q
    s = torch.empty((T,), dtype=torch.float32, device=o.device) if s is None else s
    _check_matrix(q, "q", torch.int8)
    _check_vector(s, "s", torch.float32, T)
    _lib.call("w8_attn_out_quant_bf16", o.data_ptr(), o.stride(0), o.stride(1), q.data_ptr(), _ld(q), s.data_ptr(),
              T, H, D, _stream(o))
    return q, s


def quant_rows(x, q=None, s=None):
    """Per-row symmetric int8 quant of a bf16 or fp32 [T,K] tensor -> (q int8 [T,K], s fp32 [T]).

    The reference's _quant (pipeline.py:49-52) / _quant_rows (gemma_npu.py:37-42):
    s = max(absmax, 1e-8) / 127, q = clamp(round(x / s), -127, 127), bit-identical.
    """
    _need(isinstance(x, torch.Tensor) and x.is_cuda, "x must be a CUDA tensor; there is no CPU path")
    _need(x.dim() == 2 and (x.stride(1) == 1 or x.shape[1] <= 1), "x must be 2-D row-major")
    T, K = x.shape
    if q is None:
        q = torch.empty((T, K), dtype=torch.int8, device=x.device)
    if s is None:
        s = torch.empty((T,), dtype=torch.float32, device=x.device)
    _check_matrix(q, "q", torch.int8)
    _need(tuple(q.shape) == (T, K), f"q must be ({T}, {K})")
    _check_vector(s, "s", torch.float32, T)
    if x.dtype == torch.bfloat16:
        fn = "w8_quant_rows_bf16"
    elif x.dtype == torch.float32:
        fn = "w8_quant_rows_f32"
    else:
        raise ValueError(f"x must be bfloat16 or float32 (got {x.dtype})")
    _lib.call(fn, x.data_ptr(), _ld(x), q.data_ptr(), _ld(q), s.data_ptr(), T, K, _stream(x))
    return q, s


def dequant(acc, sx, sw, dtype=torch.bfloat16, out=None):
    """bf16 [T,N] = (float(acc) * sx[:,None]) * sw[None,:] (the reference's _deq, pipeline.py:55-57)."""
    _need(dtype == torch.bfloat16, "only bfloat16 output is implemented (the reference's dtype)")
    _check_matrix(acc, "acc", torch.int32)
    T, N = acc.shape
    _check_vector(sx, "sx", torch.float32, T)
    _check_vector(sw, "sw", torch.float32, N)
    if out is None:
        out = torch.empty((T, N), dtype=torch.bfloat16, device=acc.device)
    _check_matrix(out, "out", torch.bfloat16)
    _lib.call("w8_dequant_bf16", acc.data_ptr(), _ld(acc), sx.data_ptr(), sw.data_ptr(), out.data_ptr(),
              _ld(out), T, N, _stream(acc))
    return out


def int8_linear(x2d, wq, sw, out=None):
    """bf16 [T,N] = (x2d @ wq^T) * sw: the weight-only int8 GEMV of decode.

    The reference's cpu_int8_linear (gemma_npu.py:155-156), i.e.
    torch._weight_int8pack_mm(x_bf16, wq [N,K] int8, sw [N] bf16), within max-rel 1e-2:
    the GPU holds x as 16-bit fixed point per 16-element piece and sums exactly in int32.
    """
    _need(isinstance(x2d, torch.Tensor) and x2d.is_cuda, "x2d must be a CUDA tensor; there is no CPU path")
    if x2d.dtype != torch.bfloat16:
        x2d = x2d.to(torch.bfloat16)
    if x2d.stride(-1) != 1 or x2d.data_ptr() % 16 or (x2d.shape[0] > 1 and x2d.stride(0) % 8):
        x2d = x2d.contiguous()
    _check_matrix(x2d, "x2d", torch.bfloat16)
    _check_matrix(wq, "wq", torch.int8)
    T, K = x2d.shape
    N = wq.shape[0]
    _need(wq.shape[1] == K, f"inner sizes differ: x {tuple(x2d.shape)}, wq {tuple(wq.shape)}")
    _check_vector(sw, "sw", torch.bfloat16, N)
    if out is None:
        out = torch.empty((T, N), dtype=torch.bfloat16, device=x2d.device)
    _check_matrix(out, "out", torch.bfloat16)
    _lib.call("w8_int8_linear_bf16", x2d.data_ptr(), _ld(x2d), wq.data_ptr(), _ld(wq), sw.data_ptr(),
              out.data_ptr(), _ld(out), T, N, K, _stream(x2d))
    return out


def lm_head_logits(x, wq, sw, cap=0.0, out=None, argmax=False):
    """fp32 [N] logits of one token: cap * tanh(bf16(x @ wq^T * sw) / cap) (cap <= 0: no softcap).

    Int8Head.forward (gemma_npu.py:170-172) followed by the final logit softcap
    (pipeline.py:335-338), fused into the GEMV.  With argmax=True also the greedy token
    (gemma_npu.py:291, logits.argmax(); ties to the lowest id), folded inside the same
    kernel: returns (logits, token) with token a 0-dim int64 device tensor (argmax="key":
    the raw packed key of w8_lm_head_argmax_f32 as an int64 [1] tensor instead).
    """
    _need(isinstance(x, torch.Tensor) and x.is_cuda, "x must be a CUDA tensor")
    x = x.reshape(-1)
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    x = x.contiguous()
    _check_matrix(wq, "wq", torch.int8)
    N, K = wq.shape
    _need(x.shape[0] == K, f"x must have {K} elements (got {x.shape[0]})")
    _need(wq.is_contiguous(), "wq must be contiguous [N, K]")
    _check_vector(sw, "sw", torch.bfloat16, N)
    if out is None:
        out = torch.empty((N,), dtype=torch.float32, device=x.device)
    _check_vector(out, "out", torch.float32, N)
    if not argmax:
        _lib.call("w8_lm_head_f32", x.data_ptr(), wq.data_ptr(), sw.data_ptr(), float(cap or 0.0),
                  out.data_ptr(), N, K, _stream(x))
        return out
    best = torch.empty((1,), dtype=torch.int64, device=x.device)
    _lib.call("w8_lm_head_argmax_f32", x.data_ptr(), wq.data_ptr(), sw.data_ptr(), float(cap or 0.0),
              out.data_ptr(), N, K, best.data_ptr(), _stream(x))
    return out, (argmax_token(best) if argmax != "key" else best)


def monotone_bits(f):
    """fp32 value(s) -> int64 holding the order-preserving 32-bit key of the argmax."""
    u = f.float().reshape(-1).view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return torch.where(u >= 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)


def argmax_token(best):
    """Token id (0-dim int64 on the device) from the packed key of w8_lm_head_argmax_f32."""
    return (0xFFFFFFFF - (best & 0xFFFFFFFF))[0]

