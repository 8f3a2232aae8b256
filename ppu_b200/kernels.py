"""Drop-in replacement for the reference's ``qwen35_fused.kernels`` (text-decoder operators).

Same function names, keyword-only arguments, output shapes and ``ValueError`` checks as
qwen35_fused/kernels.py; every call launches hand-written sm_100a CUDA through the C ABI
(``include/qwen35_b200.h``) on the current stream. Outputs are allocated with ``torch.empty``
from PyTorch's caching allocator (so calls stay CUDA-graph capturable); the K/V cache, conv
state and recurrent state are updated in place exactly where the reference does so.
Triton tile knobs (``block_n``, ``block_k``, ``block_v``, ``splits``) are accepted and ignored.

Added beyond the reference: ``quantize_rows`` / ``a8w8_linear`` / ``int8_gemm`` (the A8W8
linear of explore_runtime_quantization.py:129-181), ``gemm`` (prefill projection with fused
epilogues), ``fused_gemv`` (decode GEMV with fused norm / residual / SwiGLU), ``attn_decode`` and
``delta_decode`` (one-kernel decode mixers), and a batch dimension for ``gqa_decode_attention``.
"""

from __future__ import annotations

import torch

from . import lib as L

BF16 = torch.bfloat16


def _rows_and_width(x: torch.Tensor) -> tuple[int, int]:
    """kernels.py:16-21."""
    if not x.is_cuda:
        raise ValueError("fused kernels require a CUDA tensor")
    if not x.is_contiguous():
        raise ValueError("fused kernels require contiguous input")
    return x.numel() // x.shape[-1], x.shape[-1]


def _need_bf16(*ts: torch.Tensor) -> None:
    for t in ts:
        if t.dtype != BF16:
            raise ValueError(f"expected bfloat16 tensor, got {t.dtype}")


def _s(t: torch.Tensor) -> int:
    return L.stream_of(t.device)


# ---------------------------------------------------------------------------- norms / activations
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Qwen3.5 RMSNorm: FP32 reduction and direct BF16 output (kernels.py:44-53)."""
    rows, width = _rows_and_width(x)
    if weight.numel() != width:
        raise ValueError(f"weight has {weight.numel()} values, expected {width}")
    _need_bf16(x, weight)
    out = torch.empty_like(x)
    L.call("q35_rms_norm", L.ptr(x), L.ptr(weight.contiguous()), L.ptr(out), rows, width, eps, _s(x))
    return out


def residual_add_rms_norm(residual, update, weight, eps: float = 1e-6):
    """Return ``(residual + update, RMSNorm(residual + update))`` in one launch (kernels.py:85-112)."""
    if residual.shape != update.shape or residual.dtype != update.dtype:
        raise ValueError("residual and update must have identical shape and dtype")
    rows, width = _rows_and_width(residual)
    if not update.is_contiguous():
        raise ValueError("update must be contiguous")
    _need_bf16(residual, weight)
    residual_out = torch.empty_like(residual)
    norm_out = torch.empty_like(residual)
    L.call("q35_residual_add_rms_norm", L.ptr(residual), L.ptr(update), L.ptr(weight.contiguous()),
           L.ptr(residual_out), L.ptr(norm_out), rows, width, eps, _s(residual))
    return residual_out, norm_out


def gated_rms_norm(x, gate, weight, eps: float = 1e-6):
    """Qwen3.5 gated RMSNorm with eager-compatible intermediate rounding (kernels.py:139-155)."""
    if x.shape != gate.shape:
        raise ValueError("x and gate must have identical shape")
    rows, width = _rows_and_width(x)
    if not gate.is_contiguous():
        raise ValueError("gate must be contiguous")
    _need_bf16(x, gate, weight)
    out = torch.empty_like(x)
    L.call("q35_gated_rms_norm", L.ptr(x), L.ptr(gate), L.ptr(weight.contiguous()), L.ptr(out), rows, width,
           eps, _s(x))
    return out


def silu_and_mul(packed: torch.Tensor) -> torch.Tensor:
    """Apply SiLU to the first half and multiply the second half (kernels.py:170-180)."""
    rows, packed_width = _rows_and_width(packed)
    if packed_width % 2:
        raise ValueError("packed last dimension must be even")
    _need_bf16(packed)
    width = packed_width // 2
    out = torch.empty((*packed.shape[:-1], width), device=packed.device, dtype=packed.dtype)
    L.call("q35_silu_and_mul", L.ptr(packed), L.ptr(out), rows, width, _s(packed))
    return out


def sigmoid_mul(x: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """kernels.py:276-282."""
    if x.shape != gate.shape or not x.is_contiguous() or not gate.is_contiguous():
        raise ValueError("x and gate must be contiguous tensors with identical shape")
    _rows_and_width(x)
    _need_bf16(x, gate)
    out = torch.empty_like(x)
    L.call("q35_sigmoid_mul", L.ptr(x), L.ptr(gate), L.ptr(out), x.numel(), _s(x))
    return out


def attention_gate_mul(x: torch.Tensor, packed_qgkv: torch.Tensor, head_dim: int) -> torch.Tensor:
    """Multiply attention output by a gate stored inside packed QGKV output (kernels.py:312-333)."""
    if not x.is_contiguous() or not packed_qgkv.is_contiguous():
        raise ValueError("attention gate tensors must be contiguous")
    hidden = x.shape[-1]
    if packed_qgkv.shape[:-1] != x.shape[:-1]:
        raise ValueError("attention output and packed projection rows do not match")
    _rows_and_width(x)
    _need_bf16(x, packed_qgkv)
    out = torch.empty_like(x)
    rows = x.numel() // hidden
    L.call("q35_attention_gate_mul", L.ptr(x), L.ptr(packed_qgkv), L.ptr(out), rows, hidden,
           packed_qgkv.shape[-1], head_dim, _s(x))
    return out


# ---------------------------------------------------------------------------- GEMV / GEMM
def ppu_swiglu_gemv(x: torch.Tensor, packed_weight: torch.Tensor, *, block_n: int = 8) -> torch.Tensor:
    """Decode-only packed gate/up projection with fused SwiGLU (kernels.py:232-263)."""
    if x.ndim != 3 or x.shape[:2] != (1, 1) or x.dtype != BF16:
        raise ValueError("SwiGLU GEMV expects BF16 x[1,1,K]")
    if packed_weight.ndim != 2 or packed_weight.shape[0] % 2:
        raise ValueError("packed SwiGLU weight must have shape [2N,K]")
    if packed_weight.shape[1] != x.shape[-1] or packed_weight.dtype != x.dtype:
        raise ValueError("SwiGLU GEMV input and weight dimensions do not match")
    if not x.is_contiguous() or not packed_weight.is_contiguous():
        raise ValueError("SwiGLU GEMV tensors must be contiguous")
    if not x.is_cuda:
        raise ValueError("fused kernels require a CUDA tensor")
    if block_n not in (2, 4, 8):
        raise ValueError("SwiGLU GEMV block_n must be 2, 4 or 8")
    n = packed_weight.shape[0] // 2
    out = torch.empty((1, 1, n), device=x.device, dtype=x.dtype)
    L.call("q35_swiglu_gemv", L.ptr(x), L.ptr(packed_weight), L.ptr(out), n, x.shape[-1], _s(x))
    return out


def fused_gemv(weight, x=None, *, prologue=L.PRO_PLAIN, epilogue=L.EPI_STORE, norm_weight=None, w_scale=None,
               token=None, embed=None, resid=None, n_out=None, eps: float = 1e-6):
    """Batch-1 decode GEMV with the decoder's fused prologue/epilogue (``q35_gemv``).

    Returns the output vector (STORE / SWIGLU) or the updated ``resid`` (RESIDUAL / EMBED)."""
    int8 = weight.dtype == torch.int8
    k = weight.shape[1]
    rows = weight.shape[0]
    if n_out is None:
        n_out = rows // 2 if epilogue == L.EPI_SWIGLU else rows
    out = None
    if epilogue != L.EPI_RESIDUAL:
        out = torch.empty(n_out, device=weight.device, dtype=BF16)
    d = L.GemvDesc(weight=L.ptr(weight), w_scale=L.ptr(w_scale), input=L.ptr(x), norm_weight=L.ptr(norm_weight),
                   token=L.ptr(token), embed=L.ptr(embed), resid_out=L.ptr(resid), out=L.ptr(out), n_out=n_out, k=k,
                   vocab=0 if embed is None else embed.shape[0], prologue=prologue, epilogue=epilogue,
                   int8=int(int8), eps=eps)
    L.check(L.load().q35_gemv(L.C.byref(d), L.stream_of(weight.device)), "q35_gemv")
    return out if out is not None else resid


def gemm(a: torch.Tensor, weight: torch.Tensor, *, epilogue=L.EPI_STORE, out=None, tc: bool = False) -> torch.Tensor:
    """Prefill projection ``a [M,K] @ weight [N,K]^T`` (bf16; RESIDUAL adds into ``out`` in place).
    ``tc=True`` runs the tcgen05/TMEM kernel, otherwise the warp-level MMA kernel."""
    _need_bf16(a, weight)
    m, k = a.reshape(-1, a.shape[-1]).shape
    n = weight.shape[0] // 2 if epilogue == L.EPI_SWIGLU else weight.shape[0]
    if epilogue == L.EPI_RESIDUAL:
        if out is None:
            raise ValueError("RESIDUAL epilogue needs the residual tensor as `out`")
    elif out is None:
        out = torch.empty((*a.shape[:-1], n), device=a.device, dtype=BF16)
    L.call("q35_gemm_tc" if tc else "q35_gemm_bf16", L.ptr(a), L.ptr(weight), L.ptr(out), m, n, k, epilogue, _s(a))
    return out


def gemm_a8w8_tc(qa, sx, qw, sw, *, epilogue=L.EPI_STORE, out=None) -> torch.Tensor:
    """A8W8 prefill projection on tcgen05: int8 ``qa [M,K]`` / ``qw [N,K]`` with row scales."""
    m, k = qa.shape
    n = qw.shape[0] // 2 if epilogue == L.EPI_SWIGLU else qw.shape[0]
    if out is None:
        out = torch.empty((m, n), device=qa.device, dtype=BF16)
    L.call("q35_gemm_tc_a8w8", L.ptr(qa), L.ptr(sx), L.ptr(qw), L.ptr(sw), L.ptr(out), m, n, k, epilogue, _s(qa))
    return out


def tc_error() -> int:
    """Error word of the tensor-core kernels (0 = every bounded wait completed): the projection
    GEMMs' code, | 0x100 when a chunked DeltaNet kernel's wait gave up, | 0x200 when the tcgen05
    prefill attention's did."""
    lib = L.load()
    gemm = int(lib.q35_tc_error())
    delta = int(lib.q35_delta_chunk_error())
    attn = int(lib.q35_prefill_attention_tc_error())
    return gemm | (0x100 if delta else 0) | (0x200 if attn else 0)


def set_gemm_tc_pairs(on: bool) -> None:
    """Process-wide: tensor-core projections on SM pairs (cta_group::2, default) or single SMs."""
    L.call("q35_set_gemm_tc_pairs", 1 if on else 0)


# ---------------------------------------------------------------------------- A8W8
def quantize_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Weight-side per-row symmetric int8 (explore_runtime_quantization.py:143-155):
    ``s = amax/127`` (1 for a zero row), ``q = clamp(rne(x / s), -127, 127)``."""
    rows, width = _rows_and_width(x)
    _need_bf16(x)
    q = torch.empty(x.shape, device=x.device, dtype=torch.int8)
    scale = torch.empty((*x.shape[:-1], 1), device=x.device, dtype=torch.float32)
    L.call("q35_quantize_rows", L.ptr(x), L.ptr(q), L.ptr(scale), rows, width, _s(x))
    return q, scale


def scaled_int8_quant(x: torch.Tensor, scale=None, azp=None, symmetric: bool = True):
    """Activation-side dynamic per-token int8 quantisation, the call the reference makes through
    vllm (explore_runtime_quantization.py:167-172): returns ``(q int8, scale fp32 [rows, 1], None)``
    with vllm's semantics (``scale = amax/127``, ``q = sat(rne(x * 127/amax))``, zero rows give
    zero codes and scale). Only the dynamic symmetric form is provided."""
    if scale is not None or azp is not None or not symmetric:
        raise ValueError("scaled_int8_quant: only dynamic symmetric per-token quantisation is supported")
    rows, width = _rows_and_width(x)
    _need_bf16(x)
    q = torch.empty(x.shape, device=x.device, dtype=torch.int8)
    s = torch.empty((rows, 1), device=x.device, dtype=torch.float32)
    L.call("q35_quantize_tokens", L.ptr(x), L.ptr(q), L.ptr(s), rows, width, _s(x))
    return q, s, None


def int8_gemm(qx: torch.Tensor, qw: torch.Tensor) -> torch.Tensor:
    """Exact int32 ``qx @ qw^T``."""
    m, k = qx.reshape(-1, qx.shape[-1]).shape
    acc = torch.empty((m, qw.shape[0]), device=qx.device, dtype=torch.int32)
    L.call("q35_int8_gemm_i32", L.ptr(qx), L.ptr(qw), L.ptr(acc), m, qw.shape[0], k, _s(qx))
    return acc


def a8w8_linear(x: torch.Tensor, qw: torch.Tensor, w_scale: torch.Tensor) -> torch.Tensor:
    """Dynamic per-token A8W8 linear: ``bf16((float(q_x q_w^T) * s_x) * s_w)``."""
    _rows_and_width(x)
    _need_bf16(x)
    m, k = x.reshape(-1, x.shape[-1]).shape
    n = qw.shape[0]
    if m == 1:
        out = fused_gemv(qw, x.reshape(-1).contiguous(), w_scale=w_scale.reshape(-1).contiguous())
        return out.reshape(*x.shape[:-1], n)
    size = L.load().q35_a8w8_linear_workspace_size(m, k)
    ws = torch.empty(size, device=x.device, dtype=torch.uint8)
    out = torch.empty((*x.shape[:-1], n), device=x.device, dtype=BF16)
    L.call("q35_a8w8_linear", L.ptr(x), L.ptr(qw), L.ptr(w_scale), L.ptr(out), m, n, k, L.ptr(ws), size, _s(x))
    return out


# ---------------------------------------------------------------------------- attention
def qgkv_norm_rope(packed_qgkv, q_weight, k_weight, cos, sin, *, q_heads, kv_heads, dim, rotary_dim,
                   cache_key=None, cache_value=None, cache_start=None):
    """Layout packed Q+gate/K/V and fuse Q/K RMSNorm with partial RoPE (kernels.py:507-573)."""
    if not packed_qgkv.is_contiguous():
        raise ValueError("packed QGKV must be contiguous")
    batch, seq_len, packed_width = packed_qgkv.shape
    expected = 2 * q_heads * dim + 2 * kv_heads * dim
    if packed_width != expected:
        raise ValueError(f"packed QGKV width {packed_width}, expected {expected}")
    cos = cos.to(BF16).contiguous()
    sin = sin.to(BF16).contiguous()
    if cos.shape != (batch, seq_len, rotary_dim) or sin.shape != cos.shape:
        raise ValueError(f"RoPE shape {tuple(cos.shape)}, expected {(batch, seq_len, rotary_dim)}")
    _rows_and_width(packed_qgkv)
    q = torch.empty((batch, q_heads, seq_len, dim), device=packed_qgkv.device, dtype=packed_qgkv.dtype)
    if cache_key is not None:
        if cache_value is None or cache_start is None:
            raise ValueError("cache key, value and start must be provided together")
        if cache_key.shape[:2] != (batch, kv_heads) or cache_key.shape[-1] != dim:
            raise ValueError("static K cache shape does not match QGKV")
        if cache_value.shape != cache_key.shape:
            raise ValueError("static K/V cache shapes must match")
        k, v = cache_key, cache_value
        kv_len = cache_key.shape[-2]
        start = cache_start if cache_start.dtype == torch.int64 else cache_start.to(torch.int64)
    else:
        k = torch.empty((batch, kv_heads, seq_len, dim), device=packed_qgkv.device, dtype=packed_qgkv.dtype)
        v = torch.empty_like(k)
        kv_len = seq_len
        start = None
    L.call("q35_qgkv_norm_rope", L.ptr(packed_qgkv), L.ptr(q_weight.contiguous()), L.ptr(k_weight.contiguous()),
           L.ptr(cos), L.ptr(sin), L.ptr(q), L.ptr(k), L.ptr(v), L.ptr(start), batch, seq_len, q_heads, kv_heads,
           dim, rotary_dim, kv_len, 1e-6, _s(packed_qgkv))
    return q, k, v


def gqa_decode_attention(q, cache_keys, cache_values, valid_length, scale: float, *, splits: int = 4,
                         block_n: int = 64):
    """One decode attention step over a static cache (kernels.py:1031-1090); batch >= 1 here.

    ``q [B,H,1,D]``, caches ``[B,KVH,L,D]``, ``valid_length`` a device scalar including the
    current token. Returns ``[B, 1, H*D]``."""
    if q.ndim != 4 or q.shape[2] != 1:
        raise ValueError("GQA decode attention expects q[B,H,1,D]")
    if cache_keys.ndim != 4 or cache_keys.shape[0] != q.shape[0]:
        raise ValueError("static K cache must be [B,KVH,L,D]")
    if cache_values.shape != cache_keys.shape:
        raise ValueError("static K/V cache shapes must match")
    if not q.is_contiguous() or not cache_keys.is_contiguous() or not cache_values.is_contiguous():
        raise ValueError("GQA decode attention tensors must be contiguous")
    batch, heads, head_dim = q.shape[0], q.shape[1], q.shape[3]
    kv_heads, cache_len = cache_keys.shape[1], cache_keys.shape[2]
    if head_dim != cache_keys.shape[3] or heads % kv_heads:
        raise ValueError("GQA decode attention head layout does not match cache")
    n_valid = valid_length.reshape(-1)[:1].to(torch.int64)
    size = L.load().q35_gqa_decode_workspace_size(batch, heads, kv_heads, head_dim, cache_len)
    ws = torch.empty(size, device=q.device, dtype=torch.uint8)
    ws[:1024].zero_()  # the split tickets
    out = torch.empty((batch, 1, heads * head_dim), device=q.device, dtype=q.dtype)
    L.call("q35_gqa_decode_attention", L.ptr(q), L.ptr(cache_keys), L.ptr(cache_values), L.ptr(n_valid), scale,
           L.ptr(out), batch, heads, kv_heads, head_dim, cache_len, L.ptr(ws), size, _s(q))
    return out


def attn_decode(packed, q_weight, k_weight, inv_freq, cache_key, cache_value, cache_len, rope_pos, *, q_heads,
                kv_heads, rotary_dim, eps: float = 1e-6):
    """Whole decode attention mixer in one kernel: ``packed [B, 2HqD+2HkvD]`` -> gated ``[B, Hq*D]``.

    Writes the token's K/V at row ``cache_len`` (not advanced here)."""
    batch = packed.shape[0]
    dim = cache_key.shape[-1]
    max_len = cache_key.shape[2]
    size = L.load().q35_attn_decode_workspace_size(batch, q_heads, kv_heads, dim, max_len)
    ws = torch.empty(size, device=packed.device, dtype=torch.uint8)
    ws[:1024].zero_()  # the split tickets
    out = torch.empty((batch, q_heads * dim), device=packed.device, dtype=BF16)
    L.call("q35_attn_decode", L.ptr(packed), L.ptr(q_weight), L.ptr(k_weight), L.ptr(inv_freq), L.ptr(cache_key),
           L.ptr(cache_value), L.ptr(cache_len), L.ptr(rope_pos), L.ptr(out), batch, q_heads, kv_heads, dim,
           rotary_dim, max_len, eps, L.ptr(ws), size, _s(packed))
    return out


def prefill_attention(q, k, v, scale: float, q_offset: int = 0) -> torch.Tensor:
    """Causal GQA attention ``q [B,Hq,L,D]`` over ``k/v [B,Hkv,S,D]`` -> ``[B, L, Hq*D]``."""
    b, hq, length, dim = q.shape
    out = torch.empty((b, length, hq * dim), device=q.device, dtype=BF16)
    L.call("q35_prefill_attention", L.ptr(q), L.ptr(k), L.ptr(v), L.ptr(out), b, hq, k.shape[1], length,
           k.shape[2], q_offset, dim, scale, _s(q))
    return out


def prefill_attention_tc(q, k, v, scale: float, kv_len: int | None = None) -> torch.Tensor:
    """The decoder's tcgen05 causal attention: ``q [B,Hq,L,256]`` (Hq = 4 Hkv) over the first L
    rows of ``k/v [B,Hkv,S,256]`` (queries at rows 0 .. L-1) -> ``[B, L, Hq*256]``. V is passed to
    the kernel transposed, padded with zeros to a multiple of 64 keys, as the decoder writes it."""
    b, hq, length, dim = q.shape
    stride = (length + 63) // 64 * 64
    vt = torch.zeros((b, v.shape[1], dim, stride), device=v.device, dtype=BF16)
    vt[..., :length] = v[:, :, :length].transpose(-1, -2)
    out = torch.empty((b, length, hq * dim), device=q.device, dtype=BF16)
    nbytes = int(L.load().q35_prefill_attention_tc_workspace_size(b, k.shape[1], length))
    ws = torch.zeros(nbytes, device=q.device, dtype=torch.uint8)
    L.call("q35_prefill_attention_tc", L.ptr(q), L.ptr(k), L.ptr(vt), L.ptr(out), b, hq, k.shape[1], length,
           k.shape[2] if kv_len is None else kv_len, stride, scale, L.ptr(ws), nbytes, _s(q))
    return out


# ---------------------------------------------------------------------------- DeltaNet
def causal_conv1d_fused(x: torch.Tensor, weight: torch.Tensor, state: torch.Tensor) -> torch.Tensor:
    """Causal depthwise conv + SiLU, updating ``state`` in place (kernels.py:659-710)."""
    if x.ndim != 3 or weight.ndim != 2 or state.ndim != 3:
        raise ValueError("expected x[B,L,C], weight[C,K], state[B,C,K]")
    if not x.is_contiguous() or not weight.is_contiguous() or not state.is_contiguous():
        raise ValueError("causal conv tensors must be contiguous")
    batch, seq_len, input_stride = x.shape
    channels, kernel_size = weight.shape
    if input_stride < channels or state.shape != (batch, channels, kernel_size):
        raise ValueError("causal conv shapes do not match")
    _rows_and_width(x)
    out = torch.empty((batch, seq_len, channels), device=x.device, dtype=x.dtype)
    L.call("q35_causal_conv1d", L.ptr(x), L.ptr(weight), L.ptr(state), L.ptr(out), batch, seq_len, input_stride,
           channels, kernel_size, _s(x))
    return out


def delta_recurrent_fused(qkv, packed_projection, a_log, dt_bias, state, *, block_v: int = 8,
                          precompute_factors: bool = False):
    """Sequential gated-delta recurrence for prefill and decode; ``state`` updated in place
    (kernels.py:854-937). ``qkv [B,L,3HD]``; ``packed_projection`` holds ``[qkv,z,a,b]``."""
    if qkv.ndim != 3 or packed_projection.ndim != 3 or state.ndim != 4:
        raise ValueError("invalid delta recurrent tensor rank")
    if not qkv.is_contiguous() or not packed_projection.is_contiguous() or not state.is_contiguous():
        raise ValueError("delta recurrent tensors must be contiguous")
    batch, seq_len, qkv_width = qkv.shape
    _, heads, dim, value_dim = state.shape
    if dim != value_dim or qkv_width != 3 * heads * dim:
        raise ValueError("delta recurrent dimensions do not match")
    packed_width = packed_projection.shape[-1]
    need = qkv_width + heads * dim + 2 * heads
    if packed_width < need:
        raise ValueError(f"packed projection width {packed_width} is smaller than {need}")
    if state.dtype != torch.float32:
        raise ValueError("recurrent state must be float32")
    _rows_and_width(qkv)
    out = torch.empty((batch, seq_len, heads, dim), device=qkv.device, dtype=qkv.dtype)
    L.call("q35_delta_recurrent", L.ptr(qkv), L.ptr(packed_projection), L.ptr(a_log.contiguous()),
           L.ptr(dt_bias.contiguous()), L.ptr(state), L.ptr(out), batch, seq_len, heads, dim, packed_width, _s(qkv))
    return out


def delta_chunked_fused(qkv, packed_projection, a_log, dt_bias, state):
    """``delta_recurrent_fused`` in chunked WY form (chunk 64, FP32): same inputs/outputs and
    in-place state update; the algorithm of HF torch_chunk_gated_delta_rule (prefill)."""
    batch, seq_len, qkv_width = qkv.shape
    _, heads, dim, _ = state.shape
    if qkv_width != 3 * heads * dim or not qkv.is_contiguous() or not packed_projection.is_contiguous():
        raise ValueError("delta chunked tensors do not match")
    out = torch.empty((batch, seq_len, heads, dim), device=qkv.device, dtype=qkv.dtype)
    size = L.load().q35_delta_chunked_workspace_size(batch, heads, seq_len)
    ws = torch.empty(max(size, 16), device=qkv.device, dtype=torch.uint8)
    L.call("q35_delta_chunked", L.ptr(qkv), L.ptr(packed_projection), L.ptr(a_log.contiguous()),
           L.ptr(dt_bias.contiguous()), L.ptr(state), L.ptr(out), batch, seq_len, heads, dim,
           packed_projection.shape[-1], L.ptr(ws), size, _s(qkv))
    return out


def delta_chunked_conv_fused(packed_projection, conv_weight, conv_state, a_log, dt_bias, state):
    """``causal_conv1d_fused`` on the [q k v] columns (4 taps, zero history) followed by
    ``delta_chunked_fused``, in one prep + scan pair: ``packed_projection [B, L, rows]`` (raw
    projection) -> ``[B, L, H, D]``; updates ``conv_state`` and ``state`` in place."""
    batch, seq_len, rows = packed_projection.shape
    _, heads, dim, _ = state.shape
    if seq_len < 4 or not packed_projection.is_contiguous() or conv_state.shape[-1] != 4:
        raise ValueError("delta chunked conv tensors do not match")
    out = torch.empty((batch, seq_len, heads, dim), device=packed_projection.device, dtype=BF16)
    size = L.load().q35_delta_chunked_workspace_size(batch, heads, seq_len)
    ws = torch.empty(max(size, 16), device=packed_projection.device, dtype=torch.uint8)
    L.call("q35_delta_chunked_conv", L.ptr(packed_projection), L.ptr(conv_weight.contiguous()), L.ptr(conv_state),
           L.ptr(a_log.contiguous()), L.ptr(dt_bias.contiguous()), L.ptr(state), L.ptr(out), batch, seq_len, heads,
           dim, rows, L.ptr(ws), size, _s(packed_projection))
    return out


def delta_decode(packed, conv_weight, conv_state, a_log, dt_bias, norm_weight, state, *, eps: float = 1e-6):
    """Whole DeltaNet decode mixer in one kernel: ``packed [B, rows]`` -> ``[B, H*Dv]`` (gated-normed)."""
    batch = packed.shape[0]
    heads, dim = state.shape[1], state.shape[2]
    out = torch.empty((batch, heads * dim), device=packed.device, dtype=BF16)
    L.call("q35_delta_decode", L.ptr(packed), L.ptr(conv_weight), L.ptr(conv_state), L.ptr(a_log), L.ptr(dt_bias),
           L.ptr(norm_weight), L.ptr(state), L.ptr(out), batch, heads, dim, packed.shape[-1], eps, _s(packed))
    return out


# ---------------------------------------------------------------------------- LM head
def lm_head_argmax(hidden: torch.Tensor, weight: torch.Tensor, *, block_n: int = 16, block_k: int = 128,
                   norm_weight: torch.Tensor | None = None, eps: float = 1e-6) -> torch.Tensor:
    """Greedy token id without materialising the BF16 logits (kernels.py:1146-1185); int64 [1,1]."""
    if hidden.shape != (1, weight.shape[1]) or hidden.dtype != BF16:
        raise ValueError("lm_head_argmax supports BF16 batch=1 hidden vectors")
    if not hidden.is_contiguous() or not weight.is_contiguous():
        raise ValueError("LM head tensors must be contiguous")
    if not hidden.is_cuda:
        raise ValueError("fused kernels require a CUDA tensor")
    vocab, hidden_size = weight.shape
    size = L.load().q35_lm_head_workspace_size(1)
    ws = torch.zeros(max(size, 16), device=hidden.device, dtype=torch.uint8)
    out = torch.empty((1, 1), device=hidden.device, dtype=torch.int64)
    L.call("q35_lm_head_argmax", L.ptr(hidden), L.ptr(norm_weight), L.ptr(weight), L.ptr(out), 1, vocab,
           hidden_size, eps, L.ptr(ws), size, _s(hidden))
    return out


def lm_head_shard_keys(hidden: torch.Tensor, weight_shard: torch.Tensor, row_offset: int, vocab: int, *,
                       norm_weight: torch.Tensor | None = None, eps: float = 1e-6,
                       workspace: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Top-1 keys of ``hidden [n, 2048]`` (n <= 8) over rows ``[row_offset, row_offset + rows)`` of a
    ``[vocab, 2048]`` table held as ``weight_shard [rows, 2048]``: int64 ``[n]``, the maximum of which
    over all shards encodes the token ``lm_head_argmax`` gives (see ``lm_keys_to_tokens``). The
    multi-GPU split of kernels.py:1093-1185; ``workspace`` (zeroed once, reusable) and ``out`` may be
    passed to keep the call allocation-free."""
    if hidden.dim() != 2 or hidden.dtype != BF16 or weight_shard.dtype != BF16:
        raise ValueError("lm_head_shard_keys expects BF16 hidden [n, K] and a BF16 weight shard")
    if not hidden.is_cuda or not weight_shard.is_cuda:
        raise ValueError("fused kernels require a CUDA tensor")
    if not hidden.is_contiguous() or not weight_shard.is_contiguous():
        raise ValueError("LM head tensors must be contiguous")
    n, k = hidden.shape
    if weight_shard.dim() != 2 or weight_shard.shape[1] != k:
        raise ValueError("weight shard must be [rows, hidden_size]")
    size = L.load().q35_lm_shard_workspace_size()
    if workspace is None:
        workspace = torch.zeros(size, device=hidden.device, dtype=torch.uint8)
    if out is None:
        out = torch.empty(n, device=hidden.device, dtype=torch.int64)
    L.call("q35_lm_head_shard_keys", L.ptr(hidden), n, L.ptr(norm_weight), L.ptr(weight_shard), row_offset,
           weight_shard.shape[0], vocab, k, eps, L.ptr(out), L.ptr(workspace), workspace.numel(), _s(hidden))
    return out


def lm_keys_to_tokens(keys: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Token ids encoded by reduced shard keys (int64 ``[n]`` -> int64 ``[n]``)."""
    if keys.dtype != torch.int64 or not keys.is_cuda or not keys.is_contiguous():
        raise ValueError("keys must be a contiguous CUDA int64 tensor")
    if out is None:
        out = torch.empty_like(keys)
    L.call("q35_lm_keys_to_tokens", L.ptr(keys), keys.numel(), L.ptr(out), _s(keys))
    return out


# ---------------------------------------------------------------------------- vision tower
def gemm_bias(a: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, *, epilogue=L.EPI_BIAS, out=None):
    """Biased projection on tcgen05 (the vision tower's nn.Linear layers): ``epilogue(a @ weight^T +
    bias)`` with EPI_BIAS, EPI_BIAS_GELU_TANH or EPI_BIAS_GELU; bf16 ``[M, N]``."""
    _need_bf16(a, weight, bias)
    m, k = a.reshape(-1, a.shape[-1]).shape
    n = weight.shape[0]
    if out is None:
        out = torch.empty((*a.shape[:-1], n), device=a.device, dtype=BF16)
    L.call("q35_gemm_tc_bias", L.ptr(a), L.ptr(weight), L.ptr(bias), L.ptr(out), m, n, k, epilogue, _s(a))
    return out


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """kernels.py:1188-1222: LayerNorm over the last dimension (FP32 statistics, bf16 out)."""
    rows, width = _rows_and_width(x)
    _need_bf16(x, weight, bias)
    out = torch.empty_like(x)
    L.call("q35_layer_norm", L.ptr(x), L.ptr(weight), L.ptr(bias), L.ptr(out), rows, width, eps, _s(x))
    return out


def residual_add_layer_norm(residual: torch.Tensor, update: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                            eps: float = 1e-6) -> tuple[torch.Tensor, torch.Tensor]:
    """kernels.py:1225-1287: ``residual_out = bf16(residual + update)``, ``LayerNorm(residual_out)``."""
    if residual.shape != update.shape:
        raise ValueError("vision residual tensors must have identical shape")
    rows, width = _rows_and_width(residual)
    _rows_and_width(update)
    _need_bf16(residual, update, weight, bias)
    residual_out = torch.empty_like(residual)
    norm_out = torch.empty_like(residual)
    L.call("q35_residual_add_layer_norm", L.ptr(residual), L.ptr(update), L.ptr(weight), L.ptr(bias),
           L.ptr(residual_out), L.ptr(norm_out), rows, width, eps, _s(residual))
    return residual_out, norm_out


def position_embed_add(hidden: torch.Tensor, embedding_table: torch.Tensor, indices: torch.Tensor,
                       interpolation_weight: torch.Tensor) -> torch.Tensor:
    """kernels.py:1290-1336: ``hidden + bf16(sum_k w_k * table[idx_k])`` per row (FP32 sum)."""
    if hidden.ndim != 2 or not hidden.is_contiguous():
        raise ValueError("vision hidden tensor must be contiguous [rows,width]")
    rows, width = hidden.shape
    neighbors = indices.shape[-1]
    if indices.shape != interpolation_weight.shape or indices.shape[0] != rows:
        raise ValueError("position interpolation tensors do not match hidden rows")
    if not hidden.is_cuda:
        raise ValueError("fused kernels require a CUDA tensor")
    _need_bf16(hidden, embedding_table)
    idx = indices.to(device=hidden.device, dtype=torch.int64).contiguous()
    wts = interpolation_weight.to(device=hidden.device, dtype=torch.float32).contiguous()
    table = embedding_table.contiguous()
    out = torch.empty_like(hidden)
    L.call("q35_position_embed_add", L.ptr(hidden), L.ptr(table), L.ptr(idx), L.ptr(wts), L.ptr(out), rows, width,
           neighbors, _s(hidden))
    return out


def vision_qkv_rope(packed_qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *, heads: int,
                    dim: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """kernels.py:336-416: packed Vision QKV ``[tokens, 3*heads*dim]`` to BHLD ``[1, heads, tokens,
    dim]`` q / k / v with RoPE on q and k, one launch."""
    if packed_qkv.ndim != 2 or not packed_qkv.is_contiguous():
        raise ValueError("packed Vision QKV must be contiguous [tokens,3*hidden]")
    tokens, packed_width = packed_qkv.shape
    if packed_width != 3 * heads * dim:
        raise ValueError(f"packed Vision QKV width {packed_width}, expected {3 * heads * dim}")
    cos = cos.contiguous()
    sin = sin.contiguous()
    if cos.shape != (tokens, dim) or sin.shape != cos.shape:
        raise ValueError(f"Vision RoPE shape {tuple(cos.shape)}, expected {(tokens, dim)}")
    if not packed_qkv.is_cuda:
        raise ValueError("fused kernels require a CUDA tensor")
    _need_bf16(packed_qkv)
    c32 = cos.to(device=packed_qkv.device, dtype=torch.float32).contiguous()
    s32 = sin.to(device=packed_qkv.device, dtype=torch.float32).contiguous()
    q = torch.empty((1, heads, tokens, dim), device=packed_qkv.device, dtype=packed_qkv.dtype)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    L.call("q35_vision_qkv_rope", L.ptr(packed_qkv), L.ptr(c32), L.ptr(s32), L.ptr(q), L.ptr(k), L.ptr(v), tokens,
           heads, dim, _s(packed_qkv))
    return q, k, v


def vision_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """Bidirectional attention over one image: ``[1, heads, L, 64]`` q/k/v -> ``[L, heads*64]``
    (the vision attention of integration.py:616-700 with a single ``cu_seqlens`` segment)."""
    if q.shape != k.shape or q.shape != v.shape or q.dim() != 4 or q.shape[0] != 1:
        raise ValueError("vision attention expects q, k, v of one shape [1, heads, tokens, dim]")
    if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
        raise ValueError("fused kernels require contiguous input")
    if not q.is_cuda:
        raise ValueError("fused kernels require a CUDA tensor")
    _need_bf16(q, k, v)
    _, heads, tokens, dim = q.shape
    out = torch.empty((tokens, heads * dim), device=q.device, dtype=BF16)
    L.call("q35_vision_attention", L.ptr(q), L.ptr(k), L.ptr(v), L.ptr(out), tokens, heads, dim, scale, _s(q))
    return out


__all__ = [
    "rms_norm", "residual_add_rms_norm", "gated_rms_norm", "silu_and_mul", "ppu_swiglu_gemv", "sigmoid_mul",
    "attention_gate_mul", "qgkv_norm_rope", "causal_conv1d_fused", "delta_recurrent_fused",
    "gqa_decode_attention", "lm_head_argmax", "quantize_rows", "scaled_int8_quant", "int8_gemm", "a8w8_linear", "gemm",
    "fused_gemv", "attn_decode", "prefill_attention", "delta_decode", "delta_chunked_fused",
    "lm_head_shard_keys", "lm_keys_to_tokens",
    "gemm_bias", "layer_norm", "residual_add_layer_norm", "position_embed_add", "vision_qkv_rope", "vision_attention",
]
