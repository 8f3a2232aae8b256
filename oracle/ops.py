"""Operator-level CPU restatement of the reference's fused Qwen3.5 operators.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Every function states the
reference lines it follows. Citations are paths inside the reference project;
``HF:`` means transformers/models/qwen3_5/modeling_qwen3_5.py of transformers 5.5.0.

Rounding contract: wherever the reference materialises a BF16 tensor between two
operations (the eager-compatible rounding points documented in
qwen35_fused/kernels.py:74-78, 219-224, 466-471, 606-609, 1119-1121) the oracle
rounds to BF16 at the same place. Everything else is FP32.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

BF16 = torch.bfloat16


def _bf(x: torch.Tensor) -> torch.Tensor:
    return x.to(BF16)


def _silu32(x32: torch.Tensor) -> torch.Tensor:
    return x32 / (1.0 + torch.exp(-x32))


def _sigmoid32(x32: torch.Tensor) -> torch.Tensor:
    return 1.0 / (1.0 + torch.exp(-x32))


# --------------------------------------------------------------------------- norms
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Qwen RMSNorm with (1 + w) scaling.

    qwen35_fused/kernels.py:24-53; validate_kernels.py:57-60 (reference_rms);
    HF Qwen3_5RMSNorm.forward. FP32 reduction, one BF16 rounding at the end.
    """
    x32 = x.float()
    var = (x32 * x32).mean(-1, keepdim=True)
    return _bf(x32 * torch.rsqrt(var + eps) * (1.0 + weight.float()))


def residual_add_rms_norm(residual, update, weight, eps: float = 1e-6):
    """``(bf16(r + u), RMSNorm(bf16(r + u)))``; the sum is rounded before the norm.

    qwen35_fused/kernels.py:56-112 (rounding at :74-78).
    """
    added = _bf(residual.float() + update.float())
    return added, rms_norm(added, weight, eps)


def gated_rms_norm(x, gate, weight, eps: float = 1e-6):
    """``bf16(bf16(bf16(norm(x)) * w) * silu(gate))`` with a plain (not 1+w) weight.

    qwen35_fused/kernels.py:115-155; validate_kernels.py:63-68; HF Qwen3_5RMSNormGated.
    """
    x32 = x.float()
    var = (x32 * x32).mean(-1, keepdim=True)
    normed = _bf(x32 * torch.rsqrt(var + eps))
    weighted = _bf(normed.float() * weight.float())
    return _bf(weighted.float() * _silu32(gate.float()))


# --------------------------------------------------------------------------- activations
def silu_and_mul(packed: torch.Tensor) -> torch.Tensor:
    """``bf16(bf16(silu(gate)) * up)`` over a packed ``[..., 2N]`` row. kernels.py:158-180."""
    n = packed.shape[-1] // 2
    gate = packed[..., :n].float()
    up = packed[..., n:].float()
    return _bf(_bf(_silu32(gate)).float() * up)


def sigmoid_mul(x: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """``bf16(x * bf16(sigmoid(gate)))``. kernels.py:266-282."""
    return _bf(x.float() * _bf(_sigmoid32(gate.float())).float())


def attention_gate_mul(x: torch.Tensor, packed_qgkv: torch.Tensor, head_dim: int) -> torch.Tensor:
    """Output gate read from the packed Q|gate head blocks. kernels.py:285-333.

    For head ``h`` the gate occupies ``packed[h*2*D + D : (h+1)*2*D]``.
    """
    hidden = x.shape[-1]
    heads = hidden // head_dim
    lead = x.shape[:-1]
    gate = packed_qgkv[..., : 2 * hidden].reshape(*lead, heads, 2, head_dim)[..., 1, :]
    gate = gate.reshape(*lead, hidden)
    return sigmoid_mul(x, gate)


# --------------------------------------------------------------------------- linears
def linear(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """BF16 ``F.linear``: FP32 accumulation, one BF16 rounding.

    The reference calls ``F.linear`` on BF16 tensors (qwen35_fused/integration.py:183, 245,
    298). On the CPU, PyTorch's BF16 GEMM accumulates in FP32 and rounds once (checked
    against a float64 product in tests/test_oracle.py).
    """
    return F.linear(x, weight)


def swiglu_gemv(x: torch.Tensor, packed_weight: torch.Tensor) -> torch.Tensor:
    """Packed gate|up projection with SwiGLU. kernels.py:183-263; validate_kernels.py:215-221."""
    return silu_and_mul(linear(x, packed_weight))


# --------------------------------------------------------------------------- RoPE
def rope_inv_freq(rotary_dim: int = 64, theta: float = 1.0e7) -> torch.Tensor:
    """Default RoPE inverse frequencies, HF Qwen3_5TextRotaryEmbedding.compute_default_rope_parameters."""
    exponent = torch.arange(0, rotary_dim, 2, dtype=torch.int64).to(torch.float32) / rotary_dim
    return 1.0 / (theta ** exponent)


def rope_cos_sin(positions: torch.Tensor, inv_freq: torch.Tensor, mrope_section=(11, 11, 10)):
    """BF16 cos/sin tables ``[B, L, rotary_dim]`` for text or 3-axis M-RoPE positions.

    HF Qwen3_5TextRotaryEmbedding.forward + apply_interleaved_mrope: angles in FP32
    (``p * inv_freq``), frequencies of axis H/W interleaved at offsets 1/2 (stride 3),
    ``cat(freqs, freqs)``, cos/sin in FP32, cast to BF16.
    ``positions`` is ``[B, L]`` (all axes equal) or ``[3, B, L]``.
    """
    if positions.ndim == 2:
        positions = positions[None].expand(3, -1, -1)
    freqs = positions[..., None].to(torch.float32) * inv_freq.float()  # [3,B,L,half]
    out = freqs[0].clone()
    for axis, offset in ((1, 1), (2, 2)):
        length = mrope_section[axis] * 3
        idx = slice(offset, length, 3)
        out[..., idx] = freqs[axis][..., idx]
    emb = torch.cat((out, out), dim=-1)
    return _bf(emb.cos()), _bf(emb.sin())


def _norm_rope_heads(raw, weight, cos, sin, rotary_dim):
    """Per-head RMSNorm(1+w) then partial RoPE with the BF16 rounding of kernels.py:466-471.

    raw ``[B, L, H, D]``; cos/sin ``[B, L, R]`` BF16.
    """
    normed = rms_norm(raw, weight)  # bf16 [B,L,H,D]
    half = rotary_dim // 2
    rot = normed[..., :rotary_dim].float()
    rotated_half = torch.cat((-rot[..., half:], rot[..., :half]), dim=-1)  # exact in bf16
    c = cos.to(BF16).float()[:, :, None, :]
    s = sin.to(BF16).float()[:, :, None, :]
    front = _bf(_bf(rot * c).float() + _bf(rotated_half * s).float())
    return torch.cat((front, normed[..., rotary_dim:]), dim=-1)


def qgkv_norm_rope(packed_qgkv, q_weight, k_weight, cos, sin, *, q_heads, kv_heads, dim,
                   rotary_dim, cache_key=None, cache_value=None, cache_start=None):
    """Split packed ``[Q|G]*Hq || K*Hkv || V*Hkv``, Q/K RMSNorm + partial RoPE, optional
    static-cache write at ``cache_start``. kernels.py:419-573; validate_kernels.py:247-319.

    Returns ``q [B,Hq,L,D]`` and ``k, v [B,Hkv,L,D]`` (the cache tensors when given).
    """
    b, length, _ = packed_qgkv.shape
    qg = packed_qgkv[..., : 2 * q_heads * dim].reshape(b, length, q_heads, 2, dim)
    q_raw = qg[..., 0, :]
    k0 = 2 * q_heads * dim
    k_raw = packed_qgkv[..., k0 : k0 + kv_heads * dim].reshape(b, length, kv_heads, dim)
    v_raw = packed_qgkv[..., k0 + kv_heads * dim : k0 + 2 * kv_heads * dim].reshape(b, length, kv_heads, dim)
    q = _norm_rope_heads(q_raw, q_weight, cos, sin, rotary_dim).transpose(1, 2).contiguous()
    k = _norm_rope_heads(k_raw, k_weight, cos, sin, rotary_dim).transpose(1, 2).contiguous()
    v = v_raw.transpose(1, 2).contiguous()
    if cache_key is not None:
        start = int(cache_start)
        cache_key[:, :, start : start + length] = k
        cache_value[:, :, start : start + length] = v
        return q, cache_key, cache_value
    return q, k, v


# --------------------------------------------------------------------------- DeltaNet
def causal_conv1d(x: torch.Tensor, weight: torch.Tensor, state: torch.Tensor) -> torch.Tensor:
    """Depthwise causal conv (zero left padding) + SiLU, with the conv-state update in place.

    kernels.py:576-710 (prefill :576-619, decode update :622-656); validate_kernels.py:71-86.
    ``x`` is ``[B, L, C']`` with ``C' >= C`` (packed projection rows); channels ``[0, C)`` are
    convolved. The conv result is rounded to BF16 before the SiLU (kernels.py:606-609).
    Decode (L == 1) shifts the state left by one and appends ``x``; prefill writes the last
    ``min(L, K)`` inputs into the tail of the state (kernels.py:611-619).
    """
    b, length, _ = x.shape
    channels, ksize = weight.shape
    xs = x[..., :channels].float()  # [B, L, C]
    w = weight.float()
    if length == 1:
        hist = torch.cat((state.float(), xs.transpose(1, 2)), dim=-1)  # [B, C, K+1]
        acc = torch.zeros(b, channels)
        for tap in range(ksize):
            acc = acc + hist[:, :, 1 + tap] * w[:, tap]
        state.copy_(hist[:, :, 1:].to(state.dtype))
        out = _bf(_silu32(_bf(acc).float()))
        return out[:, None, :]
    acc = torch.zeros(b, length, channels)
    for tap in range(ksize):
        shift = ksize - 1 - tap
        if shift >= length:
            continue
        src = torch.zeros_like(xs)
        src[:, shift:] = xs[:, : length - shift]
        acc = acc + src * w[:, tap]
    n_keep = min(length, ksize)
    state[:, :, ksize - n_keep :] = x[:, length - n_keep :, :channels].transpose(1, 2).to(state.dtype)
    return _bf(_silu32(_bf(acc).float()))


def delta_factors(q32, k32, a, b, a_log, dt_bias, dim):
    """Per (token, head) DeltaNet scalars: ``q_hat``, ``k_hat``, ``alpha``, ``beta``.

    kernels.py:713-765 and :826-841: L2 normalisation ``x * rsqrt(sum x^2 + 1e-6)`` in FP32,
    q additionally times ``1/sqrt(D)``; ``alpha = exp(-exp(A_log) * softplus(a + dt_bias))``;
    ``beta = sigmoid(b)`` (HF Qwen3_5GatedDeltaNet.forward uses F.softplus, threshold 20).
    """
    q_hat = q32 * torch.rsqrt((q32 * q32).sum(-1, keepdim=True) + 1e-6) * (1.0 / math.sqrt(dim))
    k_hat = k32 * torch.rsqrt((k32 * k32).sum(-1, keepdim=True) + 1e-6)
    g = -torch.exp(a_log.float()) * F.softplus(a.float() + dt_bias.float())
    alpha = torch.exp(g)
    beta = _sigmoid32(b.float())
    return q_hat, k_hat, alpha, beta, g


def delta_recurrent(qkv, packed, a_log, dt_bias, state):
    """Sequential gated delta rule over L tokens; ``state [B,H,Dk,Dv]`` FP32 updated in place.

    kernels.py:768-937 (per token: ``S *= alpha; m = S^T k; d = beta (v - m);
    S += k d^T; o = S^T q``); validate_kernels.py:89-115. Output ``[B, L, H, D]`` BF16.
    ``packed`` holds ``[qkv | z | a | b]`` per token (integration.py:81-93).
    """
    b, length, width = qkv.shape
    heads = a_log.numel()
    dim = width // (3 * heads)
    q, k, v = qkv.float().reshape(b, length, 3, heads, dim).unbind(2)
    a_off = width + heads * dim
    a = packed[..., a_off : a_off + heads]
    bb = packed[..., a_off + heads : a_off + 2 * heads]
    q_hat, k_hat, alpha, beta, _ = delta_factors(q, k, a, bb, a_log, dt_bias, dim)
    outs = []
    for t in range(length):
        state.mul_(alpha[:, t, :, None, None])
        mem = (state * k_hat[:, t, :, :, None]).sum(-2)
        delta = (v[:, t] - mem) * beta[:, t, :, None]
        state.add_(k_hat[:, t, :, :, None] * delta[:, :, None, :])
        outs.append((state * q_hat[:, t, :, :, None]).sum(-2))
    return _bf(torch.stack(outs, dim=1))


def chunk_gated_delta_rule(q_hat, k_hat, v, g, beta, state, chunk_size: int = 64):
    """Chunked (WY / UT-transform) form of the gated delta rule, FP32.

    Same algorithm as HF torch_chunk_gated_delta_rule (modeling_qwen3_5.py, chunk 64), written
    for already-normalised ``q_hat`` (scale folded in) and ``k_hat``. Inputs ``[B, L, H, D]``,
    ``g``/``beta`` ``[B, L, H]``; ``state [B, H, Dk, Dv]`` is updated in place. Returns FP32
    ``[B, L, H, Dv]``. Per chunk with cumulative log-decay ``c``:
    ``A = -(diag(beta) K K^T * exp(c_i - c_j))_{i>j}``, ``T = (I - A)^{-1}`` by forward
    substitution, ``U = T (beta V)``, ``W = T (beta K exp(c))``; then
    ``Vn = U - W S``, ``O = (Q exp(c)) S + (Q K^T * exp(c_i - c_j))_{i>=j} Vn``,
    ``S <- exp(c_last) S + (K exp(c_last - c))^T Vn``.
    """
    b, length, heads, dk = k_hat.shape
    dv = v.shape[-1]
    pad = (-length) % chunk_size
    def prep(x):
        x = x.float().transpose(1, 2)  # [B,H,L,*]
        if pad:
            x = F.pad(x, (0, 0, 0, pad)) if x.ndim == 4 else F.pad(x, (0, pad))
        return x
    qh, kh, vv = prep(q_hat), prep(k_hat), prep(v)
    gg, bt = prep(g), prep(beta)
    n_chunks = (length + pad) // chunk_size
    qh = qh.reshape(b, heads, n_chunks, chunk_size, dk)
    kh = kh.reshape(b, heads, n_chunks, chunk_size, dk)
    vv = vv.reshape(b, heads, n_chunks, chunk_size, dv)
    gg = gg.reshape(b, heads, n_chunks, chunk_size).cumsum(-1)
    bt = bt.reshape(b, heads, n_chunks, chunk_size)
    strict_lower = torch.tril(torch.ones(chunk_size, chunk_size, dtype=torch.bool), -1)
    lower = torch.tril(torch.ones(chunk_size, chunk_size, dtype=torch.bool), 0)
    out = torch.zeros(b, heads, n_chunks, chunk_size, dv)
    s = state
    for c in range(n_chunks):
        q_c, k_c, v_c, g_c, b_c = qh[:, :, c], kh[:, :, c], vv[:, :, c], gg[:, :, c], bt[:, :, c]
        decay = torch.exp((g_c[..., :, None] - g_c[..., None, :]).masked_fill(~lower, 0.0))
        decay = decay.masked_fill(~lower, 0.0)
        kb = k_c * b_c[..., None]
        a_mat = -(kb @ k_c.transpose(-1, -2)) * decay
        a_mat = a_mat.masked_fill(~strict_lower, 0.0)
        t_mat = a_mat.clone()
        for i in range(1, chunk_size):
            row = t_mat[..., i, :i].clone()
            sub = t_mat[..., :i, :i].clone()
            t_mat[..., i, :i] = row + (row[..., :, None] * sub).sum(-2)
        t_mat = t_mat + torch.eye(chunk_size)
        u = t_mat @ (v_c * b_c[..., None])
        w = t_mat @ (kb * torch.exp(g_c)[..., None])
        v_new = u - w @ s
        attn = (q_c @ k_c.transpose(-1, -2)) * decay
        out[:, :, c] = (q_c * torch.exp(g_c)[..., None]) @ s + attn @ v_new
        g_last = g_c[..., -1]
        s = s * torch.exp(g_last)[..., None, None] + (
            k_c * torch.exp(g_last[..., None] - g_c)[..., None]
        ).transpose(-1, -2) @ v_new
    state.copy_(s)
    out = out.reshape(b, heads, n_chunks * chunk_size, dv)[:, :, :length]
    return out.transpose(1, 2).contiguous()


# --------------------------------------------------------------------------- attention
def gqa_decode_attention(q, cache_keys, cache_values, valid_length: int, scale: float):
    """Maskless decode attention over the valid cache prefix, FP32 online-softmax semantics.

    kernels.py:940-1090 (q scaled first, :968); validate_kernels.py:227-245 compares it to
    ``F.scaled_dot_product_attention(enable_gqa=True)``. ``q [B,H,1,D]``,
    caches ``[B,Hkv,Lmax,D]`` → ``[B,1,H*D]`` BF16.
    """
    b, heads, _, dim = q.shape
    kvh = cache_keys.shape[1]
    group = heads // kvh
    n = int(valid_length)
    k = cache_keys[:, :, :n].float().repeat_interleave(group, dim=1)
    v = cache_values[:, :, :n].float().repeat_interleave(group, dim=1)
    scores = (q.float() * scale) @ k.transpose(-1, -2)  # [B,H,1,n]
    p = torch.softmax(scores, dim=-1)
    out = p @ v  # [B,H,1,D]
    return _bf(out.reshape(b, 1, heads * dim))


def causal_attention(q, k, v, scale: float, q_offset: int = 0):
    """Causal GQA attention in FP32 (softmax over keys ``j <= i + q_offset``), BF16 out.

    Stands in for the SDPA call of the reference prefill (integration.py:360-372).
    ``q [B,H,L,D]``, ``k/v [B,Hkv,S,D]`` → ``[B, L, H*D]``.
    """
    b, heads, length, dim = q.shape
    group = heads // k.shape[1]
    kk = k.float().repeat_interleave(group, dim=1)
    vv = v.float().repeat_interleave(group, dim=1)
    scores = (q.float() * scale) @ kk.transpose(-1, -2)
    s_len = kk.shape[2]
    i = torch.arange(length)[:, None] + q_offset
    j = torch.arange(s_len)[None, :]
    scores = scores.masked_fill(j > i, float("-inf"))
    p = torch.softmax(scores, dim=-1)
    out = (p @ vv).transpose(1, 2).reshape(b, length, heads * dim)
    return _bf(out)


# --------------------------------------------------------------------------- LM head
def lm_head_argmax(hidden: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Greedy top-1 over BF16-rounded logits, lowest index on ties. kernels.py:1093-1185.

    ``hidden [B, K]`` → int64 ``[B, 1]``.
    """
    logits = linear(hidden, weight).float()
    best = logits.max(dim=-1, keepdim=True).values
    idx = torch.arange(logits.shape[-1]).expand_as(logits)
    cand = torch.where(logits == best, idx, torch.full_like(idx, logits.shape[-1]))
    return cand.min(dim=-1, keepdim=True).values.to(torch.int64)


# --------------------------------------------------------------------------- vocab-sharded LM head
INT64_MIN = -(1 << 63)


def float_order_key(v: float) -> int:
    """32-bit unsigned key that orders FP32 values like the values themselves (-0 folded to +0):
    the sign bit set for non-negative values, all bits inverted for negative ones."""
    import struct

    v = float(v)
    if v == 0.0:
        v = 0.0
    u = struct.unpack("<I", struct.pack("<f", v))[0]
    return (~u) & 0xFFFFFFFF if u & 0x80000000 else u | 0x80000000


def lm_shard_keys(hidden: torch.Tensor, weight_shard: torch.Tensor, row_offset: int) -> torch.Tensor:
    """Shard keys of the multi-GPU split of kernels.py:1093-1185 (the top-1 over BF16-rounded
    logits of ``hidden [n, K]`` against rows ``[row_offset, row_offset + rows)``, lowest index on
    ties), as int64 ``[n]``: ``((order(logit) << 32) | (0xFFFFFFFF - index)) - 2^63``, INT64_MIN for
    an empty shard. The maximum over shards is the key of the full-vocabulary top-1."""
    n = hidden.shape[0]
    if weight_shard.shape[0] == 0:
        return torch.full((n,), INT64_MIN, dtype=torch.int64)
    local = lm_head_argmax(hidden, weight_shard).reshape(-1)
    logits = linear(hidden, weight_shard).float()
    keys = []
    for b in range(n):
        i = int(local[b])
        v = float(logits[b, i])
        ukey = (float_order_key(v) << 32) | (0xFFFFFFFF - (row_offset + i))
        keys.append(ukey - (1 << 63))
    return torch.tensor(keys, dtype=torch.int64)


def lm_keys_to_tokens(keys: torch.Tensor) -> torch.Tensor:
    """Token ids encoded by reduced shard keys (INT64_MIN, an empty reduction, maps to 0)."""
    out = []
    for k in keys.reshape(-1).tolist():
        u = k + (1 << 63)
        out.append(0 if u == 0 else 0xFFFFFFFF - (u & 0xFFFFFFFF))
    return torch.tensor(out, dtype=torch.int64)
