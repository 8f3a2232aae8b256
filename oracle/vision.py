"""CPU restatement of the reference's fused Qwen3.5 vision tower (ViT encoder + 2x2 merger).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows qwen35_fused/kernels.py for the fused operators and qwen35_fused/integration.py:509-575
(``run_blocks``) plus the merger for the forward; the pieces the reference takes from
Transformers (processor patch layout, rotary tables, bilinear position interpolation, eager
attention) follow Transformers' Qwen3_5VisionModel / Qwen2VLImageProcessor. Pinned against
vectors generated from the reference's own torch expressions and from Transformers' eager
vision model (``tests/golden/make_golden_vision.py``).
"""

from __future__ import annotations

import torch

from ppu_b200.config import VisionDims  # noqa: F401  (shape dataclass shared with the package)

BF16 = torch.bfloat16


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """kernels.py:1188-1222: FP32 mean, centred variance, ``c * rsqrt(var + eps) * w + b``."""
    x32 = x.float()
    mean = x32.mean(-1, keepdim=True)
    c = x32 - mean
    var = (c * c).mean(-1, keepdim=True)
    return (c * torch.rsqrt(var + eps) * w.float() + b.float()).to(x.dtype)


def residual_add_layer_norm(r: torch.Tensor, u: torch.Tensor, w, b, eps: float = 1e-6):
    """kernels.py:1225-1287: the sum is rounded to bf16 before the norm."""
    added = (r.float() + u.float()).to(r.dtype)
    return added, layer_norm(added, w, b, eps)


def position_embed_add(hidden: torch.Tensor, table: torch.Tensor, idx: torch.Tensor, wts: torch.Tensor):
    """kernels.py:1290-1336: ``bf16(hidden + bf16(sum_k w_k table[idx_k]))``, FP32 accumulation
    (roundings to ``hidden.dtype``: none in the FP32 reference mode)."""
    pos = (table[idx].float() * wts.float()[..., None]).sum(-2)
    return (hidden.float() + pos.to(hidden.dtype).float()).to(hidden.dtype)


def linspace(end: float, steps: int) -> torch.Tensor:
    return torch.linspace(0, end, steps, dtype=torch.float32)


def token_grid(gh: int, gw: int, merge: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Grid (row, col) of each patch token in the merge-block order of the processor."""
    rows = torch.arange(gh).view(gh // merge, merge, 1, 1).expand(gh // merge, merge, gw // merge, merge)
    cols = torch.arange(gw).view(1, 1, gw // merge, merge).expand(gh // merge, merge, gw // merge, merge)
    rows = rows.permute(0, 2, 1, 3).reshape(-1)
    cols = cols.permute(0, 2, 1, 3).reshape(-1)
    return rows, cols


def interp_indices_weights(gh: int, gw: int, side: int, merge: int):
    """Bilinear neighbours of each token into the side x side learned table (Transformers
    fast_pos_embed_interpolate: linspace grid, floor / clipped ceil), FP32 weights, merge order."""
    hs, ws = linspace(side - 1, gh), linspace(side - 1, gw)
    hf, wf = hs.int(), ws.int()
    hc, wc = (hf + 1).clamp(max=side - 1), (wf + 1).clamp(max=side - 1)
    dh, dw = hs - hf, ws - wf
    rows, cols = token_grid(gh, gw, merge)
    h0, h1, w0, w1 = hf[rows], hc[rows], wf[cols], wc[cols]
    a, b_ = dh[rows], dw[cols]
    idx = torch.stack([h0 * side + w0, h0 * side + w1, h1 * side + w0, h1 * side + w1], -1).long()
    wts = torch.stack([(1 - a) * (1 - b_), (1 - a) * b_, a * (1 - b_), a * b_], -1)
    return idx, wts


def rope_inv_freq(head_dim: int, theta: float = 10000.0) -> torch.Tensor:
    """Qwen3_5VisionRotaryEmbedding(head_dim // 2).inv_freq."""
    dim = head_dim // 2
    return 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float) / dim))


def rope_cos_sin(gh: int, gw: int, merge: int, inv_freq: torch.Tensor):
    """Transformers rot_pos_emb: [row freqs | col freqs], then cat(emb, emb); FP32 cos / sin."""
    rows, cols = token_grid(gh, gw, merge)
    fr = rows.float()[:, None] * inv_freq[None]
    fc = cols.float()[:, None] * inv_freq[None]
    emb = torch.cat((fr, fc), -1)
    emb = torch.cat((emb, emb), -1)
    return emb.cos(), emb.sin()


def vision_qkv_rope(packed: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, heads: int, dim: int):
    """kernels.py:336-416: packed [L, 3*heads*dim] -> BHLD q, k, v; q/k rotated in FP32."""
    L = packed.shape[0]
    q, k, v = packed.view(L, 3, heads, dim).permute(1, 0, 2, 3).unbind(0)

    def rope(x):
        x32 = x.float()
        rot = torch.cat((-x32[..., dim // 2:], x32[..., :dim // 2]), -1)
        return (x32 * cos[:, None, :] + rot * sin[:, None, :]).to(packed.dtype)

    return (rope(q).transpose(0, 1).unsqueeze(0), rope(k).transpose(0, 1).unsqueeze(0),
            v.transpose(0, 1).unsqueeze(0).contiguous())


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """Eager bidirectional attention (Transformers eager_attention_forward): FP32 softmax, weights
    cast to bf16, P @ V; [1, H, L, D] -> [L, H*D]."""
    s = (q.float() @ k.float().transpose(-1, -2)) * scale
    p = torch.softmax(s, dim=-1).to(q.dtype)
    o = (p.float() @ v.float()).to(q.dtype)
    return o[0].transpose(0, 1).reshape(q.shape[2], -1)


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """nn.Linear with bias: FP32 product + bias, one rounding to ``x.dtype``."""
    return (x.float() @ w.float().T + b.float()).to(x.dtype)


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return torch.nn.functional.gelu(x.float(), approximate="tanh").to(x.dtype)


def gelu(x: torch.Tensor) -> torch.Tensor:
    return torch.nn.functional.gelu(x.float()).to(x.dtype)


def patchify(pixels: torch.Tensor, dims: VisionDims, dtype=BF16) -> torch.Tensor:
    """Qwen2-VL image processor layout for one image: fp32 [C, H, W] in [0,1) -> normalised bf16
    [(H/P)*(W/P), C*T*P*P], the frame repeated over the temporal patch."""
    C, H, W = pixels.shape
    P, T, M = dims.patch, dims.temporal_patch, dims.merge
    x = (pixels.float() - dims.pixel_mean) / dims.pixel_std
    x = x[None].expand(T, C, H, W)
    gh, gw = H // P, W // P
    x = x.reshape(1, T, C, gh // M, M, P, gw // M, M, P)
    x = x.permute(0, 3, 6, 4, 7, 2, 1, 5, 8)
    return x.reshape(gh * gw, C * T * P * P).to(dtype)


class VisionOracle:
    """The reference's vision forward (integration.py:509-575 + merger) on the CPU. With
    ``dtype=torch.float32`` every bf16 rounding point is skipped (the weights keep their bf16
    values): the exact forward that measures how far the bf16 forward itself drifts over depth."""

    def __init__(self, weights: dict, dims: VisionDims, prefix: str = "model.visual.", dtype=BF16):
        self.d = dims
        self.dtype = dtype
        self.w = {k[len(prefix):]: v.to(dtype) for k, v in weights.items() if k.startswith(prefix)}
        self.inv_freq = rope_inv_freq(dims.head_dim, dims.rope_theta)

    def forward(self, pixels: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Returns (final patch states [N, width], merged visual tokens [N / merge^2, out_width])."""
        d, w = self.d, self.w
        _, H, W = pixels.shape
        gh, gw = H // d.patch, W // d.patch
        patches = patchify(pixels, d, self.dtype)
        pw = w["patch_embed.proj.weight"].reshape(d.width, -1)
        hidden = linear(patches, pw, w["patch_embed.proj.bias"])
        idx, wts = interp_indices_weights(gh, gw, d.pos_side, d.merge)
        residual = position_embed_add(hidden, w["pos_embed.weight"], idx, wts)
        cos, sin = rope_cos_sin(gh, gw, d.merge, self.inv_freq)
        normed = layer_norm(residual, w["blocks.0.norm1.weight"], w["blocks.0.norm1.bias"], d.eps)
        scale = d.head_dim ** -0.5
        for i in range(d.depth):
            p = f"blocks.{i}."
            packed = linear(normed, w[p + "attn.qkv.weight"], w[p + "attn.qkv.bias"])
            q, k, v = vision_qkv_rope(packed, cos, sin, d.heads, d.head_dim)
            att = attention(q, k, v, scale)
            upd = linear(att, w[p + "attn.proj.weight"], w[p + "attn.proj.bias"])
            residual, mlp_in = residual_add_layer_norm(residual, upd, w[p + "norm2.weight"], w[p + "norm2.bias"],
                                                       d.eps)
            h1 = gelu_tanh(linear(mlp_in, w[p + "mlp.linear_fc1.weight"], w[p + "mlp.linear_fc1.bias"]))
            upd = linear(h1, w[p + "mlp.linear_fc2.weight"], w[p + "mlp.linear_fc2.bias"])
            if i + 1 < d.depth:
                n = f"blocks.{i + 1}.norm1."
                residual, normed = residual_add_layer_norm(residual, upd, w[n + "weight"], w[n + "bias"], d.eps)
            else:
                residual = (residual.float() + upd.float()).to(self.dtype)
        m = layer_norm(residual, w["merger.norm.weight"], w["merger.norm.bias"], d.eps)
        m = m.reshape(-1, d.width * d.merge * d.merge)
        m = gelu(linear(m, w["merger.linear_fc1.weight"], w["merger.linear_fc1.bias"]))
        merged = linear(m, w["merger.linear_fc2.weight"], w["merger.linear_fc2.bias"])
        return residual, merged
