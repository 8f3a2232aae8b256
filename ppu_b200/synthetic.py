"""Seeded random-init weights and inputs for the Qwen3.5 decoder (no checkpoint needed).

Weights use the Hugging Face parameter names of ``Qwen3_5ForCausalLM`` so the same dict can
be loaded into the eager model, the CPU oracle and this package's engine. Every tensor is
drawn from ``N(0, std)`` (std 0.02) in a fixed name order from one ``torch.Generator``,
except the gated RMSNorm weight, which multiplies directly (not ``1 + w``) and is drawn as
``1 + N(0, std)`` so the DeltaNet branch keeps unit scale.
"""

from __future__ import annotations

import torch

from .config import Qwen35Dims


def weight_shapes(dims: Qwen35Dims) -> list[tuple[str, tuple[int, ...]]]:
    h = dims.hidden
    out: list[tuple[str, tuple[int, ...]]] = [("model.embed_tokens.weight", (dims.vocab, h))]
    for i, kind in enumerate(dims.layer_types):
        p = f"model.layers.{i}."
        if kind == "linear_attention":
            la = p + "linear_attn."
            out += [
                (la + "dt_bias", (dims.lin_heads,)),
                (la + "A_log", (dims.lin_heads,)),
                (la + "conv1d.weight", (dims.conv_dim, 1, dims.conv_kernel)),
                (la + "norm.weight", (dims.lin_dv,)),
                (la + "out_proj.weight", (h, dims.value_dim)),
                (la + "in_proj_qkv.weight", (dims.conv_dim, h)),
                (la + "in_proj_z.weight", (dims.value_dim, h)),
                (la + "in_proj_b.weight", (dims.lin_heads, h)),
                (la + "in_proj_a.weight", (dims.lin_heads, h)),
            ]
        else:
            sa = p + "self_attn."
            out += [
                (sa + "q_proj.weight", (2 * dims.q_heads * dims.head_dim, h)),
                (sa + "k_proj.weight", (dims.kv_heads * dims.head_dim, h)),
                (sa + "v_proj.weight", (dims.kv_heads * dims.head_dim, h)),
                (sa + "o_proj.weight", (h, dims.attn_width)),
                (sa + "q_norm.weight", (dims.head_dim,)),
                (sa + "k_norm.weight", (dims.head_dim,)),
            ]
        out += [
            (p + "mlp.gate_proj.weight", (dims.intermediate, h)),
            (p + "mlp.up_proj.weight", (dims.intermediate, h)),
            (p + "mlp.down_proj.weight", (h, dims.intermediate)),
            (p + "input_layernorm.weight", (h,)),
            (p + "post_attention_layernorm.weight", (h,)),
        ]
    out.append(("model.norm.weight", (h,)))
    return out


def make_weights(dims: Qwen35Dims, seed: int = 0, device="cpu", std: float = 0.02,
                 dtype=torch.bfloat16) -> dict[str, torch.Tensor]:
    """Random-init weights ``{hf_name: tensor}``; identical values for a given seed/device type."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    weights: dict[str, torch.Tensor] = {}
    for name, shape in weight_shapes(dims):
        t = torch.empty(shape, device=device, dtype=torch.float32)
        t.normal_(0.0, std, generator=gen)
        if name.endswith("linear_attn.norm.weight"):
            t += 1.0
        weights[name] = t.to(dtype)
    return weights


def make_prompt(dims: Qwen35Dims, length: int, seed: int = 1, batch: int = 1) -> torch.Tensor:
    """Uniform-random token ids ``[batch, length]`` int64 on the CPU."""
    gen = torch.Generator()
    gen.manual_seed(seed)
    return torch.randint(0, dims.vocab, (batch, length), generator=gen, dtype=torch.int64)


def vision_weight_shapes(vd) -> list[tuple[str, tuple[int, ...]]]:
    """Hugging Face names and shapes of the vision tower (``model.visual.*`` of
    ``Qwen3_5ForConditionalGeneration``) for a ``VisionDims``-like shape ``vd``."""
    w, i = vd.width, vd.intermediate
    mw = w * vd.merge * vd.merge
    p = "model.visual."
    out = [(p + "patch_embed.proj.weight", (w, vd.in_channels, vd.temporal_patch, vd.patch, vd.patch)),
           (p + "patch_embed.proj.bias", (w,)),
           (p + "pos_embed.weight", (vd.pos_side * vd.pos_side, w))]
    for b in range(vd.depth):
        q = f"{p}blocks.{b}."
        out += [(q + "norm1.weight", (w,)), (q + "norm1.bias", (w,)), (q + "norm2.weight", (w,)),
                (q + "norm2.bias", (w,)), (q + "attn.qkv.weight", (3 * w, w)), (q + "attn.qkv.bias", (3 * w,)),
                (q + "attn.proj.weight", (w, w)), (q + "attn.proj.bias", (w,)),
                (q + "mlp.linear_fc1.weight", (i, w)), (q + "mlp.linear_fc1.bias", (i,)),
                (q + "mlp.linear_fc2.weight", (w, i)), (q + "mlp.linear_fc2.bias", (w,))]
    out += [(p + "merger.norm.weight", (w,)), (p + "merger.norm.bias", (w,)),
            (p + "merger.linear_fc1.weight", (mw, mw)), (p + "merger.linear_fc1.bias", (mw,)),
            (p + "merger.linear_fc2.weight", (vd.out_width, mw)), (p + "merger.linear_fc2.bias", (vd.out_width,))]
    return out


def make_vision_weights(vd, seed: int = 0, device="cpu", std: float = 0.02,
                        dtype=torch.bfloat16) -> dict[str, torch.Tensor]:
    """Random-init vision weights ``{hf_name: tensor}``: ``N(0, std)`` in a fixed name order from one
    generator, LayerNorm weights ``1 + N(0, std)`` (unit scale, as a LayerNorm starts)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    weights: dict[str, torch.Tensor] = {}
    for name, shape in vision_weight_shapes(vd):
        t = torch.empty(shape, device=device, dtype=torch.float32)
        t.normal_(0.0, std, generator=gen)
        if "norm" in name and name.endswith(".weight"):
            t += 1.0
        weights[name] = t.to(dtype)
    return weights


def make_image(height: int, width: int, seed: int = 0, channels: int = 3) -> torch.Tensor:
    """Uniform [0, 1) pixels ``[channels, height, width]`` fp32 on the CPU (already rescaled)."""
    gen = torch.Generator()
    gen.manual_seed(seed)
    return torch.rand((channels, height, width), generator=gen, dtype=torch.float32)
