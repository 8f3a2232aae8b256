"""Install the B200 fused inference path on a loaded Transformers Qwen3.5 model.

Drop-in for qwen35_fused/integration.py (``apply_fusions``, ``FusionConfig``), targeting the
installed Transformers (5.5) cache API. Same structure as the reference:

* ``_pack_linear_weights`` (integration.py:69-140): [qkv|z|a|b] (padded), [gate;up], [Q|G..|K|V]
  registered as buffers; originals optionally released; A8W8 (``FusionConfig.a8w8``) also keeps
  int8 copies with per-row scales for the M/F/L groups;
* patched forwards of the RMSNorm / gated RMSNorm modules, MLP, Gated DeltaNet, attention and the
  text-model loop (integration.py:143-506). Inputs that are not BF16 CUDA tensors, and padded
  batches, raise ``ValueError`` unless ``FusionConfig(eager_fallback=True)`` asks for the
  reference's behaviour (the original Transformers forward for them);
* every operator is a hand-written sm_100a kernel from ``ppu_b200.kernels`` (no F.linear / SDPA on
  the fast path).

Cache handling on Transformers 5.5: attention layers use ``StaticLayer`` (keys/values with a device
``cumulative_length``) or ``DynamicLayer``; DeltaNet layers use ``LinearAttentionLayer`` for the
BF16 conv state, while the FP32 recurrent state the reference keeps (kernels.py:804) is held on
the cache layer as ``_q35_recurrent`` (Transformers 5.5 would store it in BF16).
"""

from __future__ import annotations

import types

import torch
from transformers.cache_utils import DynamicCache
from transformers.models.qwen3_5 import modeling_qwen3_5 as qwen_impl

from . import kernels as K
from . import lib as L
from .config import FusionConfig

BF16 = torch.bfloat16


def _is_fast_tensor(x: torch.Tensor) -> bool:
    return x.is_cuda and x.dtype == BF16


def _register_buffer(module: torch.nn.Module, name: str, value: torch.Tensor | None) -> None:
    if hasattr(module, name):
        setattr(module, name, value)
    else:
        module.register_buffer(name, value, persistent=False)


def _release_linear_weight(module: torch.nn.Module) -> int:
    weight = module.weight
    released = weight.numel() * weight.element_size()
    module.register_parameter("weight", None)
    return released


def _text_model(model: torch.nn.Module) -> torch.nn.Module:
    inner = model.model
    return inner.language_model if hasattr(inner, "language_model") else inner


def _quantize_into(module, name: str, weight: torch.Tensor) -> None:
    q, s = K.quantize_rows(weight)
    _register_buffer(module, name + "_q8", q)
    _register_buffer(module, name + "_scale", s.reshape(-1).contiguous())


def _pack_linear_weights(model: torch.nn.Module, config: FusionConfig) -> dict:
    """integration.py:69-140."""
    text = _text_model(model)
    stats = {"delta": 0, "mlp": 0, "attention": 0, "vision": 0, "released_weight_bytes": 0, "a8w8": 0}
    q8 = config.a8w8
    for layer in text.layers:
        if hasattr(layer, "linear_attn") and config.delta:
            d = layer.linear_attn
            packed = torch.cat((d.in_proj_qkv.weight, d.in_proj_z.weight, d.in_proj_a.weight,
                                d.in_proj_b.weight), 0).contiguous().detach()
            pad_to = config.delta_projection_padding
            if pad_to:
                pad = (-packed.shape[0]) % pad_to
                if pad:
                    packed = torch.cat((packed, packed.new_zeros(pad, packed.shape[1])), 0)
            _register_buffer(d, "_fused_in_proj_weight", packed)
            _register_buffer(d, "_fused_conv_weight", d.conv1d.weight.detach().squeeze(1).contiguous())
            if q8 and packed.is_cuda:
                _quantize_into(d, "_fused_in_proj", packed)
                _quantize_into(d, "_fused_out_proj", d.out_proj.weight.detach())
                stats["a8w8"] += 2
            if config.release_original_weights:
                stats["released_weight_bytes"] += sum(_release_linear_weight(p) for p in (
                    d.in_proj_qkv, d.in_proj_z, d.in_proj_a, d.in_proj_b))
            stats["delta"] += 1
        if config.swiglu:
            mlp = layer.mlp
            gate_up = torch.cat((mlp.gate_proj.weight, mlp.up_proj.weight), 0).contiguous().detach()
            _register_buffer(mlp, "_fused_gate_up_weight", gate_up)
            if q8 and gate_up.is_cuda:
                _quantize_into(mlp, "_fused_gate_up", gate_up)
                _quantize_into(mlp, "_fused_down", mlp.down_proj.weight.detach())
                stats["a8w8"] += 2
            if config.release_original_weights:
                stats["released_weight_bytes"] += _release_linear_weight(mlp.gate_proj)
                stats["released_weight_bytes"] += _release_linear_weight(mlp.up_proj)
            stats["mlp"] += 1
        if hasattr(layer, "self_attn") and config.attention:
            a = layer.self_attn
            qgkv = torch.cat((a.q_proj.weight, a.k_proj.weight, a.v_proj.weight), 0).contiguous().detach()
            _register_buffer(a, "_fused_qgkv_weight", qgkv)
            biases = (a.q_proj.bias, a.k_proj.bias, a.v_proj.bias)
            if any(b is not None for b in biases):
                raise ValueError("attention projection biases are not supported by the fused path")
            if q8 and qgkv.is_cuda:
                _quantize_into(a, "_fused_qgkv", qgkv)
                _quantize_into(a, "_fused_o_proj", a.o_proj.weight.detach())
                stats["a8w8"] += 2
            if config.release_original_weights:
                for p in (a.q_proj, a.k_proj, a.v_proj):
                    stats["released_weight_bytes"] += _release_linear_weight(p)
            stats["attention"] += 1
    return stats


def _proj(x: torch.Tensor, weight: torch.Tensor, q8: torch.Tensor | None = None,
          scale: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ W^T`` with the CUDA GEMV (one row) or GEMM (prefill); A8W8 when int8 weights exist."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    if q8 is not None:
        out = K.a8w8_linear(x2, q8, scale)
    elif x2.shape[0] == 1:
        out = K.fused_gemv(weight, x2.reshape(-1)).reshape(1, -1)
    else:
        out = K.gemm(x2, weight)
    return out.reshape(*lead, out.shape[-1])


def _install(module: torch.nn.Module, fast, config: FusionConfig, primary: str, accept=None) -> bool:
    """Routes ``module.forward`` through ``fast(self, *args, **kwargs)``. The tensor named
    ``primary`` (or the first positional argument) must be a BF16 CUDA tensor; otherwise the call
    raises ``ValueError``, or, with ``config.eager_fallback``, runs the module's original
    Transformers forward as the reference does (integration.py:51-52). Returns False when the
    module was patched already."""
    if hasattr(module, "_fused_original_forward"):
        return False
    module._fused_original_forward = module.forward

    def forward(self, *args, **kwargs):
        x = args[0] if args else kwargs.get(primary)
        if x is None and primary == "input_ids":
            x = kwargs.get("inputs_embeds")
        if accept is not None and isinstance(x, torch.Tensor) and accept(x):
            return fast(self, *args, **kwargs)
        if accept is None and isinstance(x, torch.Tensor) and (x.dtype == torch.long or _is_fast_tensor(x)):
            if x.dtype != torch.long or x.is_cuda:
                return fast(self, *args, **kwargs)
        if config.eager_fallback:
            return self._fused_original_forward(*args, **kwargs)
        what = "None" if x is None else f"{tuple(x.shape)} {x.dtype} on {x.device}"
        raise ValueError(f"{type(self).__name__}: the fused path takes BF16 CUDA tensors, got {what} "
                         "(FusionConfig(eager_fallback=True) runs the Transformers forward instead)")

    module.forward = types.MethodType(forward, module)
    return True


def _fused_rms_norm(self, x):
    return K.rms_norm(x.contiguous(), self.weight, self.eps)


def _fused_gated_norm(self, hidden_states, gate=None):
    if gate is None:  # the reference's gated module is always called with its gate
        raise ValueError("gated RMSNorm: the fused path needs the gate tensor")
    return K.gated_rms_norm(hidden_states.contiguous(), gate.contiguous(), self.weight, self.variance_epsilon)


def _patch_mlp(module: torch.nn.Module, config: FusionConfig) -> None:
    """integration.py:169-188: decode SwiGLU GEMV, prefill GEMM with the SwiGLU epilogue."""
    def forward(self, x):
        q8 = getattr(self, "_fused_gate_up_q8", None)
        if q8 is not None:
            act = K.silu_and_mul(_proj(x, None, q8, self._fused_gate_up_scale))
            return _proj(act, None, self._fused_down_q8, self._fused_down_scale)
        if config.ppu_swiglu_gemv and x.shape[:-1].numel() == 1:
            act = K.ppu_swiglu_gemv(x.reshape(1, 1, -1).contiguous(), self._fused_gate_up_weight)
            act = act.reshape(*x.shape[:-1], -1)
        else:
            act = K.gemm(x.contiguous(), self._fused_gate_up_weight, epilogue=L.EPI_SWIGLU)
        return _proj(act, self.down_proj.weight)

    _install(module, forward, config, "x")


def _delta_states(module, cache_params, batch: int, device):
    """Conv state (cache's BF16 tensor) and FP32 recurrent state for this layer; ``decode`` is
    True when the cache already holds this layer's state (integration.py:191-217)."""
    conv_shape = (batch, module.conv_dim, module.conv_kernel_size)
    rec_shape = (batch, module.num_v_heads, module.head_k_dim, module.head_v_dim)
    if cache_params is None:
        return (torch.zeros(conv_shape, device=device, dtype=BF16),
                torch.zeros(rec_shape, device=device, dtype=torch.float32), False, None)
    layer = cache_params.layers[module.layer_idx]
    decode = bool(layer.has_previous_state)
    rec = getattr(layer, "_q35_recurrent", None)
    if rec is None or tuple(rec.shape) != rec_shape:
        rec = torch.zeros(rec_shape, device=device, dtype=torch.float32)
        layer._q35_recurrent = rec
    if decode:
        return layer.conv_states, rec, True, layer
    rec.zero_()
    return torch.zeros(conv_shape, device=device, dtype=BF16), rec, False, layer


def _patch_delta(module: torch.nn.Module, config: FusionConfig) -> None:
    """integration.py:220-274."""
    def forward(self, hidden_states, cache_params=None, attention_mask=None, **kwargs):
        hidden_states = qwen_impl.apply_mask_to_padding_states(hidden_states, attention_mask)
        batch, seq_len, _ = hidden_states.shape
        packed = _proj(hidden_states, self._fused_in_proj_weight, getattr(self, "_fused_in_proj_q8", None),
                       getattr(self, "_fused_in_proj_scale", None))
        conv_state, rec_state, decode, layer = _delta_states(self, cache_params, batch, hidden_states.device)
        if decode and seq_len != 1:
            raise RuntimeError("fused DeltaNet continues a cached state one token at a time")
        qkv = K.causal_conv1d_fused(packed, self._fused_conv_weight, conv_state)
        core = K.delta_recurrent_fused(qkv, packed, self.A_log, self.dt_bias, rec_state,
                                       block_v=config.delta_block_v, precompute_factors=config.delta_precompute_factors)
        if layer is not None and not decode:
            cache_params.update_conv_state(conv_state, self.layer_idx)  # copies; marks has_previous_state
        z = packed[..., self.conv_dim:self.conv_dim + self.value_dim].reshape(-1, self.head_v_dim).contiguous()
        core = K.gated_rms_norm(core.reshape(-1, self.head_v_dim), z, self.norm.weight, self.layer_norm_epsilon)
        core = core.reshape(batch, seq_len, self.value_dim)
        return _proj(core, self.out_proj.weight, getattr(self, "_fused_out_proj_q8", None),
                     getattr(self, "_fused_out_proj_scale", None))

    _install(module, forward, config, "hidden_states")


def _patch_attention(module: torch.nn.Module, config: FusionConfig) -> None:
    """integration.py:277-382."""
    def forward(self, hidden_states, position_embeddings, attention_mask, past_key_values=None, **kwargs):
        batch, seq_len, _ = hidden_states.shape
        packed = _proj(hidden_states, self._fused_qgkv_weight, getattr(self, "_fused_qgkv_q8", None),
                       getattr(self, "_fused_qgkv_scale", None))
        cos, sin = position_embeddings
        cfg = self.config
        nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
        cache_layer = None
        if past_key_values is not None:
            cand = past_key_values.layers[self.layer_idx]
            if hasattr(cand, "max_cache_len"):
                cache_layer = cand
                if not cache_layer.is_initialized:
                    shape = (batch, nkv, seq_len, self.head_dim)
                    init = torch.empty(shape, device=hidden_states.device, dtype=hidden_states.dtype)
                    cache_layer.lazy_initialization(init, torch.empty_like(init))
        o_q8 = getattr(self, "_fused_o_proj_q8", None)
        o_scale = getattr(self, "_fused_o_proj_scale", None)
        if cache_layer is not None:
            start = cache_layer.cumulative_length
            q_offset = None if (config.gqa_decode_attention and seq_len == 1) else int(start)
            q, keys, values = K.qgkv_norm_rope(packed, self.q_norm.weight, self.k_norm.weight, cos, sin,
                                               q_heads=nq, kv_heads=nkv, dim=self.head_dim,
                                               rotary_dim=cos.shape[-1], cache_key=cache_layer.keys,
                                               cache_value=cache_layer.values, cache_start=start)
            cache_layer.cumulative_length.add_(seq_len)
            if q_offset is None:
                attn = K.gqa_decode_attention(q, keys, values, cache_layer.cumulative_length, self.scaling)
            elif attention_mask is None:
                attn = K.prefill_attention(q, keys, values, self.scaling, q_offset=q_offset)
            else:
                attn = None
        else:
            q, keys, values = K.qgkv_norm_rope(packed, self.q_norm.weight, self.k_norm.weight, cos, sin,
                                               q_heads=nq, kv_heads=nkv, dim=self.head_dim,
                                               rotary_dim=cos.shape[-1])
            if past_key_values is not None:
                keys, values = past_key_values.update(keys, values, self.layer_idx)
            attn = None
            if attention_mask is None:
                attn = K.prefill_attention(q, keys.contiguous(), values.contiguous(), self.scaling,
                                           q_offset=keys.shape[2] - seq_len)
        if attn is None:  # padded batch: the model's 4D mask
            if not config.eager_fallback:
                raise ValueError("fused attention: padded batches (a 4D attention mask) need "
                                 "FusionConfig(eager_fallback=True), which runs Transformers' attention")
            iface = qwen_impl.ALL_ATTENTION_FUNCTIONS.get_interface(cfg._attn_implementation,
                                                                    qwen_impl.eager_attention_forward)
            attn, _ = iface(self, q, keys, values, attention_mask, dropout=0.0, scaling=self.scaling, **kwargs)
            attn = attn.reshape(batch, seq_len, -1).contiguous()
        attn = K.attention_gate_mul(attn.reshape(batch, seq_len, -1).contiguous(), packed, self.head_dim)
        return _proj(attn, self.o_proj.weight, o_q8, o_scale), None

    _install(module, forward, config, "hidden_states")


def _patch_text_model(text_model: torch.nn.Module, config: FusionConfig) -> None:
    """integration.py:385-506: residual + norm fused between sublayers."""
    def forward(self, input_ids=None, attention_mask=None, position_ids=None, past_key_values=None,
                inputs_embeds=None, use_cache=None, **kwargs):
        if (input_ids is None) == (inputs_embeds is None):
            raise ValueError("specify exactly one of input_ids and inputs_embeds")
        if inputs_embeds is None:
            inputs_embeds = self.embed_tokens(input_ids)
        if not _is_fast_tensor(inputs_embeds):
            if not config.eager_fallback:
                raise ValueError("fused text model: the embeddings must be BF16 CUDA tensors")
            return self._fused_original_forward(input_ids=None, attention_mask=attention_mask,
                                                position_ids=position_ids, past_key_values=past_key_values,
                                                inputs_embeds=inputs_embeds, use_cache=use_cache, **kwargs)
        if use_cache and past_key_values is None:
            past_key_values = DynamicCache(config=self.config)
        if position_ids is None:
            seen = past_key_values.get_seq_length() if past_key_values is not None else 0
            position_ids = torch.arange(inputs_embeds.shape[1], device=inputs_embeds.device) + seen
            position_ids = position_ids.view(1, 1, -1).expand(4, inputs_embeds.shape[0], -1)
        elif position_ids.ndim == 2:
            position_ids = position_ids[None, ...].expand(4, position_ids.shape[0], -1)
        if position_ids.ndim == 3 and position_ids.shape[0] == 4:
            text_position_ids, rotary_position_ids = position_ids[0], position_ids[1:]
        else:
            text_position_ids, rotary_position_ids = None, position_ids
        padded = attention_mask is not None and not isinstance(attention_mask, dict) and not bool(attention_mask.all())
        if isinstance(attention_mask, dict):
            full_mask, linear_mask = attention_mask.get("full_attention"), attention_mask.get("linear_attention")
        elif padded:
            full_mask = qwen_impl.create_causal_mask(config=self.config, inputs_embeds=inputs_embeds,
                                                     attention_mask=attention_mask, past_key_values=past_key_values,
                                                     position_ids=text_position_ids)
            linear_mask = self._update_linear_attn_mask(attention_mask, past_key_values)
        else:  # unpadded: the kernels are causal by construction (static decode passes no mask)
            full_mask, linear_mask = None, None
        position_embeddings = self.rotary_emb(inputs_embeds, rotary_position_ids)
        residual = inputs_embeds.contiguous()
        normalized = K.rms_norm(residual, self.layers[0].input_layernorm.weight, self.layers[0].input_layernorm.eps)
        n_layers = self.config.num_hidden_layers
        for index, layer in enumerate(self.layers[:n_layers]):
            if layer.layer_type == "linear_attention":
                mixer = layer.linear_attn(hidden_states=normalized, cache_params=past_key_values,
                                          attention_mask=linear_mask)
            else:
                mixer, _ = layer.self_attn(hidden_states=normalized, attention_mask=full_mask,
                                           position_ids=text_position_ids, past_key_values=past_key_values,
                                           position_embeddings=position_embeddings)
            residual, mlp_in = K.residual_add_rms_norm(residual, mixer.contiguous(),
                                                       layer.post_attention_layernorm.weight,
                                                       layer.post_attention_layernorm.eps)
            mlp = layer.mlp(mlp_in)
            nxt = self.layers[index + 1].input_layernorm if index + 1 < n_layers else self.norm
            residual, normalized = K.residual_add_rms_norm(residual, mlp.contiguous(), nxt.weight, nxt.eps)
        return qwen_impl.Qwen3_5ModelOutputWithPast(last_hidden_state=normalized, past_key_values=past_key_values)

    _install(text_model, forward, config, "input_ids")


def _vision_dims(cfg) -> "VisionDims":
    from .config import VisionDims

    side = int(round(cfg.num_position_embeddings ** 0.5))
    if side * side != cfg.num_position_embeddings:
        raise ValueError("the vision position table must be square")
    return VisionDims(depth=cfg.depth, width=cfg.hidden_size, heads=cfg.num_heads,
                      intermediate=cfg.intermediate_size, in_channels=cfg.in_channels, patch=cfg.patch_size,
                      temporal_patch=cfg.temporal_patch_size, merge=cfg.spatial_merge_size,
                      out_width=cfg.out_hidden_size, pos_side=side)


def _patch_vision_model(visual: torch.nn.Module, config: FusionConfig) -> bool:
    """integration.py:509-637: the vision forward of Qwen3_5VisionModel on this package's ViT
    runner (q35_vit_encode_patches: tcgen05 projections, fused position embedding + norm, QKV RoPE,
    attention, residual + norm, merger), one image (one ``grid_thw`` row) at a time, over the
    module's own weights (no copies). Video grids (t > 1) raise unless ``eager_fallback``."""
    vcfg = visual.config
    if vcfg.hidden_act != "gelu_pytorch_tanh" or vcfg.hidden_size // vcfg.num_heads != 64:
        return False
    vd = _vision_dims(vcfg)
    state = {k: v for k, v in visual.state_dict().items() if "inv_freq" not in k}

    def forward(self, hidden_states, grid_thw, **kwargs):
        from transformers.modeling_outputs import BaseModelOutputWithPooling

        from .vision import VisionEngine

        grids = [tuple(int(v) for v in row) for row in grid_thw.tolist()]
        if any(t != 1 for t, _, _ in grids):
            if config.eager_fallback:
                return self._fused_original_forward(hidden_states, grid_thw, **kwargs)
            raise ValueError("fused vision tower: video inputs (t > 1) need FusionConfig(eager_fallback=True)")
        need = max(h * w for _, h, w in grids)
        eng = getattr(self, "_q35_vit", None)
        if eng is None or eng.max_patches < need:
            eng = VisionEngine(state, vd, max_image=(vd.patch * vd.merge, vd.patch * vd.merge),
                               device=hidden_states.device, prefix="", max_patches=need)
            self._q35_vit = eng
        hidden, merged, off = [], [], 0
        for _, h, w in grids:
            n = h * w
            merged.append(eng.encode_patches(hidden_states[off:off + n].float(), h, w))
            hidden.append(eng.hidden(n).clone())
            off += n
        return BaseModelOutputWithPooling(last_hidden_state=torch.cat(hidden), pooler_output=torch.cat(merged))

    return _install(visual, forward, config, "hidden_states", accept=lambda x: x.is_cuda and x.is_floating_point())


def apply_fusions(model: torch.nn.Module, config: FusionConfig | None = None) -> dict:
    """Pack weights and install all enabled inference-only fast paths (integration.py:778-814),
    the vision tower's included when the model has one (``FusionConfig.vision``)."""
    config = config or FusionConfig()
    if model.training:
        raise ValueError("apply_fusions requires model.eval()")
    stats = _pack_linear_weights(model, config)
    visual = getattr(getattr(model, "model", None), "visual", None)
    if config.vision and visual is not None:
        stats["vision"] = int(_patch_vision_model(visual, config))
    text = _text_model(model)
    for layer in text.layers:
        if config.rms_norm:
            _install(layer.input_layernorm, _fused_rms_norm, config, "hidden_states")
            _install(layer.post_attention_layernorm, _fused_rms_norm, config, "hidden_states")
        if config.swiglu:
            _patch_mlp(layer.mlp, config)
        if hasattr(layer, "linear_attn") and config.delta:
            _install(layer.linear_attn.norm, _fused_gated_norm, config, "hidden_states")
            _patch_delta(layer.linear_attn, config)
        if hasattr(layer, "self_attn") and config.attention:
            _install(layer.self_attn.q_norm, _fused_rms_norm, config, "hidden_states")
            _install(layer.self_attn.k_norm, _fused_rms_norm, config, "hidden_states")
            _patch_attention(layer.self_attn, config)
    if config.rms_norm:
        _install(text.norm, _fused_rms_norm, config, "hidden_states")
    if config.residual_norm:
        _patch_text_model(text, config)
    model._qwen35_fusion_config = config
    stats["delta_precompute_factors"] = int(config.delta and config.delta_precompute_factors)
    stats["ppu_swiglu_gemv"] = int(config.swiglu and config.ppu_swiglu_gemv)
    return stats


__all__ = ["FusionConfig", "apply_fusions"]
