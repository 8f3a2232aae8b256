"""CPU restatement of the reference's fused Qwen3.5 text-decoder step (prefill + greedy decode).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows the patched text-model forward of qwen35_fused/integration.py:390-504:

* ``residual = embed(ids)``; ``normalized = rms_norm(residual, layers[0].input_layernorm)``;
* per layer: mixer(normalized) → ``residual, mlp_in = residual_add_rms_norm(residual, mixer,
  post_attention_layernorm)`` → MLP → ``residual, normalized = residual_add_rms_norm(residual,
  mlp, next input_layernorm | final norm)``;
* DeltaNet mixer (integration.py:228-272): packed projection → ``causal_conv1d`` →
  ``delta_recurrent`` (the reference's sequential scan, also used for prefill) →
  ``gated_rms_norm(core, z)`` → ``out_proj``;
* attention mixer (integration.py:282-380): packed QGKV → ``qgkv_norm_rope`` with static-cache
  write → decode ``gqa_decode_attention`` / prefill causal attention → ``attention_gate_mul`` →
  ``o_proj``;
* MLP (integration.py:169-188): ``silu_and_mul(F.linear(x, gate_up))`` → ``down_proj``;
* greedy token: ``lm_head_argmax(normalized[:, -1], embed)`` (evaluation_wrapper.py:360-363).

With ``a8w8=True`` every projection of the M/F/L groups (explore_runtime_quantization.py:66-84)
is an A8W8 linear (``oracle.a8w8``); the tied LM head stays BF16.
"""

from __future__ import annotations

import math

import torch

from . import a8w8 as q8
from . import ops

BF16 = torch.bfloat16


class OracleDecoder:
    def __init__(self, weights: dict, dims, *, a8w8: bool = False, max_cache_len: int = 2048,
                 chunked_prefill: bool = False):
        self.d = dims
        self.w = weights
        self.a8w8 = a8w8
        self.chunked_prefill = chunked_prefill
        self.max_cache_len = max_cache_len
        self.probe: list | None = None  # set to a list to record A8W8 input codes (diagnostics)
        self.inv_freq = ops.rope_inv_freq(dims.rotary_dim, dims.rope_theta)
        self.layers = []
        for i, kind in enumerate(dims.layer_types):
            p = f"model.layers.{i}."
            L = {"kind": kind, "in_ln": weights[p + "input_layernorm.weight"],
                 "post_ln": weights[p + "post_attention_layernorm.weight"]}
            gate_up = torch.cat((weights[p + "mlp.gate_proj.weight"], weights[p + "mlp.up_proj.weight"]), 0)
            L["gate_up"] = self._lin(gate_up)
            L["down"] = self._lin(weights[p + "mlp.down_proj.weight"])
            if kind == "linear_attention":
                la = p + "linear_attn."
                packed = torch.cat((weights[la + "in_proj_qkv.weight"], weights[la + "in_proj_z.weight"],
                                    weights[la + "in_proj_a.weight"], weights[la + "in_proj_b.weight"]), 0)
                L["in_proj"] = self._lin(packed)
                L["out_proj"] = self._lin(weights[la + "out_proj.weight"])
                L["conv_w"] = weights[la + "conv1d.weight"].reshape(dims.conv_dim, dims.conv_kernel)
                L["A_log"] = weights[la + "A_log"]
                L["dt_bias"] = weights[la + "dt_bias"]
                L["gnorm"] = weights[la + "norm.weight"]
            else:
                sa = p + "self_attn."
                qgkv = torch.cat((weights[sa + "q_proj.weight"], weights[sa + "k_proj.weight"],
                                  weights[sa + "v_proj.weight"]), 0)
                L["qgkv"] = self._lin(qgkv)
                L["o_proj"] = self._lin(weights[sa + "o_proj.weight"])
                L["q_norm"] = weights[sa + "q_norm.weight"]
                L["k_norm"] = weights[sa + "k_norm.weight"]
            self.layers.append(L)
        self.embed = weights["model.embed_tokens.weight"]
        self.final_norm = weights["model.norm.weight"]
        self.reset()

    # ------------------------------------------------------------------ helpers
    def _lin(self, w):
        if self.a8w8:
            return ("q8",) + q8.quantize_weight(w)
        return ("bf16", w)

    def _apply(self, lin, x):
        if lin[0] == "q8":
            if self.probe is not None:  # per-token codes and scales of this A8W8 input
                self.probe.append(q8.quantize_tokens(x.reshape(-1, x.shape[-1])))
            return q8.a8w8_linear(x, lin[1], lin[2])
        return ops.linear(x, lin[1])

    def reset(self, batch: int = 1):
        d = self.d
        self.conv_state = [torch.zeros(batch, d.conv_dim, d.conv_kernel, dtype=BF16)
                           for _ in range(d.n_delta)]
        self.rec_state = [torch.zeros(batch, d.lin_heads, d.lin_dk, d.lin_dv, dtype=torch.float32)
                          for _ in range(d.n_delta)]
        self.k_cache = [torch.zeros(batch, d.kv_heads, self.max_cache_len, d.head_dim, dtype=BF16)
                        for _ in range(d.n_attn)]
        self.v_cache = [torch.zeros_like(k) for k in self.k_cache]
        self.length = 0
        self.rope_delta = 0  # text RoPE position minus cache row (non-zero after an image prompt)

    # ------------------------------------------------------------------ mixers
    def _delta(self, j, L, x):
        d = self.d
        b, n, _ = x.shape
        packed = self._apply(L["in_proj"], x)  # [B, n, rows]
        qkv = ops.causal_conv1d(packed, L["conv_w"], self.conv_state[j])
        if self.chunked_prefill and n > 1:
            heads, dk = d.lin_heads, d.lin_dk
            q, k, v = qkv.float().reshape(b, n, 3, heads, dk).unbind(2)
            a_off = 3 * heads * dk + heads * d.lin_dv
            a = packed[..., a_off:a_off + heads]
            bb = packed[..., a_off + heads:a_off + 2 * heads]
            q_hat, k_hat, _alpha, beta, g = ops.delta_factors(q, k, a, bb, L["A_log"], L["dt_bias"], dk)
            core = ops.chunk_gated_delta_rule(q_hat, k_hat, v, g, beta, self.rec_state[j]).to(BF16)
        else:
            core = ops.delta_recurrent(qkv, packed, L["A_log"], L["dt_bias"], self.rec_state[j])
        z0 = d.conv_dim
        z = packed[..., z0:z0 + d.value_dim].reshape(-1, d.lin_dv)
        core = ops.gated_rms_norm(core.reshape(-1, d.lin_dv), z, L["gnorm"], d.eps)
        return self._apply(L["out_proj"], core.reshape(b, n, d.value_dim))

    def _attn(self, j, L, x, positions):
        d = self.d
        b, n, _ = x.shape
        packed = self._apply(L["qgkv"], x)
        cos, sin = ops.rope_cos_sin(positions, self.inv_freq, d.mrope_section)
        q, kc, vc = ops.qgkv_norm_rope(packed, L["q_norm"], L["k_norm"], cos, sin, q_heads=d.q_heads,
                                       kv_heads=d.kv_heads, dim=d.head_dim, rotary_dim=d.rotary_dim,
                                       cache_key=self.k_cache[j], cache_value=self.v_cache[j],
                                       cache_start=self.length)
        valid = self.length + n
        scale = d.head_dim ** -0.5
        if n == 1:
            out = ops.gqa_decode_attention(q, kc, vc, valid, scale)
        else:
            out = ops.causal_attention(q, kc[:, :, :valid], vc[:, :, :valid], scale, q_offset=self.length)
        out = ops.attention_gate_mul(out, packed, d.head_dim)
        return self._apply(L["o_proj"], out)

    # ------------------------------------------------------------------ forward
    def forward(self, ids: torch.Tensor, positions: torch.Tensor | None = None,
                image_embeds: torch.Tensor | None = None, image_rows: torch.Tensor | None = None) -> torch.Tensor:
        """Run ``ids [B, n]`` through the decoder, appending to the caches. Returns the final
        normalised hidden states ``[B, n, H]`` (BF16).

        Multimodal prompts (batch 1): rows ``image_rows`` of the input take ``image_embeds`` instead
        of their token embeddings (Transformers' masked_scatter of the image features), and
        ``positions`` may be the 3-axis M-RoPE positions ``[3, 1, n]``; later calls continue at the
        text position after their maximum (Transformers' rope deltas)."""
        d = self.d
        b, n = ids.shape
        if positions is None:
            positions = (torch.arange(n) + self.length + self.rope_delta)[None].expand(b, n)
        else:
            self.rope_delta = int(positions.max()) + 1 - (self.length + n)
        residual = self.embed[ids]
        if image_embeds is not None:
            residual = residual.clone()
            residual[0, image_rows] = image_embeds.to(residual.dtype)
        normalized = ops.rms_norm(residual, self.layers[0]["in_ln"], d.eps)
        jd = ja = 0
        for i, L in enumerate(self.layers):
            if L["kind"] == "linear_attention":
                mix = self._delta(jd, L, normalized)
                jd += 1
            else:
                mix = self._attn(ja, L, normalized, positions)
                ja += 1
            residual, mlp_in = ops.residual_add_rms_norm(residual, mix, L["post_ln"], d.eps)
            mlp = self._apply(L["down"], ops.silu_and_mul(self._apply(L["gate_up"], mlp_in)))
            nxt = self.layers[i + 1]["in_ln"] if i + 1 < len(self.layers) else self.final_norm
            residual, normalized = ops.residual_add_rms_norm(residual, mlp, nxt, d.eps)
        self.length += n
        return normalized

    def next_token(self, hidden_last: torch.Tensor) -> torch.Tensor:
        return ops.lm_head_argmax(hidden_last, self.embed)

    def generate(self, prompt: torch.Tensor, steps: int, *, return_margins: bool = False):
        """Greedy generation: prefill ``prompt [1, L]`` then ``steps`` decode steps.

        Returns the ``steps + 1`` generated tokens (first from the prefill)."""
        self.reset(prompt.shape[0])
        hidden = self.forward(prompt)
        tokens, margins = [], []
        h = hidden[:, -1]
        for step in range(steps + 1):
            tok = self.next_token(h)
            tokens.append(int(tok[0, 0]))
            if return_margins:
                logits = ops.linear(h, self.embed).float()[0]
                top2 = torch.topk(logits, 2).values
                margins.append(float(top2[0] - top2[1]))
            if step == steps:
                break
            h = self.forward(tok)[:, -1]
        return (tokens, margins) if return_margins else tokens

    def teacher_forced_top1(self, prompt: torch.Tensor, forced: list[int]):
        """At every step, fed ``forced`` tokens: ``(oracle top-1, its BF16 logit, the BF16 logit
        of the forced token)``."""
        self.reset(prompt.shape[0])
        h = self.forward(prompt)[:, -1]
        out = []
        for step in range(len(forced)):
            logits = ops.linear(h, self.embed).float()[0]
            top = int(ops.lm_head_argmax(h, self.embed)[0, 0])
            out.append((top, float(logits[top]), float(logits[forced[step]])))
            if step + 1 < len(forced):
                h = self.forward(torch.tensor([[forced[step]]]))[:, -1]
        return out


def bf16_ulp(x: float) -> float:
    """Spacing of BF16 numbers at ``x``."""
    if x == 0:
        return 2.0 ** -133
    e = math.floor(math.log2(abs(x)))
    return 2.0 ** (e - 7)
