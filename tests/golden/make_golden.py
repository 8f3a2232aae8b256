#!/usr/bin/env python3
"""Generate golden vectors for the oracle from the reference's own torch implementations.

Run in a container where the reference project is importable (path given by
``--reference``). It imports, from the reference:

* ``qwen35_fused.validate_kernels.reference_rms / reference_gated / reference_conv /
  reference_delta`` (validate_kernels.py:57-115), and reproduces the eager expectations that
  ``validate_kernels.main`` (validate_kernels.py:118-393) builds with plain torch ops, with the
  same seed (20260819) on the CPU;
* ``explore_runtime_quantization.PPUA8W8Linear`` (explore_runtime_quantization.py:129-158) for
  the int8 weight quantisation;

and, from the installed Transformers, the eager Qwen3.5 modules (RMSNorm, gated RMSNorm,
``torch_chunk_gated_delta_rule``, ``torch_recurrent_gated_delta_rule``, and a tiny random
``Qwen3_5ForCausalLM`` for greedy decoding).

Shapes are shrunk where the reference's would make the fixture large (the SwiGLU GEMV
weight); everything else uses the reference's shapes. Output: ``tests/golden/golden.pt``.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--out", default=str(HERE / "golden.pt"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from qwen35_fused import validate_kernels as vk  # noqa: E402
    import explore_runtime_quantization as erq  # noqa: E402
    from transformers.models.qwen3_5 import modeling_qwen3_5 as hf  # noqa: E402

    torch.manual_seed(20260819)
    dt = torch.bfloat16
    g: dict[str, object] = {}

    # --- norms (validate_kernels.py:130-144, 206-209)
    for width in (128, 256, 2048):
        x = torch.randn(7, width, dtype=dt)
        w = torch.randn(width, dtype=dt)
        g[f"rms_{width}"] = dict(x=x, w=w, out=vk.reference_rms(x, w))
    r = torch.randn(7, 2048, dtype=dt)
    u = torch.randn_like(r)
    w = torch.randn(2048, dtype=dt)
    added = r + u
    g["residual_add_rms"] = dict(r=r, u=u, w=w, added=added, out=vk.reference_rms(added, w))
    x = torch.randn(32, 128, dtype=dt)
    gate = torch.randn_like(x)
    w = torch.randn(128, dtype=dt)
    g["gated_rms"] = dict(x=x, gate=gate, w=w, out=vk.reference_gated(x, gate, w))
    hf_gated = hf.Qwen3_5RMSNormGated(128).to(dt)
    with torch.no_grad():
        hf_gated.weight.copy_(w)
    g["gated_rms_hf"] = dict(x=x, gate=gate, w=w, out=hf_gated(x, gate).detach())
    hf_rms = hf.Qwen3_5RMSNorm(2048).to(dt)
    xr = torch.randn(5, 2048, dtype=dt)
    wr = torch.randn(2048, dtype=dt) * 0.1
    with torch.no_grad():
        hf_rms.weight.copy_(wr)
    g["rms_hf"] = dict(x=xr, w=wr, out=hf_rms(xr).detach())

    # --- activations (validate_kernels.py:211-225)
    packed = torch.randn(7, 12288, dtype=dt)
    g["silu_mul"] = dict(packed=packed, out=F.silu(packed[:, :6144]) * packed[:, 6144:])
    xs = torch.randn(1, 1, 512, dtype=dt)
    ws = torch.randn(2 * 384, 512, dtype=dt) * 0.05
    lin = F.linear(xs, ws)
    g["swiglu_gemv"] = dict(x=xs, w=ws, out=F.silu(lin[..., :384]) * lin[..., 384:])
    gt = torch.randn(7, 2048, dtype=dt)
    val = torch.randn_like(gt)
    g["sigmoid_mul"] = dict(x=val, gate=gt, out=val * gt.sigmoid())

    # --- GQA decode vs SDPA (validate_kernels.py:227-245)
    q = torch.randn(1, 8, 1, 256, dtype=dt)
    keys = torch.randn(1, 2, 512, 256, dtype=dt)
    values = torch.randn_like(keys)
    outs = {}
    for n in (1, 7, 370, 512):
        outs[n] = F.scaled_dot_product_attention(
            q.float(), keys[:, :, :n].float(), values[:, :, :n].float(), scale=0.0625, enable_gqa=True
        ).reshape(1, 1, -1)
    g["gqa_decode"] = dict(q=q, k=keys, v=values, out=outs)

    # --- QGKV norm + RoPE (+ cache write), attention gate (validate_kernels.py:247-325)
    b, L, qh, kvh, hd, rot = 1, 5, 8, 2, 256, 64
    pw = 2 * qh * hd + 2 * kvh * hd
    pq = torch.randn(b, L, pw, dtype=dt)
    qw = torch.randn(hd, dtype=dt)
    kw = torch.randn(hd, dtype=dt)
    cos = torch.randn(b, L, rot, dtype=dt)
    sin = torch.randn_like(cos)
    qpr = pq[..., : 2 * qh * hd].view(b, L, qh, 2 * hd)
    q_raw = qpr[..., :hd]
    k0 = 2 * qh * hd
    k_raw = pq[..., k0 : k0 + kvh * hd].view(b, L, kvh, hd)
    v_raw = pq[..., k0 + kvh * hd :].view(b, L, kvh, hd)
    qn = vk.reference_rms(q_raw, qw).transpose(1, 2)
    kn = vk.reference_rms(k_raw, kw).transpose(1, 2)

    def rope(x):
        rotated = torch.cat((-x[..., rot // 2 : rot], x[..., : rot // 2]), dim=-1)
        front = x[..., :rot] * cos.unsqueeze(1) + rotated * sin.unsqueeze(1)
        return torch.cat((front, x[..., rot:]), dim=-1)

    attn_out = torch.randn(b, L, qh * hd, dtype=dt)
    gate_raw = qpr[..., hd:].reshape(b, L, qh * hd)
    g["qgkv"] = dict(packed=pq, qw=qw, kw=kw, cos=cos, sin=sin, q=rope(qn), k=rope(kn),
                     v=v_raw.transpose(1, 2), attn_out=attn_out, gated=attn_out * gate_raw.sigmoid())

    # --- LM head top-1 and tie KAT (validate_kernels.py:327-342)
    h = torch.randn(1, 128, dtype=dt)
    e = torch.randn(257, 128, dtype=dt)
    g["lm_head"] = dict(h=h, w=e, out=F.linear(h, e).argmax(dim=-1, keepdim=True))
    g["lm_head_tie"] = dict(h=torch.zeros(1, 128, dtype=dt), w=torch.zeros(257, 128, dtype=dt),
                            out=torch.zeros(1, 1, dtype=torch.int64))

    # --- causal conv (validate_kernels.py:344-362)
    for n in (1, 17):
        ch = 64
        x = torch.randn(1, n, ch, dtype=dt)
        cw = torch.randn(ch, 4, dtype=dt)
        init = torch.randn(1, ch, 4, dtype=dt)
        st = init.clone()
        out = vk.reference_conv(x, cw, st)
        px = torch.randn(1, n, ch + 32, dtype=dt)
        pst = init.clone()
        pout = vk.reference_conv(px[..., :ch].contiguous(), cw, pst)
        g[f"conv_{n}"] = dict(x=x, w=cw, state0=init, out=out, state=st, px=px, pout=pout, pstate=pst)

    # --- delta recurrence (validate_kernels.py:364-393)
    b, L, heads, dim = 1, 3, 16, 128
    qkv_w = 3 * heads * dim
    pwid = qkv_w + heads * dim + 2 * heads
    qkv = torch.randn(b, L, qkv_w, dtype=dt)
    pdelta = torch.randn(b, L, pwid, dtype=dt)
    pdelta[..., :qkv_w].copy_(qkv)
    a_log = torch.randn(heads, dtype=dt)
    dt_bias = torch.randn(heads, dtype=dt)
    s0 = torch.randn(b, heads, dim, dim, dtype=torch.float32) * 0.01
    st = s0.clone()
    out = vk.reference_delta(qkv, pdelta, a_log, dt_bias, st)
    g["delta"] = dict(qkv=qkv, packed=pdelta, a_log=a_log, dt_bias=dt_bias, state0=s0, out=out, state=st)

    # --- HF chunked vs recurrent gated delta rule (oracle chunk restatement check)
    gen = torch.Generator().manual_seed(7)
    L2 = 150
    qc = torch.randn(1, L2, 4, 128, generator=gen)
    kc = torch.randn(1, L2, 4, 128, generator=gen)
    vc = torch.randn(1, L2, 4, 128, generator=gen)
    gc = -F.softplus(torch.randn(1, L2, 4, generator=gen))
    bc = torch.sigmoid(torch.randn(1, L2, 4, generator=gen))
    init = torch.randn(1, 4, 128, 128, generator=gen) * 0.05
    o_chunk, s_chunk = hf.torch_chunk_gated_delta_rule(qc, kc, vc, gc, bc, chunk_size=64, initial_state=init,
                                                       output_final_state=True, use_qk_l2norm_in_kernel=True)
    o_rec, s_rec = hf.torch_recurrent_gated_delta_rule(qc, kc, vc, gc, bc, initial_state=init,
                                                       output_final_state=True, use_qk_l2norm_in_kernel=True)
    g["chunk_rule"] = dict(q=qc, k=kc, v=vc, g=gc, beta=bc, state0=init, out_chunk=o_chunk, state_chunk=s_chunk,
                           out_rec=o_rec, state_rec=s_rec)

    # --- A8W8 weight quantisation (explore_runtime_quantization.py:129-158)
    wq = torch.randn(96, 256, dtype=dt) * 0.02
    wq[5].zero_()
    linq = torch.nn.Linear(256, 96, bias=False).to(dt)
    with torch.no_grad():
        linq.weight.copy_(wq)
    mod = erq.PPUA8W8Linear(linq)
    g["a8w8_weight"] = dict(w=wq, q=mod.weight.clone(), scale=mod.weight_scale.clone())

    # --- tiny HF eager decoder: greedy tokens and final hidden state
    cfg = hf.Qwen3_5TextConfig(
        vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=4, num_attention_heads=2,
        num_key_value_heads=1, head_dim=128, linear_num_key_heads=2, linear_num_value_heads=2,
        linear_key_head_dim=64, linear_value_head_dim=64, tie_word_embeddings=True,
        rope_parameters={"rope_type": "default", "rope_theta": 1.0e7, "partial_rotary_factor": 0.25,
                         "mrope_section": [3, 3, 2], "mrope_interleaved": True},
    )
    cfg._attn_implementation = "eager"
    model = hf.Qwen3_5ForCausalLM(cfg).to(dt).eval()
    gen = torch.Generator().manual_seed(11)
    sd = {}
    with torch.no_grad():
        for name, p in model.named_parameters():
            t = torch.randn(p.shape, generator=gen) * 0.02
            if name.endswith("linear_attn.norm.weight"):
                t += 1.0
            p.copy_(t.to(dt))
            sd[name] = p.detach().clone()
    prompt = torch.randint(0, 512, (1, 24), generator=gen)
    with torch.no_grad():
        full = model.model(input_ids=prompt).last_hidden_state
        logits = model.lm_head(full[:, -1])
        out_ids = model.generate(prompt, max_new_tokens=8, do_sample=False, use_cache=True)
    g["tiny_model"] = dict(weights=sd, prompt=prompt, hidden=full, logits=logits,
                           tokens=out_ids[0, prompt.shape[1]:].clone(),
                           dims=dict(vocab=512, hidden=256, intermediate=512, layers=4, q_heads=2, kv_heads=1,
                                     head_dim=128, rotary_dim=32, lin_heads=2, lin_dk=64, lin_dv=64,
                                     mrope_section=(3, 3, 2)))
    torch.save(g, args.out)
    print("wrote", args.out, Path(args.out).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
