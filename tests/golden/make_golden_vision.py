#!/usr/bin/env python3
"""Generate golden vectors for the vision-tower oracle (``oracle/vision.py``).

Sources, all run on the CPU in this container:

* the expectations ``qwen35_fused/validate_kernels.py:146-200`` builds for the fused vision
  operators (layer_norm, residual_add_layer_norm, position_embed_add, vision_qkv_rope) with plain
  torch ops, reproduced here with the reference's shapes (13 rows of width 1024; 13 tokens x 4
  heads x 64) and its seed (20260819);
* Transformers' ``Qwen2VLImageProcessor`` (the processor the reference's wrapper loads) for the
  patch layout of one 64 x 96 image;
* Transformers' eager ``Qwen3_5VisionModel`` at a small shape (depth 2, width 256, 4 heads,
  intermediate 512, 2x2 merge to 512, a 16 x 16 position table) holding
  ``ppu_b200.synthetic.make_vision_weights(seed=5)``, run on that image: the final patch states
  and the merged tokens.

The reference project itself is only read for its expectations' formulas; nothing of it is
imported. Output: ``tests/golden/golden_vision.pt`` (a few hundred KB).
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

TINY = dict(depth=2, width=256, heads=4, intermediate=512, out_width=512, pos_side=16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE / "golden_vision.pt"))
    args = ap.parse_args()
    from transformers import Qwen2VLImageProcessor
    from transformers.models.qwen3_5 import modeling_qwen3_5 as hf
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5VisionConfig

    from ppu_b200.config import VisionDims
    from ppu_b200.synthetic import make_image, make_vision_weights

    torch.manual_seed(20260819)
    dt = torch.bfloat16
    g: dict[str, object] = {}

    # --- fused operators (validate_kernels.py:146-200)
    x = torch.randn(13, 1024, dtype=dt)
    u = torch.randn_like(x)
    w = torch.randn(1024, dtype=dt)
    b = torch.randn(1024, dtype=dt)
    g["layer_norm"] = dict(x=x, w=w, b=b, out=F.layer_norm(x, (1024,), w, b, 1e-6))
    added = x + u
    g["residual_add_layer_norm"] = dict(x=x, u=u, w=w, b=b, added=added,
                                        out=F.layer_norm(added, (1024,), w, b, 1e-6))
    table = torch.randn(64, 1024, dtype=dt)
    idx = torch.randint(0, 64, (13, 4))
    interp = torch.rand(13, 4)
    g["position_embed_add"] = dict(x=x, table=table, idx=idx, wts=interp,
                                   out=x + (F.embedding(idx, table) * interp[:, :, None]).sum(1).to(dt))
    tokens, heads, dim = 13, 4, 64
    packed = torch.randn(tokens, 3 * heads * dim, dtype=dt)
    cos = torch.randn(tokens, dim, dtype=torch.float32)
    sin = torch.randn_like(cos)
    q, k, v = packed.view(tokens, 3, heads, dim).permute(1, 0, 2, 3).unbind(0)

    def rope_ref(t):
        t32 = t.float()
        rot = torch.cat((-t32[..., dim // 2:], t32[..., :dim // 2]), dim=-1)
        return (t32 * cos[:, None, :] + rot * sin[:, None, :]).to(dt)

    g["vision_qkv_rope"] = dict(packed=packed, cos=cos, sin=sin, heads=heads, dim=dim,
                                q=rope_ref(q).transpose(0, 1).unsqueeze(0), k=rope_ref(k).transpose(0, 1).unsqueeze(0),
                                v=v.transpose(0, 1).unsqueeze(0).contiguous())

    # --- processor patch layout (one 64 x 96 image, pixels already rescaled to [0, 1))
    img = make_image(64, 96, seed=3)
    proc = Qwen2VLImageProcessor(patch_size=16, temporal_patch_size=2, merge_size=2, image_mean=[0.5] * 3,
                                 image_std=[0.5] * 3, do_resize=False, do_rescale=False)
    feats = proc(images=[img.numpy().astype(np.float32)], return_tensors="pt", input_data_format="channels_first")
    g["patchify"] = dict(pixels=img, pixel_values=feats["pixel_values"], grid_thw=feats["image_grid_thw"])

    # --- eager vision tower at a small shape
    vd = VisionDims(**TINY)
    weights = make_vision_weights(vd, seed=5)
    cfg = Qwen3_5VisionConfig(depth=vd.depth, hidden_size=vd.width, num_heads=vd.heads,
                              intermediate_size=vd.intermediate, out_hidden_size=vd.out_width,
                              num_position_embeddings=vd.pos_side ** 2, patch_size=vd.patch,
                              temporal_patch_size=vd.temporal_patch, spatial_merge_size=vd.merge,
                              in_channels=vd.in_channels, hidden_act="gelu_pytorch_tanh")
    cfg._attn_implementation = "eager"
    model = hf.Qwen3_5VisionModel(cfg).to(dt).eval()
    # the rotary inverse frequencies stay FP32 as in a checkpoint loaded in bf16 (.to() cast them)
    model.rotary_pos_emb.inv_freq = 1.0 / (10000.0 ** (torch.arange(0, 32, 2, dtype=torch.float) / 32))
    state = {k[len("model.visual."):]: v for k, v in weights.items()}
    missing, unexpected = model.load_state_dict(state, strict=False)
    assert not unexpected and all("inv_freq" in m for m in missing), (missing, unexpected)
    with torch.inference_mode():
        out = model(feats["pixel_values"].to(dt), grid_thw=feats["image_grid_thw"])
    g["vision_model"] = dict(dims=TINY, seed=5, image_seed=3, height=64, width=96,
                             hidden=out.last_hidden_state, merged=out.pooler_output)
    torch.save(g, args.out)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
