"""The vision-tower oracle against the golden vectors (CPU): the reference's fused-operator
expectations (validate_kernels.py:146-200), Transformers' image-processor patch layout, and
Transformers' eager Qwen3_5VisionModel at a small shape."""

from pathlib import Path

import torch

from oracle import vision as OV
from ppu_b200.config import VisionDims
from ppu_b200.synthetic import make_image, make_vision_weights

from .helpers import assert_bf16_close, rel_err

G = torch.load(Path(__file__).parent / "golden" / "golden_vision.pt", weights_only=False)


def test_layer_norms_match_reference_expectations():
    c = G["layer_norm"]
    assert_bf16_close(OV.layer_norm(c["x"], c["w"], c["b"]), c["out"], max_ulp=1, max_frac=0.02)
    c = G["residual_add_layer_norm"]
    added, out = OV.residual_add_layer_norm(c["x"], c["u"], c["w"], c["b"])
    assert torch.equal(added, c["added"])
    assert_bf16_close(out, c["out"], max_ulp=1, max_frac=0.02)


def test_position_embed_add_matches_reference_expectation():
    c = G["position_embed_add"]
    assert_bf16_close(OV.position_embed_add(c["x"], c["table"], c["idx"], c["wts"]), c["out"], max_ulp=1,
                      max_frac=0.02)


def test_vision_qkv_rope_matches_reference_expectation():
    c = G["vision_qkv_rope"]
    q, k, v = OV.vision_qkv_rope(c["packed"], c["cos"], c["sin"], c["heads"], c["dim"])
    assert torch.equal(q, c["q"]) and torch.equal(k, c["k"]) and torch.equal(v, c["v"])


def test_patchify_matches_the_image_processor():
    c = G["patchify"]
    vd = VisionDims()
    got = OV.patchify(c["pixels"], vd)
    assert c["grid_thw"].tolist() == [[1, 4, 6]]
    assert torch.equal(got, c["pixel_values"].to(torch.bfloat16))


def test_interpolation_weights_sum_to_one_and_hit_the_corners():
    idx, wts = OV.interp_indices_weights(28, 28, 48, 2)
    assert torch.allclose(wts.sum(-1), torch.ones(28 * 28), atol=1e-6)
    assert int(idx.min()) == 0 and int(idx.max()) == 48 * 48 - 1
    rows, cols = OV.token_grid(28, 28, 2)
    assert rows[:4].tolist() == [0, 0, 1, 1] and cols[:4].tolist() == [0, 1, 0, 1]


def test_vision_oracle_matches_transformers_eager_tower():
    c = G["vision_model"]
    vd = VisionDims(**c["dims"])
    weights = make_vision_weights(vd, seed=c["seed"])
    img = make_image(c["height"], c["width"], seed=c["image_seed"])
    hidden, merged = OV.VisionOracle(weights, vd).forward(img)
    # the eager tower rounds the bilinear weights and their partial sums to bf16 where the fused
    # operator accumulates in FP32 (kernels.py:1290-1336); everything else agrees to rounding
    assert rel_err(hidden, c["hidden"]) < 1e-2
    assert rel_err(merged, c["merged"]) < 1e-2
