"""Vision tower on the GPU (C ABI) against the CPU oracle and the golden vectors: the fused
operators of kernels.py:336-416 and 1188-1336, the biased tcgen05 projections, the attention, and
the whole ViT + merger (integration.py:509-736) at the golden's small shape and at BASELINE config
5's shape (24 layers, width 1024, 448 x 448 image -> 196 tokens of 2048)."""

from pathlib import Path

import pytest
import torch

from oracle import vision as OV
from ppu_b200 import kernels as K
from ppu_b200 import lib as L
from ppu_b200.config import VisionDims
from ppu_b200.synthetic import make_image, make_vision_weights
from ppu_b200.vision import VisionEngine

from .helpers import assert_bf16_close, rel_err

pytestmark = pytest.mark.gpu

G = torch.load(Path(__file__).parent / "golden" / "golden_vision.pt", weights_only=False)
BF16 = torch.bfloat16


def cu(t):
    return t.cuda()


def randn(*shape, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(BF16)


@pytest.mark.parametrize("rows,width", [(13, 1024), (784, 1024), (5, 256), (7, 1000)])
def test_layer_norm_and_residual_variant(rows, width):
    x, u = randn(rows, width, seed=1), randn(rows, width, seed=2)
    w, b = randn(width, seed=3), randn(width, seed=4)
    assert_bf16_close(K.layer_norm(cu(x), cu(w), cu(b)).cpu(), OV.layer_norm(x, w, b), max_ulp=1, max_frac=0.02)
    r, n = K.residual_add_layer_norm(cu(x), cu(u), cu(w), cu(b))
    ra, na = OV.residual_add_layer_norm(x, u, w, b)
    assert torch.equal(r.cpu(), ra)
    assert_bf16_close(n.cpu(), na, max_ulp=1, max_frac=0.02)


def test_golden_layer_norms_and_position_embedding():
    c = G["layer_norm"]
    assert_bf16_close(K.layer_norm(cu(c["x"]), cu(c["w"]), cu(c["b"])).cpu(), c["out"], max_ulp=1, max_frac=0.02)
    c = G["residual_add_layer_norm"]
    r, n = K.residual_add_layer_norm(cu(c["x"]), cu(c["u"]), cu(c["w"]), cu(c["b"]))
    assert torch.equal(r.cpu(), c["added"])
    assert_bf16_close(n.cpu(), c["out"], max_ulp=1, max_frac=0.02)
    c = G["position_embed_add"]
    got = K.position_embed_add(cu(c["x"]), cu(c["table"]), cu(c["idx"]), cu(c["wts"]))
    assert_bf16_close(got.cpu(), c["out"], max_ulp=1, max_frac=0.02)


def test_golden_vision_qkv_rope_bit_exact():
    c = G["vision_qkv_rope"]
    q, k, v = K.vision_qkv_rope(cu(c["packed"]), cu(c["cos"]), cu(c["sin"]), heads=c["heads"], dim=c["dim"])
    assert torch.equal(q.cpu(), c["q"]) and torch.equal(k.cpu(), c["k"]) and torch.equal(v.cpu(), c["v"])


def test_vision_qkv_rope_rejects_bad_shapes():
    with pytest.raises(ValueError, match="width"):
        K.vision_qkv_rope(torch.zeros(4, 100, device="cuda", dtype=BF16), torch.zeros(4, 64), torch.zeros(4, 64),
                          heads=1, dim=64)


@pytest.mark.parametrize("tokens,heads", [(784, 16), (24, 4), (70, 2)])
def test_vision_attention_matches_fp32_softmax(tokens, heads):
    q, k, v = (randn(1, heads, tokens, 64, seed=s) for s in (11, 12, 13))
    got = K.vision_attention(cu(q), cu(k), cu(v), 0.125)
    want = OV.attention(q, k, v, 0.125)
    s = (q.float() @ k.float().transpose(-1, -2)) * 0.125
    exact = (torch.softmax(s, -1) @ v.float())[0].transpose(0, 1).reshape(tokens, -1)
    assert rel_err(got, want) < 1e-2
    assert rel_err(got, exact) < 1e-2


@pytest.mark.parametrize("m,n,k,epi", [(784, 3072, 1024, L.EPI_BIAS), (784, 4096, 1024, L.EPI_BIAS_GELU_TANH),
                                       (196, 4096, 4096, L.EPI_BIAS_GELU), (196, 2048, 4096, L.EPI_BIAS),
                                       (784, 1024, 1536, L.EPI_BIAS)])
def test_gemm_bias_epilogues(m, n, k, epi):
    a, w, b = randn(m, k, seed=21), randn(n, k, seed=22, scale=0.02), randn(n, seed=23, scale=0.5)
    got = K.gemm_bias(cu(a), cu(w), cu(b), epilogue=epi)
    torch.cuda.synchronize()
    assert K.tc_error() == 0
    want = OV.linear(a, w, b)
    if epi == L.EPI_BIAS_GELU_TANH:
        want = OV.gelu_tanh(want)
    elif epi == L.EPI_BIAS_GELU:
        want = OV.gelu(want)
    assert rel_err(got, want) < 1e-2
    if epi == L.EPI_BIAS:
        assert_bf16_close(got.cpu(), want, max_ulp=2, max_frac=0.05)
    else:
        # GELU's negative tail turns a one-ulp difference of its bf16 input into many ulps of a
        # tiny output: bound the error by the input's ulp at the largest magnitude (gelu' <= 1.13)
        err = (got.cpu().float() - want.float()).abs().max()
        assert float(err) <= 2.0 ** -6 * float(want.float().abs().max())


def test_patchify_and_rope_table():
    vd = VisionDims()
    img = make_image(448, 448, seed=4)
    out = torch.empty(784, vd.patch_features, device="cuda", dtype=BF16)
    L.call("q35_vision_patchify", cu(img).data_ptr(), out.data_ptr(), 3, 448, 448, 16, 2, 2, 0.5, 0.5,
           L.stream_of())
    assert torch.equal(out.cpu(), OV.patchify(img, vd))
    inv = OV.rope_inv_freq(64)
    cos = torch.empty(784, 64, device="cuda")
    sin = torch.empty_like(cos)
    L.call("q35_vision_rope_table", cu(inv).data_ptr(), cos.data_ptr(), sin.data_ptr(), 28, 28, 2, L.stream_of())
    c_ref, s_ref = OV.rope_cos_sin(28, 28, 2, inv)
    assert torch.allclose(cos.cpu(), c_ref, atol=2e-6) and torch.allclose(sin.cpu(), s_ref, atol=2e-6)


def test_vit_small_matches_golden_and_oracle():
    c = G["vision_model"]
    vd = VisionDims(**c["dims"])
    w = make_vision_weights(vd, seed=c["seed"])
    img = make_image(c["height"], c["width"], seed=c["image_seed"])
    eng = VisionEngine(w, vd, max_image=(c["height"], c["width"]))
    merged = eng.encode(cu(img))
    torch.cuda.synchronize()
    assert K.tc_error() == 0
    hidden = eng.hidden(merged.shape[0] * 4).cpu()
    h_ref, m_ref = OV.VisionOracle(w, vd).forward(img)
    assert rel_err(hidden, h_ref) < 1e-2 and rel_err(merged, m_ref) < 1e-2
    assert rel_err(hidden, c["hidden"]) < 1e-2 and rel_err(merged, c["merged"]) < 1e-2


def test_vit_config5_shape_matches_oracle_and_graph_replay():
    vd = VisionDims()
    w = make_vision_weights(vd, seed=9)
    img = make_image(448, 448, seed=10)
    eng = VisionEngine(w, vd)
    merged = eng.encode(cu(img))
    torch.cuda.synchronize()
    assert merged.shape == (196, 2048) and K.tc_error() == 0
    # 24 blocks in bf16 drift from the exact (FP32) forward by ~1.3 % in the oracle itself, so the
    # GPU result is held to the exact forward: no further from it than 1.5x the oracle's own
    # bf16 drift, and within 2 % of it; and within 2 % of the bf16 oracle
    h_ref, m_ref = OV.VisionOracle(w, vd).forward(img)
    h_exact, m_exact = OV.VisionOracle(w, vd, dtype=torch.float32).forward(img)
    hidden = eng.hidden(784).cpu()
    for got, ref, exact in ((hidden, h_ref, h_exact), (merged.cpu(), m_ref, m_exact)):
        own = rel_err(ref, exact)
        print(f"oracle bf16 vs exact {own:.4f}, GPU vs exact {rel_err(got, exact):.4f}, GPU vs oracle "
              f"{rel_err(got, ref):.4f}")
        assert rel_err(got, exact) <= max(1.5 * own, 1e-2) and rel_err(got, exact) < 2e-2
        assert rel_err(got, ref) < 2e-2
    graph, pix, out = eng.capture(448, 448)
    pix.copy_(cu(img))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, merged)


def test_vit_batch_of_images_matches_one_at_a_time():
    """q35_vit_encode_batch: three images through one launch sequence (GEMMs over all patches,
    position embedding / RoPE / attention per image) against three single encodes, and the
    captured batch graph against the eager batch."""
    c = G["vision_model"]
    vd = VisionDims(**c["dims"])
    w = make_vision_weights(vd, seed=c["seed"])
    h, wd = c["height"], c["width"]
    n_patch = vd.grid(h, wd)[0] * vd.grid(h, wd)[1]
    eng = VisionEngine(w, vd, max_image=(h, wd), max_patches=3 * n_patch)
    imgs = torch.stack([make_image(h, wd, seed=40 + i) for i in range(3)])
    batch = eng.encode_batch(cu(imgs)).cpu()
    m = vd.merged_tokens(h, wd)
    assert batch.shape == (3 * m, vd.out_width)
    for i in range(3):
        alone = eng.encode(cu(imgs[i])).cpu()
        assert_bf16_close(batch[i * m:(i + 1) * m], alone, max_ulp=2, max_frac=0.02)
    graph, pix, out = eng.capture(h, wd, images=3)
    pix.copy_(cu(imgs))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), batch)
    with pytest.raises(ValueError, match="max_patches"):
        eng.encode_batch(cu(torch.stack([imgs[0]] * 4)))
