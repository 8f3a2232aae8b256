"""Drop-in surface: apply_fusions on a Transformers Qwen3.5 model, GreedyDecodeGraph over a
StaticCache, and VLMModel.generate_with_metrics, all checked against the CPU oracle."""

import pytest
import torch

from oracle.model import OracleDecoder, bf16_ulp
from ppu_b200.config import FusionConfig, Qwen35Dims
from ppu_b200.evaluation_wrapper import GenerationConfig, GenerationResult, VLMModel, compute_throughput
from ppu_b200.synthetic import make_prompt, make_weights

pytestmark = pytest.mark.gpu

# Smallest shape the kernels are built for: attention head 256, linear-attention heads 128.
TINY = Qwen35Dims(vocab=1024, hidden=512, intermediate=1024, layers=4, q_heads=2, kv_heads=1, lin_heads=2)


def _hf_model(dims, weights):
    from transformers.models.qwen3_5 import modeling_qwen3_5 as hf

    cfg = hf.Qwen3_5TextConfig(
        vocab_size=dims.vocab, hidden_size=dims.hidden, intermediate_size=dims.intermediate,
        num_hidden_layers=dims.layers, num_attention_heads=dims.q_heads, num_key_value_heads=dims.kv_heads,
        head_dim=dims.head_dim, linear_num_key_heads=dims.lin_heads, linear_num_value_heads=dims.lin_heads,
        linear_key_head_dim=dims.lin_dk, linear_value_head_dim=dims.lin_dv, tie_word_embeddings=True,
        rope_parameters={"rope_type": "default", "rope_theta": dims.rope_theta, "partial_rotary_factor": 0.25,
                         "mrope_section": list(dims.mrope_section), "mrope_interleaved": True})
    model = hf.Qwen3_5ForCausalLM(cfg).to(torch.bfloat16)
    model.load_state_dict({k: v for k, v in weights.items()}, strict=False)
    model.lm_head.weight = model.model.embed_tokens.weight
    return model.cuda().eval()


def _assert_greedy_ok(weights, dims, prompt, tokens, a8w8=False):
    ref = OracleDecoder(weights, dims, a8w8=a8w8, max_cache_len=512).teacher_forced_top1(prompt, tokens)
    for tok, (top, top_val, tok_val) in zip(tokens, ref):
        assert tok == top or tok_val >= top_val - bf16_ulp(top_val), (tokens, [r[0] for r in ref])


@pytest.mark.parametrize("a8w8", [False, True])
def test_apply_fusions_static_cache_graph(a8w8):
    from transformers.cache_utils import StaticCache

    from ppu_b200.graph import GreedyDecodeGraph
    from ppu_b200.integration import apply_fusions
    from ppu_b200.kernels import lm_head_argmax

    w = make_weights(TINY, seed=21)
    prompt = make_prompt(TINY, 37, seed=22)
    model = _hf_model(TINY, w)
    stats = apply_fusions(model, FusionConfig(a8w8=a8w8))
    assert stats["delta"] == 3 and stats["attention"] == 1 and stats["mlp"] == 4
    cache = StaticCache(config=model.config, max_cache_len=512)
    with torch.inference_mode():
        out = model.model(input_ids=prompt.cuda(), past_key_values=cache, use_cache=True, return_dict=True)
        tok = lm_head_argmax(out.last_hidden_state[:, -1, :].contiguous(), model.lm_head.weight)
        tokens = [int(tok)]
        pos = torch.full((4, 1, 1), prompt.shape[1], device="cuda", dtype=torch.int64)
        runner = GreedyDecodeGraph(model, cache, tok, pos, steps=1)
        for _ in range(8):
            tokens.append(int(runner.replay().item()))
    _assert_greedy_ok(w, TINY, prompt, tokens, a8w8=a8w8)


def test_apply_fusions_dynamic_cache_eager_decode():
    from ppu_b200.integration import apply_fusions
    from ppu_b200.kernels import lm_head_argmax

    w = make_weights(TINY, seed=31)
    prompt = make_prompt(TINY, 20, seed=32)
    model = _hf_model(TINY, w)
    apply_fusions(model)
    with torch.inference_mode():
        out = model.model(input_ids=prompt.cuda(), use_cache=True, return_dict=True)
        cache = out.past_key_values
        tok = lm_head_argmax(out.last_hidden_state[:, -1, :].contiguous(), model.lm_head.weight)
        tokens = [int(tok)]
        for _ in range(5):
            out = model.model(input_ids=tok, past_key_values=cache, use_cache=True, return_dict=True)
            tok = lm_head_argmax(out.last_hidden_state[:, -1, :].contiguous(), model.lm_head.weight)
            tokens.append(int(tok))
    _assert_greedy_ok(w, TINY, prompt, tokens)


def test_vlmmodel_synthetic_backend():
    dims = Qwen35Dims(layers=4, vocab=4096)
    vm = VLMModel(backend="synthetic", dims=dims, seed=5, max_len=512, max_prefill=256)
    assert vm.backend_name == "synthetic"
    prompt = make_prompt(dims, 100, seed=6)[0].tolist()
    res = vm.generate_with_metrics(image=None, prompt=prompt, choices={"A": "x"},
                                   generation_config=GenerationConfig(max_new_tokens=12), sample_id="s0")
    assert isinstance(res, GenerationResult) and res.token_count == 12
    assert 0 < res.ttft_seconds < res.elapsed_seconds
    assert compute_throughput(res) > 0
    tokens = [int(t) for t in res.text.split()]
    w = {k: v.cpu() for k, v in make_weights(dims, seed=5, device="cuda").items()}  # the backend seeds on device
    _assert_greedy_ok(w, dims, torch.tensor([prompt]), tokens)
    # a second request reuses the engine, the cache and the captured graph
    res2 = vm.generate_with_metrics(image=None, prompt=prompt, generation_config=GenerationConfig(max_new_tokens=12))
    assert res2.text == res.text


def test_vlmmodel_transformers_backend(tmp_path):
    w = make_weights(TINY, seed=41)
    model = _hf_model(TINY, w)
    model.save_pretrained(tmp_path)
    vm = VLMModel(str(tmp_path), backend="transformers")
    prompt = make_prompt(TINY, 30, seed=42)[0].tolist()
    res = vm.generate_with_metrics(image=None, prompt=prompt, generation_config=GenerationConfig(max_new_tokens=6))
    assert res.meta["backend"] == "transformers-b200-fused" and res.token_count == 6
    _assert_greedy_ok(w, TINY, torch.tensor([prompt]), [int(t) for t in res.text.split()])


def test_dummy_backend_matches_reference_contract():
    vm = VLMModel(backend="dummy")
    res = vm.generate_with_metrics(image=None, prompt="q", choices={"A": "a", "B": "b"},
                                   generation_config=GenerationConfig(max_new_tokens=8), sample_id="x")
    assert res.meta["backend"] == "dummy" and res.text.startswith("Answer: ")


def test_apply_fusions_vision_tower_matches_eager():
    """integration.py:509-637 drop-in: Transformers' Qwen3_5VisionModel forward replaced by the ViT
    runner over the module's own weights, against the unpatched eager forward on the GPU."""
    from pathlib import Path

    from transformers.models.qwen3_5 import modeling_qwen3_5 as hf
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5VisionConfig

    from ppu_b200.config import VisionDims
    from ppu_b200.integration import _patch_vision_model
    from ppu_b200.synthetic import make_vision_weights

    from .helpers import rel_err

    g = torch.load(Path(__file__).parent / "golden" / "golden_vision.pt", weights_only=False)
    c = g["vision_model"]
    vd = VisionDims(**c["dims"])
    cfg = Qwen3_5VisionConfig(depth=vd.depth, hidden_size=vd.width, num_heads=vd.heads,
                              intermediate_size=vd.intermediate, out_hidden_size=vd.out_width,
                              num_position_embeddings=vd.pos_side ** 2, hidden_act="gelu_pytorch_tanh")
    cfg._attn_implementation = "eager"
    visual = hf.Qwen3_5VisionModel(cfg).to(torch.bfloat16)
    visual.load_state_dict({k[len("model.visual."):]: v for k, v in make_vision_weights(vd, seed=c["seed"]).items()},
                           strict=False)
    visual = visual.cuda().eval()
    visual.rotary_pos_emb.inv_freq = (1.0 / (10000.0 ** (torch.arange(0, 32, 2, dtype=torch.float) / 32))).cuda()
    pix = g["patchify"]["pixel_values"].cuda().to(torch.bfloat16)
    grid = g["patchify"]["grid_thw"].cuda()
    two = torch.cat((pix, pix)), torch.cat((grid, grid))  # two images in one call
    with torch.inference_mode():
        want = visual(*two)
        assert _patch_vision_model(visual, FusionConfig())
        got = visual(*two)
    assert got.pooler_output.shape == want.pooler_output.shape == (12, vd.out_width)
    assert rel_err(got.last_hidden_state, want.last_hidden_state) < 1e-2
    assert rel_err(got.pooler_output, want.pooler_output) < 1e-2
    assert torch.equal(got.pooler_output[:6], got.pooler_output[6:])


def test_vlmmodel_synthetic_backend_with_an_image():
    """generate_with_metrics(image=...) on the synthetic backend: the ViT + M-RoPE prefill path;
    the same request twice gives the same tokens, and the image changes the answer's context."""
    from ppu_b200.synthetic import make_image

    dims = Qwen35Dims(layers=4, vocab=4096)
    vm = VLMModel(backend="synthetic", dims=dims, seed=5, max_len=512, max_prefill=256)
    prompt = make_prompt(dims, 60, seed=7)[0].tolist()
    img = make_image(64, 96, seed=8)
    cfg = GenerationConfig(max_new_tokens=10)
    res = vm.generate_with_metrics(image=img, prompt=prompt, generation_config=cfg)
    assert res.meta["image"] and res.token_count == 10 and 0 < res.ttft_seconds < res.elapsed_seconds
    again = vm.generate_with_metrics(image=img, prompt=prompt, generation_config=cfg)
    assert again.text == res.text
    text_only = vm.generate_with_metrics(image=None, prompt=prompt, generation_config=cfg)
    assert not text_only.meta["image"]
