"""apply_fusions on the CPU: the patched model refuses inputs the B200 kernels cannot take
(no silent CPU path), unless ``FusionConfig(eager_fallback=True)`` asks for the reference's
behaviour of running the original Transformers forwards (qwen35_fused/integration.py:51-52)."""

import pytest
import torch

from ppu_b200.config import FusionConfig, Qwen35Dims
from ppu_b200.synthetic import make_prompt, make_weights

TINY = Qwen35Dims(vocab=1024, hidden=512, intermediate=1024, layers=4, q_heads=2, kv_heads=1, lin_heads=2)


def _cpu_model(dims, weights):
    from transformers.models.qwen3_5 import modeling_qwen3_5 as hf

    cfg = hf.Qwen3_5TextConfig(
        vocab_size=dims.vocab, hidden_size=dims.hidden, intermediate_size=dims.intermediate,
        num_hidden_layers=dims.layers, num_attention_heads=dims.q_heads, num_key_value_heads=dims.kv_heads,
        head_dim=dims.head_dim, linear_num_key_heads=dims.lin_heads, linear_num_value_heads=dims.lin_heads,
        linear_key_head_dim=dims.lin_dk, linear_value_head_dim=dims.lin_dv, tie_word_embeddings=True,
        rope_parameters={"rope_type": "default", "rope_theta": dims.rope_theta, "partial_rotary_factor": 0.25,
                         "mrope_section": list(dims.mrope_section), "mrope_interleaved": True})
    model = hf.Qwen3_5ForCausalLM(cfg).to(torch.bfloat16)
    model.load_state_dict(dict(weights), strict=False)
    return model.eval()


def test_patched_model_rejects_cpu_inputs():
    from ppu_b200.integration import apply_fusions

    model = _cpu_model(TINY, make_weights(TINY, seed=3))
    apply_fusions(model, FusionConfig(release_original_weights=False))
    ids = make_prompt(TINY, 9, seed=4)
    with pytest.raises(ValueError, match="BF16 CUDA"):
        model.model(input_ids=ids)
    with pytest.raises(ValueError, match="BF16 CUDA"):
        model.model.layers[0].mlp(torch.zeros(1, 1, TINY.hidden, dtype=torch.bfloat16))


def test_eager_fallback_runs_the_transformers_forwards():
    from ppu_b200.integration import apply_fusions

    w = make_weights(TINY, seed=5)
    ids = make_prompt(TINY, 9, seed=6)
    plain = _cpu_model(TINY, w)
    with torch.inference_mode():
        want = plain.model(input_ids=ids).last_hidden_state
    model = _cpu_model(TINY, w)
    apply_fusions(model, FusionConfig(release_original_weights=False, eager_fallback=True))
    with torch.inference_mode():
        got = model.model(input_ids=ids).last_hidden_state
    assert torch.equal(got, want)
