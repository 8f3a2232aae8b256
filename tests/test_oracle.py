"""Pin the CPU oracle against the reference's own torch implementations (golden vectors).

The fixtures in tests/golden/golden.pt come from tests/golden/make_golden.py, which runs the
reference's validate_kernels.reference_* functions, its PPUA8W8Linear weight quantiser and
the Transformers eager Qwen3.5 modules.
"""

from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

from oracle import a8w8, ops
from oracle.model import OracleDecoder
from ppu_b200.config import Qwen35Dims

GOLDEN = torch.load(Path(__file__).parent / "golden" / "golden.pt")


def ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Distance in BF16 ulps (of the larger magnitude) between two BF16 tensors."""
    a32, b32 = a.float(), b.float()
    mag = torch.maximum(a32.abs(), b32.abs()).clamp_min(1e-30)
    ulp = torch.exp2(torch.floor(torch.log2(mag)) - 7)
    return (a32 - b32).abs() / ulp


def assert_bf16_close(actual, expected, max_ulp=1.0, max_frac=0.02):
    assert actual.shape == expected.shape, (actual.shape, expected.shape)
    d = ulp_diff(actual, expected)
    assert float(d.max()) <= max_ulp, f"max ulp {float(d.max())}"
    assert float((d > 0).float().mean()) <= max_frac, f"mismatch fraction {float((d > 0).float().mean())}"


def test_rms_norm_golden():
    for w in (128, 256, 2048):
        c = GOLDEN[f"rms_{w}"]
        assert torch.equal(ops.rms_norm(c["x"], c["w"]), c["out"])
    c = GOLDEN["rms_hf"]
    assert torch.equal(ops.rms_norm(c["x"], c["w"]), c["out"])


def test_residual_add_rms_golden():
    c = GOLDEN["residual_add_rms"]
    added, normed = ops.residual_add_rms_norm(c["r"], c["u"], c["w"])
    assert torch.equal(added, c["added"])
    assert torch.equal(normed, c["out"])


def test_gated_rms_golden():
    for key in ("gated_rms", "gated_rms_hf"):
        c = GOLDEN[key]
        # SiLU as x/(1+e^-x) (kernels.py:135) vs x*sigmoid(x) (F.silu): <=1 ulp apart.
        assert_bf16_close(ops.gated_rms_norm(c["x"], c["gate"], c["w"]), c["out"])


def test_silu_mul_and_swiglu_golden():
    c = GOLDEN["silu_mul"]
    assert_bf16_close(ops.silu_and_mul(c["packed"]), c["out"])
    c = GOLDEN["swiglu_gemv"]
    assert_bf16_close(ops.swiglu_gemv(c["x"], c["w"]), c["out"])


def test_sigmoid_mul_golden():
    c = GOLDEN["sigmoid_mul"]
    assert_bf16_close(ops.sigmoid_mul(c["x"], c["gate"]), c["out"])


def test_gqa_decode_golden():
    c = GOLDEN["gqa_decode"]
    for n, expected in c["out"].items():
        out = ops.gqa_decode_attention(c["q"], c["k"], c["v"], n, 0.0625)
        rel = (out.float() - expected).norm() / expected.norm()
        assert rel < 4e-3, (n, float(rel))


def test_qgkv_norm_rope_golden():
    c = GOLDEN["qgkv"]
    kw = dict(q_heads=8, kv_heads=2, dim=256, rotary_dim=64)
    q, k, v = ops.qgkv_norm_rope(c["packed"], c["qw"], c["kw"], c["cos"], c["sin"], **kw)
    assert torch.equal(q, c["q"])
    assert torch.equal(k, c["k"])
    assert torch.equal(v, c["v"])
    kc = torch.zeros(1, 2, 13, 256, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q2, k2, v2 = ops.qgkv_norm_rope(c["packed"], c["qw"], c["kw"], c["cos"], c["sin"], cache_key=kc,
                                    cache_value=vc, cache_start=torch.tensor(3), **kw)
    assert torch.equal(q2, c["q"])
    assert torch.equal(k2[:, :, 3:8], c["k"]) and torch.equal(v2[:, :, 3:8], c["v"])
    assert not k2[:, :, :3].any() and not v2[:, :, 8:].any()
    assert_bf16_close(ops.attention_gate_mul(c["attn_out"], c["packed"], 256), c["gated"])


def test_lm_head_golden_and_tie():
    c = GOLDEN["lm_head"]
    assert torch.equal(ops.lm_head_argmax(c["h"], c["w"]), c["out"])
    c = GOLDEN["lm_head_tie"]
    assert int(ops.lm_head_argmax(c["h"], c["w"])) == 0


@pytest.mark.parametrize("n", [1, 17])
def test_conv_golden(n):
    c = GOLDEN[f"conv_{n}"]
    st = c["state0"].clone()
    out = ops.causal_conv1d(c["x"], c["w"], st)
    assert_bf16_close(out, c["out"])
    assert torch.equal(st, c["state"])
    st = c["state0"].clone()
    out = ops.causal_conv1d(c["px"], c["w"], st)
    assert_bf16_close(out, c["pout"])
    assert torch.equal(st, c["pstate"])


def test_delta_recurrent_golden():
    c = GOLDEN["delta"]
    st = c["state0"].clone()
    out = ops.delta_recurrent(c["qkv"], c["packed"], c["a_log"], c["dt_bias"], st)
    # reference_delta divides q by sqrt(D); the kernels multiply by 1/sqrt(D): FP32-level.
    assert_bf16_close(out, c["out"], max_ulp=1, max_frac=0.01)
    assert torch.allclose(st, c["state"], rtol=1e-5, atol=1e-6)


def test_chunk_rule_matches_hf():
    c = GOLDEN["chunk_rule"]
    q, k = c["q"], c["k"]
    qh = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) * (1 / 128 ** 0.5)
    kh = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    st = c["state0"].clone()
    out = ops.chunk_gated_delta_rule(qh, kh, c["v"], c["g"], c["beta"], st)
    assert torch.allclose(out, c["out_chunk"], rtol=1e-4, atol=1e-4)
    assert torch.allclose(st, c["state_chunk"], rtol=1e-4, atol=1e-4)
    # and the chunked form agrees with the sequential recurrence
    assert torch.allclose(out, c["out_rec"], rtol=1e-3, atol=1e-3)


def test_a8w8_weight_quant_golden():
    c = GOLDEN["a8w8_weight"]
    q, s = a8w8.quantize_weight(c["w"])
    assert torch.equal(q, c["q"])
    assert torch.equal(s, c["scale"])
    assert float(s[5]) == 1.0 and not q[5].any()


def test_a8w8_linear_is_exact_integer_math():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(3, 512, generator=g).bfloat16()
    w = (torch.randn(64, 512, generator=g) * 0.02).bfloat16()
    qw, sw = a8w8.quantize_weight(w)
    qx, sx = a8w8.quantize_tokens(x)
    acc = a8w8.int8_matmul_exact(qx, qw)
    ref = (qx.long()[:, None, :] * qw.long()[None]).sum(-1)
    assert torch.equal(acc.long(), ref)
    y = a8w8.a8w8_linear(x, qw, sw)
    assert torch.equal(y, ((acc.float() * sx) * sw.T).bfloat16())
    rel = (y.float() - F.linear(x, w).float()).norm() / F.linear(x, w).float().norm()
    assert rel < 0.02


def test_activation_quantiser_follows_vllm_semantics():
    """Activation codes are x * (127/amax) rounded half to even (vllm scaled_int8_quant), not
    x / (amax/127): with amax = 1.125 the rounded reciprocal puts x = 0.5625 exactly on 63.5 (even
    code 64), while dividing by the rounded scale lands just below (63); with amax = 1.1875 it is
    the other way round."""
    x = torch.zeros(3, 16, dtype=torch.bfloat16)
    x[0, 0], x[0, 1], x[0, 2] = 1.125, 0.5625, -0.5625
    x[1, 0], x[1, 1] = 1.1875, 0.59375
    q, s = a8w8.quantize_tokens(x)
    assert q[0, :3].tolist() == [127, 64, -64] and q[1, :2].tolist() == [127, 63]
    assert float(s[0]) == (torch.tensor(1.125) / 127.0).item()
    assert q[2].abs().sum() == 0 and float(s[2]) == 0.0  # all-zero row: zero codes, zero scale
    qw, sw = a8w8.quantize_rows(x)
    assert qw[0, :3].tolist() == [127, 63, -63] and qw[1, :2].tolist() == [127, 64]
    assert float(sw[2]) == 1.0  # the weight formula's all-zero row


def test_linear_rounds_once():
    """The oracle's BF16 F.linear agrees with an exact product rounded once (<=1 ulp)."""
    g = torch.Generator().manual_seed(5)
    x = torch.randn(5, 2048, generator=g).bfloat16()
    w = (torch.randn(384, 2048, generator=g) * 0.02).bfloat16()
    exact = (x.double() @ w.double().T).bfloat16()
    assert_bf16_close(ops.linear(x, w), exact, max_ulp=1, max_frac=0.01)


def _tiny():
    c = GOLDEN["tiny_model"]
    dims = Qwen35Dims(**{k: (tuple(v) if k == "mrope_section" else v) for k, v in c["dims"].items()},
                      delta_padding=16)
    return c, dims


def test_tiny_model_oracle_vs_hf_eager():
    """Oracle decoder vs the Transformers eager model (tiny config). Not bit-exact by design:
    eager normalises q/k and computes beta in BF16 and rounds attention scores to BF16, while the
    reference's fused path (restated by the oracle) does these in FP32."""
    c, dims = _tiny()
    dec = OracleDecoder(c["weights"], dims, max_cache_len=64)
    hidden = dec.forward(c["prompt"])
    rel = (hidden.float() - c["hidden"].float()).norm() / c["hidden"].float().norm()
    assert rel < 3e-2, float(rel)
    toks = dec.generate(c["prompt"], steps=7)
    assert toks[0] == int(c["logits"].float().argmax())
    match = sum(int(a == b) for a, b in zip(toks, c["tokens"].tolist()))
    assert match >= 6, (toks, c["tokens"].tolist())


def test_tiny_model_chunked_prefill_matches_sequential():
    c, dims = _tiny()
    seq = OracleDecoder(c["weights"], dims, max_cache_len=128)
    chk = OracleDecoder(c["weights"], dims, max_cache_len=128, chunked_prefill=True)
    prompt = torch.randint(0, dims.vocab, (1, 100), generator=torch.Generator().manual_seed(2))
    a = seq.forward(prompt)
    b = chk.forward(prompt)
    rel = (a.float() - b.float()).norm() / a.float().norm()
    assert rel < 1e-2, float(rel)
    for s1, s2 in zip(seq.rec_state, chk.rec_state):
        assert torch.allclose(s1, s2, rtol=1e-3, atol=1e-4)
