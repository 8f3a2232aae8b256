"""Batched decoding on the GPU: the batched projection (q35_gemv_batch) against the batch-1
projection per request, the fused decode attention mixer at batch 8 with a 16384-row cache against
the oracle, and the batched decoder (q35_decoder with batch > 1) against the oracle per request
under teacher forcing and against batch-1 engines."""

import pytest
import torch

from oracle import ops as O
from oracle.model import OracleDecoder
from ppu_b200 import kernels as K
from ppu_b200 import lib as L
from ppu_b200.config import Qwen35Dims
from ppu_b200.engine import Qwen35Engine
from ppu_b200.synthetic import make_prompt, make_weights

from .helpers import assert_bf16_close, rel_err

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda"
SMALL = Qwen35Dims(layers=4, vocab=8192)
LOGIT_NOISE = 0.16


def randn(*shape, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(BF16)


def _batch_gemv(w, x, batch, pro, epi, *, nw=None, token=None, embed=None, resid=None, n_out=None):
    n_out = n_out or (w.shape[0] // 2 if epi == L.EPI_SWIGLU else w.shape[0])
    out = None if epi == L.EPI_RESIDUAL else torch.empty(batch, n_out, device=DEV, dtype=BF16)
    d = L.GemvDesc(weight=w.data_ptr(), w_scale=None, input=L.ptr(x), norm_weight=L.ptr(nw), token=L.ptr(token),
                   embed=L.ptr(embed), resid_out=L.ptr(resid), out=L.ptr(out), n_out=n_out, k=w.shape[1],
                   vocab=0 if embed is None else embed.shape[0], prologue=pro, epilogue=epi, int8=0, eps=1e-6)
    L.check(L.load().q35_gemv_batch(L.C.byref(d), batch, L.stream_of()), "q35_gemv_batch")
    return out


@pytest.mark.parametrize("batch", [1, 3, 8])
def test_batched_projections_match_the_batch1_projection(batch):
    H, I = 2048, 6144
    x = randn(batch, H, seed=1).cuda()
    nw = randn(H, seed=2, scale=0.1).cuda()
    w_in = randn(8224, H, seed=3, scale=0.02).cuda()
    w_gu = randn(2 * I, H, seed=4, scale=0.02).cuda()
    w_dn = randn(H, I, seed=5, scale=0.02).cuda()
    w_out = randn(H, H, seed=6, scale=0.02).cuda()
    act = randn(batch, I, seed=7).cuda()
    y_in = _batch_gemv(w_in, x, batch, L.PRO_NORM, L.EPI_STORE, nw=nw)
    y_gu = _batch_gemv(w_gu, x, batch, L.PRO_NORM, L.EPI_SWIGLU, nw=nw)
    r_dn = x.clone()
    _batch_gemv(w_dn, act, batch, L.PRO_PLAIN, L.EPI_RESIDUAL, resid=r_dn)
    r_out = x.clone()
    _batch_gemv(w_out, act[:, :H].contiguous(), batch, L.PRO_PLAIN, L.EPI_RESIDUAL, resid=r_out)
    torch.cuda.synchronize()
    for b in range(batch):
        want_in = K.fused_gemv(w_in, x[b], prologue=L.PRO_NORM, epilogue=L.EPI_STORE, norm_weight=nw)
        want_gu = K.fused_gemv(w_gu, x[b], prologue=L.PRO_NORM, epilogue=L.EPI_SWIGLU, norm_weight=nw)
        rd, ro = x[b].clone(), x[b].clone()
        K.fused_gemv(w_dn, act[b], epilogue=L.EPI_RESIDUAL, resid=rd)
        K.fused_gemv(w_out, act[b, :H].contiguous(), epilogue=L.EPI_RESIDUAL, resid=ro)
        assert_bf16_close(y_in[b].cpu(), want_in.cpu(), max_ulp=1, max_frac=0.02)
        assert rel_err(y_gu[b], want_gu) < 5e-3
        # residual adds: one ulp of the update (summation order) plus one of the sum
        assert_bf16_close(r_dn[b].cpu(), rd.cpu(), max_ulp=2, max_frac=0.02)
        assert_bf16_close(r_out[b].cpu(), ro.cpu(), max_ulp=2, max_frac=0.02)


def test_batched_embedding_prologue():
    H, V, batch = 2048, 4096, 5
    embed = randn(V, H, seed=11).cuda()
    nw = randn(H, seed=12, scale=0.1).cuda()
    w = randn(5120, H, seed=13, scale=0.02).cuda()
    token = torch.tensor([3, 4095, 0, 17, 17], device=DEV, dtype=torch.int64)
    resid = torch.zeros(batch, H, device=DEV, dtype=BF16)
    y = _batch_gemv(w, None, batch, L.PRO_EMBED, L.EPI_STORE, nw=nw, token=token, embed=embed, resid=resid)
    torch.cuda.synchronize()
    assert torch.equal(resid, embed[token])
    for b in range(batch):
        want = O.linear(O.rms_norm(embed[token[b]].cpu(), nw.cpu()), w.cpu())
        assert_bf16_close(y[b].cpu(), want, max_ulp=1, max_frac=0.02)


def test_attn_decode_fused_batch8_16384_rows():
    """The fused decode attention mixer (RoPE + gate + cache write) at batch 8 over 16384 cached
    rows, against the oracle per request (config 2's largest case with the whole mixer)."""
    B, Lmax, p, pos = 8, 16384, 16000, 16100
    packed = randn(B, 5120, seed=21)
    qw, kw = randn(256, seed=22, scale=0.1), randn(256, seed=23, scale=0.1)
    kc = randn(B, 2, Lmax, 256, seed=24)
    vc = randn(B, 2, Lmax, 256, seed=25)
    inv = O.rope_inv_freq(64, 1e7)
    kcd, vcd = kc.cuda(), vc.cuda()
    out = K.attn_decode(packed.cuda(), qw.cuda(), kw.cuda(), inv.cuda(), kcd, vcd, torch.tensor([p], device=DEV),
                        torch.tensor([pos], device=DEV), q_heads=8, kv_heads=2, rotary_dim=64)
    torch.cuda.synchronize()
    cos, sin = O.rope_cos_sin(torch.full((B, 1), pos), inv)
    kco, vco = kc.clone(), vc.clone()
    q, _, _ = O.qgkv_norm_rope(packed[:, None], qw, kw, cos, sin, q_heads=8, kv_heads=2, dim=256, rotary_dim=64,
                               cache_key=kco, cache_value=vco, cache_start=p)
    att = O.gqa_decode_attention(q, kco, vco, p + 1, 0.0625)
    want = O.attention_gate_mul(att, packed[:, None], 256)[:, 0]
    assert rel_err(out, want) < 1e-2
    assert torch.equal(vcd[:, :, p].cpu(), vco[:, :, p])


def test_batched_decoder_matches_oracle_per_request():
    B, n, steps = 4, 48, 10
    w = make_weights(SMALL, seed=41)
    prompts = [make_prompt(SMALL, n, seed=50 + b)[0] for b in range(B)]
    eng = Qwen35Engine(w, SMALL, max_len=256, max_prefill=64, batch=B)
    assert eng.kernels_per_step == 5 * SMALL.layers + 2 and not eng.has_persistent
    tokens, ttft, elapsed = eng.generate_batch(prompts, steps)
    assert len(tokens) == B and all(len(t) == steps for t in tokens) and 0 < ttft < elapsed
    assert int(eng.cache_len) == n + steps - 1
    for b in range(B):
        ref = OracleDecoder(w, SMALL, max_cache_len=256).teacher_forced_top1(prompts[b][None], tokens[b])
        for step, (tok, (top, top_val, tok_val)) in enumerate(zip(tokens[b], ref)):
            assert tok == top or tok_val >= top_val - LOGIT_NOISE, (b, step, tok, top)
    # the same requests one at a time through a batch-1 engine: states agree up to summation order
    single = Qwen35Engine(w, SMALL, max_len=256, max_prefill=64)
    for b in (0, B - 1):
        alone, _, _ = single.generate(prompts[b], steps)
        agree = next((i for i, (x, y) in enumerate(zip(alone, tokens[b])) if x != y), steps)
        assert agree >= 1


def test_batched_prefill_matches_per_slot_prefill():
    """q35_decoder_prefill_batch (all requests' rows through one set of GEMMs, per-request scans,
    attention and cache writes) against one prefill per slot: first tokens, DeltaNet states and
    KV caches agree up to the GEMMs' row-tile summation order."""
    B, n = 4, 40
    w = make_weights(SMALL, seed=61)
    prompts = torch.stack([make_prompt(SMALL, n, seed=70 + b)[0] for b in range(B)])
    one = Qwen35Engine(w, SMALL, max_len=128, max_prefill=B * n, batch=B)
    for b in range(B):
        one.prefill(prompts[b].cuda(), b)
    torch.cuda.synchronize()
    ref = {"tok": one.token.clone(), "conv": [t.clone() for t in one.conv_states],
           "rec": [t.clone() for t in one.rec_states], "k": [t[:, :, :n].clone() for t in one.k_caches]}
    one.prefill_batch(prompts.cuda())
    torch.cuda.synchronize()
    assert int(one.cache_len) == n and int(one.rope_pos) == n
    for a, b in zip(one.rec_states, ref["rec"]):
        assert rel_err(a, b) < 1e-3
    for a, b in zip(one.conv_states, ref["conv"]):
        assert rel_err(a, b) < 1e-2
    for a, b in zip(one.k_caches, ref["k"]):
        assert rel_err(a[:, :, :n], b) < 1e-2
    # first tokens: equal, or within the logit noise of the oracle's top-1 for that request
    for b in range(B):
        got, want = int(one.token[b]), int(ref["tok"][b])
        if got != want:
            (top, top_val, tok_val), = OracleDecoder(w, SMALL, max_cache_len=128).teacher_forced_top1(
                prompts[b][None], [got])
            assert tok_val >= top_val - LOGIT_NOISE, (b, got, want, top)


def test_batched_prefill_rejects_too_many_rows():
    w = make_weights(SMALL, seed=62)
    eng = Qwen35Engine(w, SMALL, max_len=128, max_prefill=64, batch=4)
    with pytest.raises(ValueError, match="max_prefill"):
        eng.prefill_batch(torch.zeros(4, 20, dtype=torch.int64, device=DEV))
    with pytest.raises(ValueError, match="slots"):
        eng.prefill_batch(torch.zeros(2, 20, dtype=torch.int64, device=DEV), slot=3)
