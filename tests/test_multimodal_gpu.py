"""Image + text prompts on the GPU: the vision tower's tokens placed into the prompt and the text
model prefilled with 3-axis M-RoPE positions (q35_decoder_prefill_mm), against the CPU oracle
decoder fed the same image features and positions (Transformers' masked_scatter + get_rope_index,
integration.py:390-504). Also the config-5 request path end to end (MultimodalEngine)."""

import pytest
import torch

from oracle import ops
from oracle.model import OracleDecoder, bf16_ulp
from ppu_b200.config import Qwen35Dims, VisionDims
from ppu_b200.engine import Qwen35Engine
from ppu_b200.multimodal import IMAGE_TOKEN_ID, MultimodalEngine, prompt_layout
from ppu_b200.synthetic import make_image, make_prompt, make_vision_weights, make_weights
from ppu_b200.vision import VisionEngine

from .helpers import rel_err

pytestmark = pytest.mark.gpu

SMALL = Qwen35Dims(layers=4, vocab=8192)
TINY_VIT = VisionDims(depth=2, width=256, heads=4, intermediate=512, out_width=2048, pos_side=16)
LOGIT_NOISE = 0.16


def test_prompt_layout_follows_get_rope_index():
    rows, pos, nxt = prompt_layout(VisionDims(), (448, 448), 300)
    assert rows.tolist() == list(range(196)) and pos.shape == (3, 496) and nxt == 314
    assert pos[0, :196].eq(0).all() and pos[1, :196].max() == 13 and pos[2, :196].max() == 13
    assert pos[1, 14] == 1 and pos[2, 14] == 0  # second merged row starts at token 14
    assert pos[:, 196:].eq(torch.arange(14, 314)).all()


def _mm_case(seed=0):
    w = make_weights(SMALL, seed=31 + seed)
    vw = make_vision_weights(TINY_VIT, seed=32 + seed)
    img = make_image(224, 224, seed=33 + seed)
    text = make_prompt(SMALL, 40, seed=34 + seed)[0]
    return w, vw, img, text


def test_multimodal_prefill_matches_oracle_states_and_mrope():
    w, vw, img, text = _mm_case()
    vis = VisionEngine(vw, TINY_VIT, max_image=(224, 224))
    image_tokens = vis.encode(img.cuda())
    rows, pos, nxt = prompt_layout(TINY_VIT, (224, 224), text.numel())
    n_img = rows.numel()
    ids = torch.cat((torch.full((n_img,), IMAGE_TOKEN_ID % SMALL.vocab, dtype=torch.int64), text))
    eng = Qwen35Engine(w, SMALL, max_len=256, max_prefill=128)
    eng.prefill_multimodal(ids.cuda(), image_tokens, rows.cuda(), pos.cuda(), nxt)
    torch.cuda.synchronize()
    assert int(eng.cache_len) == ids.numel() and int(eng.rope_pos) == nxt
    feats = image_tokens.cpu()
    oracle = OracleDecoder(w, SMALL, max_cache_len=256)
    h = oracle.forward(ids[None], positions=pos[:, None, :], image_embeds=feats, image_rows=rows)
    n = ids.numel()
    assert rel_err(eng.conv_states[0], oracle.conv_state[0]) < 1e-2
    assert rel_err(eng.rec_states[0], oracle.rec_state[0]) < 1e-3
    k_gpu, k_ref = eng.k_caches[0][:, :, :n].cpu(), oracle.k_cache[0][:, :, :n]
    err = rel_err(k_gpu, k_ref)
    # the same cache from text positions 0..n-1 differs in the rotated dims: the axes matter
    wrong = OracleDecoder(w, SMALL, max_cache_len=256)
    wrong.forward(ids[None], image_embeds=feats, image_rows=rows)
    assert err < 2e-2 < rel_err(k_gpu, wrong.k_cache[0][:, :, :n])
    top = int(oracle.next_token(h[:, -1]))
    got = int(eng.token)
    lg = ops.linear(h[:, -1], oracle.embed).float()[0]
    assert got == top or float(lg[got]) >= float(lg[top]) - LOGIT_NOISE
    # decode continues at the text position after the prompt on both sides
    graph = eng.capture(1)
    for step in range(6):
        eng.token.fill_(top)
        graph.replay()
        h = oracle.forward(torch.tensor([[top]]))
        top = int(oracle.next_token(h[:, -1]))
        got = int(eng.token)
        lg = ops.linear(h[:, -1], oracle.embed).float()[0]
        assert got == top or float(lg[got]) >= float(lg[top]) - LOGIT_NOISE, step
    assert int(eng.rope_pos) == nxt + 6 and oracle.rope_delta == nxt - n


def test_multimodal_engine_generate_matches_oracle_teacher_forced():
    """The config-5 request path with a small decoder: host image + text ids -> tokens."""
    w, vw, img, text = _mm_case(seed=1)
    mm = MultimodalEngine(w, vw, SMALL, TINY_VIT, image_hw=(224, 224), max_text=64, max_new_tokens=8)
    tokens, ttft, elapsed = mm.generate(img, text, 8)
    assert len(tokens) == 8 and 0 < ttft < elapsed
    feats = mm._vgraph[2].cpu()
    rows, pos, nxt = prompt_layout(TINY_VIT, (224, 224), text.numel())
    ids = torch.cat((torch.full((rows.numel(),), IMAGE_TOKEN_ID % SMALL.vocab, dtype=torch.int64), text))
    oracle = OracleDecoder(w, SMALL, max_cache_len=256)
    h = oracle.forward(ids[None], positions=pos[:, None, :], image_embeds=feats, image_rows=rows)[:, -1]
    for step, tok in enumerate(tokens):
        lg = ops.linear(h, oracle.embed).float()[0]
        top = int(lg.argmax())
        assert tok == top or float(lg[tok]) >= float(lg[top]) - max(LOGIT_NOISE, bf16_ulp(float(lg[top]))), step
        h = oracle.forward(torch.tensor([[tok]]))[:, -1]


def test_multimodal_group_prefill_matches_per_request_prefill():
    """Config 5 with a batched text engine: the group's images through one ViT encode and its
    prompts through one prefill (q35_decoder_prefill_batch with per-request image rows and M-RoPE
    positions) against each request encoded and prefilled alone."""
    B = 3
    w = make_weights(SMALL, seed=81)
    vw = make_vision_weights(TINY_VIT, seed=82)
    imgs = torch.stack([make_image(224, 224, seed=83 + b) for b in range(B)]).cuda()
    texts = torch.stack([make_prompt(SMALL, 40, seed=90 + b)[0] for b in range(B)]).cuda()
    n_img = TINY_VIT.merged_tokens(224, 224)
    vis = VisionEngine(vw, TINY_VIT, max_image=(224, 224), max_patches=B * 4 * n_img)
    eng = Qwen35Engine(w, SMALL, max_len=256, max_prefill=B * (n_img + 40), batch=B)
    mm = MultimodalEngine(None, None, SMALL, TINY_VIT, image_hw=(224, 224), max_text=40, max_new_tokens=4,
                          text_engine=eng, vision_engine=vis)
    assert mm.group_prefill and mm.group_images == B
    tokens = mm.encode_images(imgs)
    assert tokens.shape == (B * n_img, SMALL.hidden)
    mm.prefill_group(tokens, texts)
    torch.cuda.synchronize()
    group = {"tok": eng.token.clone(), "rec": [t.clone() for t in eng.rec_states],
             "k": [t[:, :, :n_img + 40].clone() for t in eng.k_caches]}
    rope_group = int(eng.rope_pos)
    for b in range(B):
        mm.prefill(imgs[b], texts[b], b)
    torch.cuda.synchronize()
    assert int(eng.rope_pos) == rope_group == prompt_layout(TINY_VIT, (224, 224), 40)[2]
    for a, b in zip(group["rec"], eng.rec_states):
        assert rel_err(a, b) < 1e-3
    for a, b in zip(group["k"], eng.k_caches):
        assert rel_err(a, b[:, :, :n_img + 40]) < 1e-2
    agree = sum(int(x) == int(y) for x, y in zip(group["tok"], eng.token))
    assert agree >= B - 1
