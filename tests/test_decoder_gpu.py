"""End-to-end decoder parity: the device decoder loop (C ABI) against the CPU oracle decoder.

Random-init weights make this network amplify last-bit rounding differences with depth. Measured
at config 4 (2B shape, 1024-token prefill): the fraction of A8W8 input codes that differ between
two correct implementations grows ~2-4x per layer until it saturates near 50-85 %, both between
this GPU path and the oracle and between the reference's own two DeltaNet prefill algorithms
(Triton's sequential scan, kernels.py:768-851, and Transformers' chunk rule). Greedy streams of
two correct implementations therefore part after a few tokens: in BF16 the two reference
algorithms already differ at the second token, in A8W8 at the first. The tests check:

* teacher-forced top-1 agreement: fed the same tokens, every GPU greedy choice is the oracle's
  top-1 or within LOGIT_NOISE of the oracle's top logit (the oracle's own measured noise), and
  such near-ties are about as rare as the oracle's own flips;
* internal states (recurrent state, conv state, KV cache) track the oracle's under teacher
  forcing within the oracle's own rounding sensitivity;
* at config 4, the free-running BF16 stream agrees with the eager oracle at least as long as the
  two reference algorithms agree with each other, and the A8W8 code-flip profile per layer stays
  within the reference's own algorithm-to-algorithm profile.
"""

import pytest
import torch

from oracle import ops
from oracle.model import OracleDecoder, bf16_ulp
from ppu_b200.config import Qwen35Dims
from ppu_b200 import lib as L
from ppu_b200.engine import Qwen35Engine
from ppu_b200.synthetic import make_prompt, make_weights

from .helpers import rel_err

pytestmark = pytest.mark.gpu

SMALL = Qwen35Dims(layers=4, vocab=8192)
LOGIT_NOISE = 0.16  # >= the largest |logit change| of the oracle under a GEMM-order change (0.154)
# A8W8: the largest teacher-forced gaps of the oracle against itself (tests/calibrate_logit_noise.py
# and the RMSNorm order change) are 0.266 (RMSNorm summation order), 0.094 (attention as two
# merged key halves) and 0.109 (the reference's two DeltaNet prefill algorithms); the GPU path
# differs from the oracle by the first two at once, so the bound is their sum
LOGIT_NOISE_A8W8 = 0.37


def _near_top(tok, top, top_val, tok_val, noise=LOGIT_NOISE) -> bool:
    return tok == top or tok_val >= top_val - noise


def _check_stream(oracle: OracleDecoder, prompt, gpu_tokens, noise=LOGIT_NOISE):
    """Teacher-force the oracle with the GPU tokens; returns the number of steps where the GPU
    picked a near-tie instead of the oracle's top-1 (asserting every step is within `noise`)."""
    ref = oracle.teacher_forced_top1(prompt, gpu_tokens)
    ties = 0
    for step, (tok, (top, top_val, tok_val)) in enumerate(zip(gpu_tokens, ref)):
        assert _near_top(tok, top, top_val, tok_val, noise), (step, tok, top, top_val, tok_val)
        if tok != top:
            ties += 1
            print(f"step {step}: gpu {tok} vs oracle top-1 {top}, oracle logit gap {top_val - tok_val:.4f}")
    return ties


@pytest.mark.parametrize("a8w8,persistent", [(False, False), (False, True), (True, False)],
                         ids=["bf16-per-op", "bf16-persistent", "a8w8-per-op"])
def test_small_decoder_teacher_forced(a8w8, persistent):
    # A8W8 re-quantises every activation: a last-bit input difference can move an int8 code by
    # one step, so its states drift about twice as far as BF16's.
    """Prefill 96 tokens, then 16 decode steps fed with the oracle's tokens; after every step the
    GPU's greedy choice and its DeltaNet / conv / KV states are compared with the oracle's. Runs
    the per-op decode step and the persistent one-kernel step."""
    dims = SMALL
    w = make_weights(dims, seed=1)
    prompt = make_prompt(dims, 96, seed=2)
    oracle = OracleDecoder(w, dims, a8w8=a8w8, max_cache_len=256)
    eng = Qwen35Engine(w, dims, a8w8=a8w8, max_len=256, max_prefill=96, persistent=persistent)
    h = oracle.forward(prompt)
    eng.prefill(prompt[0].cuda())
    graph = eng.capture(1)
    mismatches = 0
    for step in range(17):
        top = int(oracle.next_token(h[:, -1]))
        got = int(eng.token)
        lg = ops.linear(h[:, -1], oracle.embed).float()[0]
        noise = LOGIT_NOISE_A8W8 if a8w8 else LOGIT_NOISE
        assert _near_top(got, top, float(lg[top]), float(lg[got]), noise), (step, got, top)
        mismatches += got != top
        tol = 1e-1 if a8w8 else 5e-2
        for s_gpu, s_ref in zip(eng.rec_states, oracle.rec_state):
            assert rel_err(s_gpu, s_ref) < tol, step
        for c_gpu, c_ref in zip(eng.conv_states, oracle.conv_state):
            assert rel_err(c_gpu, c_ref) < tol, step
        n = oracle.length
        for k_gpu, k_ref in zip(eng.k_caches, oracle.k_cache):
            assert rel_err(k_gpu[:, :, :n], k_ref[:, :, :n]) < tol, step
        assert int(eng.cache_len) == n
        if step == 16:
            break
        eng.token.fill_(top)  # teacher forcing: both sides consume the oracle's token
        graph.replay()
        h = oracle.forward(torch.tensor([[top]]))
    torch.cuda.synchronize()
    assert mismatches <= 2
    assert L.load().q35_decoder_persistent_error() == 0


def test_persistent_step_matches_per_op_step():
    """From the same state, one persistent step and one per-op step give the same recurrent /
    conv / KV state up to FP32 summation order, and the same token unless the two candidates are
    a near-tie of the oracle's logits (teacher-forced on the persistent stream); 8 steps."""
    dims = SMALL
    w = make_weights(dims, seed=5)
    prompt = make_prompt(dims, 200, seed=6)
    eng = Qwen35Engine(w, dims, max_len=320, max_prefill=256, persistent=True)
    eng.prefill(prompt[0].cuda())
    consumed, pk_tokens, op_tokens = [int(eng.token)], [], []
    for step in range(8):
        snap = eng.snapshot()
        eng.persistent = False
        eng.decode_step()
        ref = eng.snapshot()
        eng.restore(snap)
        eng.persistent = True
        eng.decode_step()
        got = eng.snapshot()
        torch.cuda.synchronize()
        assert L.load().q35_decoder_persistent_error() == 0
        pk_tokens.append(int(got["token"]))
        op_tokens.append(int(ref["token"]))
        consumed.append(pk_tokens[-1])
        assert int(got["cache_len"]) == int(ref["cache_len"]) == 200 + step + 1
        assert int(got["rope_pos"]) == int(ref["rope_pos"])
        # one step from identical states: only FP32 summation order differs, and its last-bit
        # BF16 flips compound through the layers (the oracle moves 0.2-0.8 % against itself)
        for a, b in zip(got["rec"], ref["rec"]):
            assert rel_err(a, b) < 1e-2, step
        for a, b in zip(got["conv"], ref["conv"]):
            assert rel_err(a, b) < 1e-2, step
        n = int(ref["cache_len"])
        for a, b in zip(got["k"] + got["v"], ref["k"] + ref["v"]):
            assert rel_err(a[:, :, :n], b[:, :, :n]) < 1e-2, step
    mismatched = [i for i, (a, b) in enumerate(zip(pk_tokens, op_tokens)) if a != b]
    assert len(mismatched) <= 2, (pk_tokens, op_tokens)
    if mismatched:
        oracle = OracleDecoder(w, dims, max_cache_len=320)
        oracle.forward(prompt)
        for step in range(max(mismatched) + 1):
            h = oracle.forward(torch.tensor([[consumed[step]]]))[:, -1]
            if step in mismatched:
                lg = ops.linear(h, oracle.embed).float()[0]
                top = float(lg.max())
                for tok in (pk_tokens[step], op_tokens[step]):
                    assert float(lg[tok]) >= top - LOGIT_NOISE, (step, tok, float(lg[tok]), top)


def test_prefill_state_matches_oracle():
    dims = SMALL
    w = make_weights(dims, seed=3)
    prompt = make_prompt(dims, 300, seed=4)
    oracle = OracleDecoder(w, dims, max_cache_len=512)
    hidden = oracle.forward(prompt)
    tok_ref = int(oracle.next_token(hidden[:, -1]))
    eng = Qwen35Engine(w, dims, max_len=512, max_prefill=512)
    eng.prefill(prompt[0].cuda())
    torch.cuda.synchronize()
    # layer 0 sees the embedding through one RMSNorm: its conv state (raw projection outputs) and
    # recurrent state match closely; deeper layers carry propagated rounding.
    assert rel_err(eng.conv_states[0], oracle.conv_state[0]) < 1e-2
    assert rel_err(eng.rec_states[0], oracle.rec_state[0]) < 1e-3
    for s_gpu, s_ref in zip(eng.rec_states, oracle.rec_state):
        assert rel_err(s_gpu, s_ref) < 1e-1
    for v_gpu, v_ref in zip(eng.v_caches, oracle.v_cache):
        assert rel_err(v_gpu[:, :, :300], v_ref[:, :, :300]) < 1e-1
    assert int(eng.cache_len) == 300 and int(eng.rope_pos) == 300
    ties = _check_stream(OracleDecoder(w, dims, max_cache_len=512), prompt, [int(eng.token)])
    assert ties == 0 or int(eng.token) != tok_ref


def _prefix(a, b) -> int:
    return next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), min(len(a), len(b)))


def _oracle_stream(oracle: OracleDecoder, hidden_last: torch.Tensor, steps: int) -> list[int]:
    """Greedy continuation of an oracle whose prefill has run (``hidden_last`` its last state)."""
    tokens, h = [], hidden_last
    for step in range(steps + 1):
        tok = oracle.next_token(h)
        tokens.append(int(tok[0, 0]))
        if step < steps:
            h = oracle.forward(tok)[:, -1]
    return tokens


# The full-model oracle runs the DeltaNet prefill with Transformers' chunk rule
# (torch_chunk_gated_delta_rule, the reference's eager path); the reference's Triton path scans
# sequentially (kernels.py:768-851), and the two reference algorithms are compared with each other
# as the measure of how far two correct implementations of this random-init network drift apart.


def test_full_2b_config4_greedy_stream_bf16():
    """BASELINE config 4 in BF16: random-init 2B-shape decoder, prefill 1024 uniform-random ids,
    then 32 greedy decode steps with the fused LM-head top-1, batch 1 (CUDA-graph decode).

    Random-init weights make the network amplify last-bit differences layer by layer (see the
    A8W8 code-flip profile below), so two correct implementations agree on the greedy stream only
    for a while: the reference's two DeltaNet prefill algorithms (sequential scan, chunk rule)
    already part after one token. Asserted: the GPU stream equals the eager oracle's (chunk rule)
    for at least as many tokens as the two reference algorithms agree with each other, and at
    least its first token; and, teacher-forced, every GPU choice is the oracle's top-1 or within
    the oracle's own measured noise of it."""
    dims = Qwen35Dims()
    w = make_weights(dims, seed=0)
    prompt = make_prompt(dims, 1024, seed=1)
    eng = Qwen35Engine(w, dims, max_len=1152, max_prefill=1024)
    got, ttft, _ = eng.generate(prompt[0], 33, use_graph=True)
    chunk = OracleDecoder(w, dims, max_cache_len=1152, chunked_prefill=True)
    want = _oracle_stream(chunk, chunk.forward(prompt)[:, -1], 32)
    seq = OracleDecoder(w, dims, max_cache_len=1152)
    seq_stream = _oracle_stream(seq, seq.forward(prompt)[:, -1], 8)
    agree, ref_agree = _prefix(got, want), _prefix(seq_stream, want)
    print(f"bf16: GPU vs eager oracle identical for {agree}/33 tokens; the reference's sequential scan vs its "
          f"chunk rule for {ref_agree}")
    print("oracle (chunk rule)", want)
    print("oracle (sequential)", seq_stream)
    print("gpu                ", got)
    assert agree >= max(1, ref_agree)
    ties = _check_stream(OracleDecoder(w, dims, max_cache_len=1152, chunked_prefill=True), prompt, got)
    assert ties <= 6


A8W8_PROJ = ("in", "out", "gate_up", "down")


def test_full_2b_config4_a8w8_code_flips_and_stream():
    """BASELINE config 4 with A8W8. Per layer and projection, the per-token int8 codes of the GPU
    prefill (vllm scaled_int8_quant semantics, 1024 x k per projection) are compared with the eager
    oracle's, and with the same profile between the reference's two DeltaNet prefill algorithms.

    Measured cause of the divergence: no systematic difference. Layer 0's in-projection codes are
    identical; the first flips come from the FP32 summation order of the RMSNorm before gate/up
    (0.3 % of codes), and every layer multiplies the fraction by ~2-4 until it saturates, exactly as
    between the two reference algorithms. Asserted per (layer, projection): GPU-vs-oracle flips
    <= 3 x (sequential-vs-chunk flips) + 1 %, plus identical layer-0 in-projection codes and the
    teacher-forced near-tie bound on the 33-token stream."""
    dims = Qwen35Dims()
    w = make_weights(dims, seed=0)
    prompt = make_prompt(dims, 1024, seed=1)
    eng = Qwen35Engine(w, dims, a8w8=True, max_len=1152, max_prefill=1024)
    gpu_codes = eng.prefill_probe(prompt[0].cuda())
    chunk = OracleDecoder(w, dims, a8w8=True, max_cache_len=1152, chunked_prefill=True)
    chunk.probe = []
    h = chunk.forward(prompt)[:, -1]
    ref_codes, chunk.probe = chunk.probe, None
    want = _oracle_stream(chunk, h, 32)
    seq = OracleDecoder(w, dims, a8w8=True, max_cache_len=1152)
    seq.probe = []
    seq.forward(prompt)
    self_codes = seq.probe
    assert len(ref_codes) == len(gpu_codes) == len(self_codes) == 4 * dims.layers
    for i, ((qg, sg), (qo, so), (qs, _)) in enumerate(zip(gpu_codes, ref_codes, self_codes)):
        flips = float((qg != qo).float().mean())
        self_flips = float((qs != qo).float().mean())
        scale_rel = float(((sg - so).abs() / so.abs().clamp_min(1e-30)).max())
        print(f"layer {i // 4:2d} {A8W8_PROJ[i % 4]:>7}: code flips GPU vs oracle {flips:.5f}, sequential vs "
              f"chunk rule {self_flips:.5f}; max scale rel diff {scale_rel:.2e}")
        assert flips <= 3 * self_flips + 0.01, (i, flips, self_flips)
    assert float((gpu_codes[0][0] != ref_codes[0][0]).float().mean()) < 1e-5
    got, _, _ = eng.generate(prompt[0], 33, use_graph=True)
    print(f"a8w8: free-running streams identical for {_prefix(got, want)}/33 tokens")
    print("oracle", want)
    print("gpu   ", got)
    ties = _check_stream(OracleDecoder(w, dims, a8w8=True, max_cache_len=1152, chunked_prefill=True), prompt, got,
                         LOGIT_NOISE_A8W8)
    assert ties <= 16
