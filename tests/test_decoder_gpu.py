"""End-to-end decoder parity: the device decoder loop (C ABI) against the CPU oracle decoder.

Random-init weights make this network sensitive to last-bit rounding. Re-running the oracle
itself with exact (float64) GEMMs instead of PyTorch's BF16 GEMM (both round once per output)
moves the DeltaNet states of the second and third layer by 0.2-0.8 % and the KV cache by ~0.8 %
after a 96-token prefill; at the full 2B shape (prefill 1024, 32 teacher-forced decode steps) it
moves logits by up to 0.10-0.15 at every step (p99 ~0.06, several BF16 ulps at |logit| ~ 4) and
flips the oracle's own greedy top-1 at 3 of 33 steps. With A8W8 the int8 activation codes amplify
this: changing only the FP32 summation order of the oracle's RMSNorm moves A8W8 logits by up to
0.27 (p99 ~0.12) and flips its own top-1 at 6 of 33 steps. Exact equality of every greedy token is
therefore not a property of the reference either; the tests check:

* teacher-forced top-1 agreement: fed the same tokens, every GPU greedy choice is the oracle's
  top-1 or within LOGIT_NOISE of the oracle's top logit (the oracle's own measured noise), and
  such near-ties are about as rare as the oracle's own flips;
* internal states (recurrent state, conv state, KV cache) track the oracle's under teacher
  forcing within the oracle's own rounding sensitivity;
* the free-running streams, reported (and identical in the common case).
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
LOGIT_NOISE_A8W8 = 0.28  # >= the same for A8W8 under an RMSNorm summation-order change (0.266)


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


def test_full_2b_config4_greedy_stream_bf16():
    """BASELINE config 4 in BF16: random-init 2B-shape decoder, prefill 1024 uniform-random ids,
    then 32 greedy decode steps with the fused LM-head top-1, batch 1 (CUDA-graph decode). The
    free-running stream must equal the oracle's, token for token."""
    dims = Qwen35Dims()
    w = make_weights(dims, seed=0)
    prompt = make_prompt(dims, 1024, seed=1)
    eng = Qwen35Engine(w, dims, max_len=1152, max_prefill=1024)
    got, ttft, _ = eng.generate(prompt[0], 33, use_graph=True)
    want = OracleDecoder(w, dims, max_cache_len=1152).generate(prompt, steps=32)
    print("oracle", want)
    print("gpu   ", got)
    assert got == want


A8W8_PROJ = ("in", "out", "gate_up", "down")
# Largest fraction of an A8W8 projection's input codes (config 4 prefill, 1024 x k per layer)
# that may differ from the oracle's: propagated last-bit BF16 differences (FP32 summation order
# of norms, scans and softmax) move a code by one step where x * 127/amax sits near a half-way
# point, at a rate that grows with depth.
A8W8_MAX_CODE_FLIPS = 0.02


def test_full_2b_config4_a8w8_code_flips_and_stream():
    """BASELINE config 4 with A8W8. Per layer and projection, the per-token int8 codes and scales
    of the GPU prefill are compared with the oracle's (vllm scaled_int8_quant semantics on both
    sides): the code-flip rate is reported and bounded, the first layer's codes are compared
    exactly, and the 33-token stream is checked under teacher forcing against the oracle's top-1."""
    dims = Qwen35Dims()
    w = make_weights(dims, seed=0)
    prompt = make_prompt(dims, 1024, seed=1)
    eng = Qwen35Engine(w, dims, a8w8=True, max_len=1152, max_prefill=1024)
    gpu_codes = eng.prefill_probe(prompt[0].cuda())
    oracle = OracleDecoder(w, dims, a8w8=True, max_cache_len=1152)
    oracle.probe = []
    oracle.forward(prompt)
    ref_codes = oracle.probe
    assert len(ref_codes) == len(gpu_codes) == 4 * dims.layers
    worst = 0.0
    for i, ((qg, sg), (qo, so)) in enumerate(zip(gpu_codes, ref_codes)):
        flips = float((qg != qo).float().mean())
        off_by = int((qg.int() - qo.int()).abs().max())
        scale_rel = float(((sg - so).abs() / so.abs().clamp_min(1e-30)).max())
        print(f"layer {i // 4:2d} {A8W8_PROJ[i % 4]:>7}: code flips {flips:.5f} (max |dq| {off_by}), "
              f"max scale rel diff {scale_rel:.2e}")
        worst = max(worst, flips)
    # layer 0's in-projection input is RMSNorm(embedding): one norm away from identical inputs
    assert float((gpu_codes[0][0] != ref_codes[0][0]).float().mean()) < 1e-3
    assert worst <= A8W8_MAX_CODE_FLIPS, worst
    got, _, _ = eng.generate(prompt[0], 33, use_graph=True)
    want = OracleDecoder(w, dims, a8w8=True, max_cache_len=1152).generate(prompt, steps=32)
    same = next((i for i, (a, b) in enumerate(zip(got, want)) if a != b), len(got))
    print(f"a8w8: free-running streams identical for {same}/33 tokens")
    print("oracle", want)
    print("gpu   ", got)
    ties = _check_stream(OracleDecoder(w, dims, a8w8=True, max_cache_len=1152), prompt, got, LOGIT_NOISE_A8W8)
    assert ties <= 16
