"""Calibration of the teacher-forced near-tie bounds in test_decoder_gpu.py (CPU only, minutes).

The bound is the oracle's own logit spread between two correct forms of the same computation:
one oracle's greedy stream is teacher-forced into the other, and the largest gap between the
second's top logit and the logit of the token the first chose is printed, at BASELINE config 4
(2B shape, 1024-token prompt, 33 tokens), for two pairs:
* the causal attention as two key halves merged by their running maxima and sums (the
  FlashAttention form the GPU kernels use) instead of one softmax;
* the reference's two DeltaNet prefill algorithms (Triton's sequential scan and Transformers'
  chunk rule), whose A8W8 input codes already part in the first layers.

    python -m tests.calibrate_logit_noise
"""

from __future__ import annotations

import torch

from oracle import ops
from oracle.model import OracleDecoder
from ppu_b200.config import Qwen35Dims
from ppu_b200.synthetic import make_prompt, make_weights


def _split_attention(q, k, v, scale: float, q_offset: int = 0):
    """``ops.causal_attention`` with the keys in two halves merged by running max / sum."""
    b, heads, length, dim = q.shape
    group = heads // k.shape[1]
    kk = k.float().repeat_interleave(group, dim=1)
    vv = v.float().repeat_interleave(group, dim=1)
    s_len = kk.shape[2]
    i = torch.arange(length)[:, None] + q_offset
    parts = []
    for lo, hi in ((0, s_len // 2), (s_len // 2, s_len)):
        if hi <= lo:
            continue
        sc = (q.float() * scale) @ kk[:, :, lo:hi].transpose(-1, -2)
        j = torch.arange(lo, hi)[None, :]
        sc = sc.masked_fill(j > i, float("-inf"))
        m = sc.amax(-1, keepdim=True)
        e = torch.where(torch.isinf(m), torch.zeros_like(sc), torch.exp(sc - m))
        parts.append((m, e.sum(-1, keepdim=True), e @ vv[:, :, lo:hi]))
    m = torch.stack([p[0] for p in parts]).amax(0)
    num = sum(torch.where(torch.isinf(p[0]), torch.zeros_like(p[2]), p[2] * torch.exp(p[0] - m)) for p in parts)
    den = sum(torch.where(torch.isinf(p[0]), torch.zeros_like(p[1]), p[1] * torch.exp(p[0] - m)) for p in parts)
    out = (num / den).transpose(1, 2).reshape(b, length, heads * dim)
    return ops._bf(out)


def spread(a8w8: bool, pair: str, steps: int = 32) -> float:
    dims = Qwen35Dims()
    w = make_weights(dims, seed=0)
    prompt = make_prompt(dims, 1024, seed=1)
    base = OracleDecoder(w, dims, a8w8=a8w8, max_cache_len=1152, chunked_prefill=pair == "attention")
    stream = [int(t) for t in base.generate(prompt, steps)]
    original = ops.causal_attention
    if pair == "attention":
        ops.causal_attention = _split_attention
    try:
        alt = OracleDecoder(w, dims, a8w8=a8w8, max_cache_len=1152, chunked_prefill=True)
        ref = alt.teacher_forced_top1(prompt, stream)
    finally:
        ops.causal_attention = original
    gaps = [top_val - tok_val for (_, top_val, tok_val) in ref]
    return max(gaps)


if __name__ == "__main__":
    for a8 in (False, True):
        for pair in ("attention", "deltanet"):
            print(f"{'A8W8' if a8 else 'BF16'} {pair}: largest teacher-forced logit gap {spread(a8, pair):.4f}",
                  flush=True)
