#!/usr/bin/env python3
"""Benchmark of the Qwen3.5-2B-shape fused decode path.

Workload per step (one request): prefill 1024 uniform-random token ids, then 32 greedy decode
steps with the fused LM-head top-1, batch 1, random-init 2B-shape weights (N(0, 0.02)), all
resident in HBM before the timed region. Metric: decode tokens/s (whole job, all ranks), timed
on the device with CUDA events; TTFT is reported beside it. One process per GPU; each rank is
an independent model replica on its own seeded requests (request-level data parallelism, no
collectives on the data path: "scaling": "weak").

The same JSON line also carries, measured in the same process:
* ``a8w8``: the A8W8 engine (int8 M/F/L projections, BF16 LM head) on the same workload;
* ``prefill_roofline``: the prefill's dense FLOPs over TTFT against the sustained bf16 peak;
* ``lm_shard`` (N > 1): lock-step decode with the LM head vocab-sharded over the ranks (NCCL
  all-gather of the final residuals + int64 MAX all-reduce of the top-1 keys per token), with the
  per-token collective time measured alone;
* ``cpu_baseline`` (rank 0, N = 1): the reference's CPU path, Transformers eager
  ``Qwen3_5ForCausalLM`` (attn_implementation="eager") on the same seeded weights, config 4.

``--impl reference`` times that Transformers eager CPU path alone on the host cores (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from ppu_b200.config import Qwen35Dims  # noqa: E402
from ppu_b200.synthetic import make_prompt, make_weights  # noqa: E402

METRIC = "bs1 decode tok/s (Qwen3.5-2B-shape text decoder, greedy, fused LM-head top-1)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--prompt-len", type=int, default=1024)
    ap.add_argument("--new-tokens", type=int, default=32)
    ap.add_argument("--a8w8", action="store_true", help="headline on the A8W8 engine instead of bf16")
    ap.add_argument("--no-a8w8-leg", action="store_true", help="skip the A8W8 sub-measurement")
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--gemv", default="registers", choices=["registers", "bulk"],
                    help="decode GEMV weight streaming: shared-memory bulk copies or register loads")
    ap.add_argument("--gemv-ctas", type=int, default=0, help="decode GEMV grid cap in CTAs per SM (0: all that fit)")
    ap.add_argument("--prefill-delta", default="chunked", choices=["chunked", "sequential"])
    ap.add_argument("--decode", default="kernels", choices=["kernels", "persistent"],
                    help="decode step: one persistent cooperative kernel (bf16) or the per-op kernels")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-tokens", type=int, default=16, help="decode tokens per CPU sample (reference path)")
    ap.add_argument("--lm-shard", action="store_true",
                    help="N > 1: headline on the lock-step vocab-sharded decode instead of full replicas")
    ap.add_argument("--no-lm-shard-leg", action="store_true", help="N > 1: skip the lock-step sub-measurement")
    ap.add_argument("--mm-requests", type=int, default=256, help="config-5 image + text requests (0: skip)")
    ap.add_argument("--mm-new-tokens", type=int, default=16)
    ap.add_argument("--batch", type=int, default=8, help="requests per decode step of the batched legs (1: skip)")
    return ap.parse_args()


def peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, bf16 TFLOP/s sustained, 'measured' | 'fallback')."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


def prefill_flops(dims: Qwen35Dims, length: int) -> int:
    """Dense FLOPs of one prefill of ``length`` tokens: 2 * L * (linear parameters) for every
    projection, causal attention (QK^T and PV over the causal half) and the DeltaNet chunk
    products (chunk 64: K K^T, Q K^T, the triangular solve and the state products per chunk),
    plus the LM head of the last token."""
    h = dims.hidden
    lin = (dims.n_delta * (dims.delta_rows * h + h * dims.value_dim)
           + dims.n_attn * (dims.qgkv_rows * h + h * dims.attn_width) + dims.layers * 3 * dims.intermediate * h)
    attn = dims.n_attn * 4 * dims.q_heads * dims.head_dim * length * (length + 1) // 2
    c, dk, dv = 64, dims.lin_dk, dims.lin_dv
    chunks = (length + c - 1) // c
    per_chunk = 2 * c * c * dk * 2 + 2 * c * c * c + 2 * c * c * dv * 2 + 2 * c * dk * dv * 3
    delta = dims.n_delta * dims.lin_heads * chunks * per_chunk
    return 2 * length * lin + attn + delta + 2 * dims.vocab * h


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.samples.append([x.strip() for x in out.stdout.strip().split(",")])
            except Exception:
                pass
            self._stop.wait(0.1)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"], "samples": 0}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if len(s) > 5 + i and "Active" in s[5 + i]
                          and "Not" not in s[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------------------------------------
# The reference's CPU path: Transformers eager Qwen3_5ForCausalLM on the host cores.
def hf_eager_model(weights_cpu: dict, dims: Qwen35Dims):
    """Transformers eager ``Qwen3_5ForCausalLM`` (attn_implementation="eager", the torch fallbacks
    of the DeltaNet kernels) holding the seeded weights; built on the meta device and filled in place
    (no random initialisation pass)."""
    from transformers.models.qwen3_5 import modeling_qwen3_5 as hf

    cfg = hf.Qwen3_5TextConfig(
        vocab_size=dims.vocab, hidden_size=dims.hidden, intermediate_size=dims.intermediate,
        num_hidden_layers=dims.layers, num_attention_heads=dims.q_heads, num_key_value_heads=dims.kv_heads,
        head_dim=dims.head_dim, linear_num_key_heads=dims.lin_heads, linear_num_value_heads=dims.lin_heads,
        linear_key_head_dim=dims.lin_dk, linear_value_head_dim=dims.lin_dv, linear_conv_kernel_dim=dims.conv_kernel,
        rms_norm_eps=dims.eps, tie_word_embeddings=True,
        rope_parameters={"rope_type": "default", "rope_theta": dims.rope_theta,
                         "partial_rotary_factor": dims.rotary_dim / dims.head_dim,
                         "mrope_section": list(dims.mrope_section), "mrope_interleaved": True})
    cfg._attn_implementation = "eager"
    # The torch implementations of the DeltaNet pieces (torch_chunk_gated_delta_rule, the torch
    # conv update, Qwen3_5RMSNormGated): with a GPU visible, Transformers would pick the Triton
    # kernels of flash-linear-attention, which cannot run on CPU tensors.
    fast = ("FusedRMSNormGated", "chunk_gated_delta_rule", "fused_recurrent_gated_delta_rule", "causal_conv1d_fn",
            "causal_conv1d_update")
    saved = {name: getattr(hf, name, None) for name in fast + ("is_fast_path_available",)}
    try:
        for name in fast:
            setattr(hf, name, None)
        hf.is_fast_path_available = False
        with torch.device("meta"):
            model = hf.Qwen3_5ForCausalLM(cfg)
    finally:
        for name, value in saved.items():
            setattr(hf, name, value)
    missing, unexpected = model.load_state_dict(weights_cpu, strict=False, assign=True)
    if unexpected or any(not k.startswith("lm_head") for k in missing):
        raise RuntimeError(f"eager model weights: missing {missing}, unexpected {unexpected}")
    model.lm_head.weight = model.model.embed_tokens.weight
    rot = model.model.rotary_emb
    inv, _ = rot.compute_default_rope_parameters(cfg, device="cpu")
    rot.inv_freq = inv
    rot.original_inv_freq = inv.clone()
    return model.eval()


def hf_eager_request(model, prompt: torch.Tensor, n_tokens: int):
    """Prefill + ``n_tokens`` greedy decode tokens through the eager model; returns (TTFT seconds,
    per-decode-token seconds)."""
    from transformers.cache_utils import DynamicCache

    with torch.inference_mode():
        cache = DynamicCache(config=model.config)
        t0 = time.perf_counter()
        out = model(input_ids=prompt, past_key_values=cache, use_cache=True, logits_to_keep=1)
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
        ttft = time.perf_counter() - t0
        per_tok = []
        for _ in range(n_tokens):
            t1 = time.perf_counter()
            out = model(input_ids=tok, past_key_values=cache, use_cache=True, logits_to_keep=1)
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
            per_tok.append(time.perf_counter() - t1)
    return ttft, per_tok


def cpu_reference_sample(dims, weights_cpu, prompt_len: int, n_tokens: int, threads: int, seed: int = 99):
    torch.set_num_threads(threads)
    model = hf_eager_model(weights_cpu, dims)
    ttft, per_tok = hf_eager_request(model, make_prompt(dims, prompt_len, seed=seed), n_tokens)
    return ttft, per_tok


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    dims = Qwen35Dims()
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    weights = make_weights(dims, seed=0)
    model = hf_eager_model(weights, dims)
    del weights
    per_step = max(args.cpu_tokens, 1)  # decode tokens per step: a bounded sample of the 32-token workload
    from transformers.cache_utils import DynamicCache

    per_tok, step_s = [], []
    with torch.inference_mode():
        cache = DynamicCache(config=model.config)
        t0 = time.perf_counter()
        out = model(input_ids=make_prompt(dims, args.prompt_len, seed=1), past_key_values=cache, use_cache=True,
                    logits_to_keep=1)
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
        ttft = time.perf_counter() - t0
        for s in range(args.warmup + args.steps):
            t_step = time.perf_counter()
            for _ in range(per_step):
                t1 = time.perf_counter()
                out = model(input_ids=tok, past_key_values=cache, use_cache=True, logits_to_keep=1)
                tok = out.logits[:, -1].argmax(-1, keepdim=True)
                if s >= args.warmup:
                    per_tok.append(time.perf_counter() - t1)
            if s >= args.warmup:
                step_s.append(time.perf_counter() - t_step)
    med = statistics.median(per_tok)
    value = 1.0 / med
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1000 * statistics.mean(step_s), 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights, "
        "uniform-random token ids)", "impl": "reference",
        "config": {"workload": "config4: prefill 1024 + greedy decode, 2B-shape decoder, batch 1",
                   "model": "Qwen3.5-2B-shape text decoder (random init)", "global_batch": 1,
                   "seq_len": args.prompt_len, "parallelism": "cpu (all host threads, one process)",
                   "decode_tokens_per_step": per_step},
        "ttft_ms": round(1000 * ttft, 1),
        "decode_ms_per_token": {"median": round(1000 * med, 3), "mean": round(1000 * statistics.mean(per_tok), 3),
                                "min": round(1000 * min(per_tok), 3), "max": round(1000 * max(per_tok), 3)},
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads, "kind": "hf-eager",
                         "sample": f"Transformers eager Qwen3_5ForCausalLM (attn_implementation=eager), bf16, "
                                   f"{threads} threads: prefill {args.prompt_len} tokens, then {per_step} greedy "
                                   "decode tokens per step; value = 1 / median per-token time"},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# ---------------------------------------------------------------------------------------------
def time_requests(eng, graph, prompts, warmup: int, steps: int, new_tokens: int, sampler_idx=None):
    """Device-timed requests (prefill + ``new_tokens`` graph replays each); returns (total_ms,
    decode_ms, prefill_ms, clock summary or None) for this rank."""
    from ppu_b200 import replicas as R

    def request(i, ev=None):
        if ev:
            ev[0].record()
        eng.prefill(prompts[i])
        if ev:
            ev[1].record()
        for _ in range(new_tokens):
            graph.replay()
        if ev:
            ev[2].record()

    for i in range(warmup):
        request(i)
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    R.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(sampler_idx) if sampler_idx is not None else None
    if clocks:
        clocks.__enter__()
    try:
        for s in range(steps):
            request(warmup + s, evs[s])
        torch.cuda.synchronize()
        R.barrier()
        torch.cuda.synchronize()
    finally:
        if clocks:
            clocks.__exit__()
    total_ms = evs[0][0].elapsed_time(evs[-1][2])
    decode_ms = sum(e[1].elapsed_time(e[2]) for e in evs)
    prefill_ms = sum(e[0].elapsed_time(e[1]) for e in evs)
    return total_ms, decode_ms, prefill_ms, (clocks.summary() if clocks else None)


def gate_up_roofline(eng, dims, dev, hbm_peak, peak_kind, a8w8: bool):
    """The dominant decode kernel (gate/up GEMV with fused RMSNorm + SwiGLU), CUDA-graph timed over
    the 24 layers' cold weights: achieved GB/s of algorithmic bytes against the copy peak."""
    from ppu_b200 import kernels as K
    from ppu_b200 import lib as L

    gate_up_w = [t["gate_up"] for t in eng.layer_tensors]
    post_ln = [t["post_ln"] for t in eng.layer_tensors]
    gate_up_s = [t.get("gate_up_scale") for t in eng.layer_tensors]
    resid = torch.randn(dims.hidden, device=dev).to(torch.bfloat16)
    n_rep = 3

    def launches():
        for j in range(len(gate_up_w)):
            K.fused_gemv(gate_up_w[j], resid, prologue=L.PRO_NORM, epilogue=L.EPI_SWIGLU, norm_weight=post_ln[j],
                         w_scale=gate_up_s[j])

    launches()
    torch.cuda.synchronize()
    kgraph = torch.cuda.CUDAGraph()  # captured so host launch overhead does not pace the kernels
    with torch.cuda.graph(kgraph):
        for _ in range(n_rep):
            launches()
    kgraph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    kgraph.replay()
    e1.record()
    torch.cuda.synchronize()
    del kgraph
    kern_s = e0.elapsed_time(e1) / 1000.0 / (n_rep * len(gate_up_w))
    w_bytes = gate_up_w[0].numel() * gate_up_w[0].element_size() + (gate_up_w[0].shape[0] * 4 if a8w8 else 0)
    achieved = w_bytes / kern_s / 1e9
    tname = "gemv_swiglu_a8w8_traffic.json" if a8w8 else "gemv_swiglu_traffic.json"
    tfile = ROOT / "profiles" / tname
    traffic = json.loads(tfile.read_text()).get("bytes_per_launch") if tfile.exists() else None
    kname = "gemv_fast<2048,NORM,SWIGLU,int8>" if a8w8 else "gemv_fast<2048,NORM,SWIGLU>"
    return {"kernel": f"{kname} (gate/up + RMSNorm + SwiGLU)", "bound": "hbm", "achieved": round(achieved, 1),
            "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
            "traffic_source": f"stored ncu capture (profiles/{tname}: dram__bytes_read.sum + dram__bytes_write.sum "
                              "per launch), not measured in this run",
            "algorithmic_bytes_per_launch": w_bytes, "avg_launch_us": round(kern_s * 1e6, 3),
            "timing": "CUDA events around a CUDA graph of 72 launches, 24 distinct weight sets",
            "peak_kind": peak_kind}


def vision_engine(dev, max_images=1):
    from ppu_b200.config import VisionDims
    from ppu_b200.synthetic import make_vision_weights
    from ppu_b200.vision import VisionEngine

    vd = VisionDims()
    vw = make_vision_weights(vd, seed=1, device=dev)
    return VisionEngine(vw, vd, max_image=(448, 448), device=dev, max_patches=max_images * 784)


def multimodal_leg(eng, vis, decode_graph, dims, dev, rank, world, args, tf_sust, peak_kind):
    """``args.mm_requests`` seeded image + text requests spread over the ranks
    (request i on rank i mod N): a 448 x 448 image through the 24-layer ViT and the 2x2 merger (196
    tokens), prepended to 300 text tokens, a 496-token multimodal prefill and greedy decode to
    ``args.mm_new_tokens`` tokens. A batched text engine serves its requests in groups of
    ``eng.batch`` (each image encoded and prefilled into its slot, then the group decodes in lock
    step). Device-timed (inputs resident in HBM); the vision tower's FLOPs over its time against the
    sustained bf16 peak; e2e through MultimodalEngine.generate (batch-1 engines)."""
    from ppu_b200 import replicas as R
    from ppu_b200.multimodal import MultimodalEngine

    vd = vis.vd
    n_text, n_new, nb = 300, args.mm_new_tokens, eng.batch
    mm = MultimodalEngine(None, None, dims, vd, image_hw=(448, 448), max_text=n_text, max_new_tokens=n_new,
                          text_engine=eng, vision_engine=vis, decode_graph=decode_graph)
    mine = R.requests_for_rank(args.mm_requests, world, rank)

    def image(i):
        g = torch.Generator(device=dev)
        g.manual_seed(100_000 + i)
        return torch.rand((3, 448, 448), generator=g, device=dev)

    imgs = [image(i) for i in mine]
    texts = [make_prompt(dims, n_text, seed=200_000 + i)[0].to(dev) for i in mine]
    groups = [list(range(j, min(j + nb, len(mine)))) for j in range(0, len(mine), nb)]
    # batched engines: a group's images go through the ViT together and its prompts through one
    # prefill (inputs stacked once, resident like the single images)
    together = mm.group_prefill
    stacked = {g[0]: (torch.stack([imgs[j] for j in g]), torch.stack([texts[j] for j in g])) for g in groups} \
        if together else {}

    def group(js, ev=None):
        if ev:
            ev["start"].record()
        if together:
            pix, ids = stacked[js[0]]
            tokens = mm.encode_images(pix)
            if ev:
                ev["vis"][0].record()
            mm.prefill_group(tokens, ids, 0)
            if ev:
                ev["first"][0].record()
        else:
            for slot, j in enumerate(js):
                tokens = mm.encode_image(imgs[j])
                if ev:
                    ev["vis"][slot].record()
                mm.prefill_prompt(tokens, texts[j], slot)
                if ev:
                    ev["first"][slot].record()
        for _ in range(n_new - 1):
            mm.decode_step()
        if ev:
            ev["end"].record()

    def events(n):
        e = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
        n = 1 if together else n
        return {"start": e(), "end": e(), "vis": [e() for _ in range(n)], "first": [e() for _ in range(n)]}

    for js in groups[:min(2, len(groups))]:
        group(js)
    torch.cuda.synchronize()
    evs = [events(len(js)) for js in groups]
    R.barrier()
    torch.cuda.synchronize()
    for js, ev in zip(groups, evs):
        group(js, ev)
    torch.cuda.synchronize()
    R.barrier()
    total_ms = R.max_over_ranks(evs[0]["start"].elapsed_time(evs[-1]["end"]), dev)
    vis_ms, ttft_ms, dec_ms = [], [], []
    for js, ev in zip(groups, evs):
        prev = ev["start"]
        for v, f in zip(ev["vis"], ev["first"]):
            if together:  # one encode of the group's images: its time per image; the group's TTFT
                vis_ms += [prev.elapsed_time(v) / len(js)] * len(js)
                ttft_ms += [ev["start"].elapsed_time(f)] * len(js)
            else:
                vis_ms.append(prev.elapsed_time(v))
                ttft_ms.append(ev["start"].elapsed_time(f))
            prev = f
        dec_ms.append(ev["first"][-1].elapsed_time(ev["end"]))
    mean = lambda xs: R.max_over_ranks(sum(xs) / len(xs), dev)  # noqa: E731
    v_ms, t_ms, d_ms = mean(vis_ms), mean(ttft_ms), mean(dec_ms)
    vflops = vd.linear_flops(448, 448)
    line = {
        "workload": f"config5: {args.mm_requests} requests over {world} GPU(s): 448x448 image -> ViT (24 layers, "
                    f"width 1024) -> 196 tokens + {n_text} text tokens, {n_new} greedy tokens each",
        "requests_per_s": round(args.mm_requests / (total_ms / 1e3), 2),
        "tok_per_s": round(args.mm_requests * n_new / (total_ms / 1e3), 1),
        "ttft_ms_mean": round(t_ms, 3), "vision_ms_mean": round(v_ms, 3),
        "decode_ms_per_step": round(d_ms / max(n_new - 1, 1), 4), "requests_per_decode_step": nb,
        "prefill": (f"{mm.group_images} images per ViT encode, {nb} prompts per prefill" if together
                    else "one image per ViT encode, one prompt per prefill"),
        "vision_roofline": {"flops": vflops, "achieved_tflops": round(vflops / (v_ms / 1e3) / 1e12, 1),
                            "peak_tflops": tf_sust, "frac": round(vflops / (v_ms / 1e3) / 1e12 / tf_sust, 4),
                            "bound": "tensor", "peak_kind": f"{peak_kind} bf16 sustained"},
        "decode": ("lock-step across ranks, LM head vocab-sharded" if decode_graph is not None
                   else f"per-rank replicas, {nb} request(s) per decode step"),
        "data": "synthetic: seeded random-init ViT N(0,0.02) (LayerNorm 1+N), uniform [0,1) pixels, "
                "uniform-random text ids",
    }
    if nb == 1:
        host_img = torch.rand((3, 448, 448), generator=torch.Generator().manual_seed(300_000 + rank))
        e_tok, e_ttft, e_el = mm.generate(host_img, make_prompt(dims, n_text, seed=310_000 + rank)[0], n_new)
        e_el = R.max_over_ranks(e_el, dev)
        line["e2e"] = {"requests_per_s": round(world / e_el, 2), "ttft_ms": round(1000 * e_ttft, 3),
                       "tokens": len(e_tok), "h2d_bytes_per_request": 3 * 448 * 448 * 4 + n_text * 8,
                       "path": "MultimodalEngine.generate (host image + ids -> H2D, ViT graph, prefill, per-token D2H)"}
    return line


def batched_decode_leg(engB, dims, dev, rank, world, args, hbm_peak, peak_kind):
    """Config 4's requests ``engB.batch`` at a time: each slot prefilled with its own 1024-token
    prompt, then ``new_tokens`` lock-step decode steps (CUDA graph); tokens/s over the decode time."""
    from ppu_b200 import replicas as R

    nb, P, T = engB.batch, args.prompt_len, args.new_tokens
    n_groups, warm = max(1, min(args.steps, 4)), 1
    prompts = [make_prompt(dims, P, seed=400_000 + 1000 * rank + i)[0].to(dev) for i in range(nb)]
    g = engB.capture(1)

    def rnd(ev=None):
        for slot in range(nb):
            engB.prefill(prompts[slot], slot)
        if ev:
            ev[0].record()
        for _ in range(T):
            g.replay()
        if ev:
            ev[1].record()

    for _ in range(warm):
        rnd()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(n_groups)]
    R.barrier()
    for ev in evs:
        rnd(ev)
    torch.cuda.synchronize()
    dec_ms = R.max_over_ranks(sum(e[0].elapsed_time(e[1]) for e in evs), dev)
    value = R.aggregate_rate(n_groups * T * nb, dec_ms / 1000.0, world)
    step_ms = dec_ms / (n_groups * T)
    bytes_step = dims.weight_bytes_per_token() + (nb - 1) * dims.n_delta * 2 * 4 * dims.lin_heads * dims.lin_dk * \
        dims.lin_dv + nb * 2 * dims.n_attn * dims.kv_heads * dims.head_dim * 2 * (P + T // 2)
    return {"value": round(value, 2), "unit": "tok/s", "requests_per_step": nb, "rounds": n_groups,
            "decode_ms_per_step": round(step_ms, 4),
            "step_hbm": {"bytes_per_step": bytes_step, "achieved_gbs": round(bytes_step / step_ms / 1e6, 1),
                         "peak_gbs": hbm_peak, "frac": round(bytes_step / step_ms / 1e6 / hbm_peak, 4),
                         "peak_kind": peak_kind},
            "workload": f"config4 requests {nb} at a time: prefill {P} per slot, {T} lock-step greedy decode steps"}


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    from ppu_b200 import lib as L
    from ppu_b200 import replicas as R
    from ppu_b200.engine import Qwen35Engine, cache_bucket

    rank, world, local = R.dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    R.init("nccl", timeout_s=300, device=dev)  # request replicas: no collective on the data path

    def max_over_ranks(x: float) -> float:
        return R.max_over_ranks(x, dev)

    dims = Qwen35Dims()
    P, T = args.prompt_len, args.new_tokens
    L.call("q35_set_gemv_variant", L.Q35_GEMV_BULK if args.gemv == "bulk" else L.Q35_GEMV_REGISTERS)
    L.call("q35_set_gemv_ctas_per_sm", args.gemv_ctas)
    weights = make_weights(dims, seed=0, device=dev)
    headline_a8w8 = args.a8w8
    eng = Qwen35Engine(weights, dims, a8w8=headline_a8w8, max_len=cache_bucket(P, T), max_prefill=P, device=dev,
                       use_pdl=not args.no_pdl, prefill_chunked=args.prefill_delta == "chunked",
                       persistent=(args.decode == "persistent" and not headline_a8w8))
    engB = None
    if args.batch > 1 and not headline_a8w8:
        # its prefill rows also hold a whole group of config-5 prompts (196 image + 300 text tokens)
        mm_rows = args.batch * (196 + 300) if args.mm_requests > 0 else 0
        engB = Qwen35Engine(weights, dims, max_len=cache_bucket(P, T), max_prefill=max(P, mm_rows), device=dev,
                            batch=args.batch, use_pdl=not args.no_pdl,
                            prefill_chunked=args.prefill_delta == "chunked")
    eng8 = None
    if not headline_a8w8 and not args.no_a8w8_leg:
        eng8 = Qwen35Engine(weights, dims, a8w8=True, max_len=cache_bucket(P, T), max_prefill=P, device=dev,
                            use_pdl=not args.no_pdl, prefill_chunked=args.prefill_delta == "chunked")
    weights_cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        weights_cpu = {k: v.cpu() for k, v in weights.items()}
    del weights
    torch.cuda.empty_cache()

    n_req = args.warmup + args.steps
    prompts = [make_prompt(dims, P, seed=R.request_seed(rank, i))[0].to(dev) for i in range(n_req)]
    sharded = None
    if world > 1 and (args.lm_shard or not args.no_lm_shard_leg):
        from ppu_b200.vocab_shard import ShardedDecode
        sharded = ShardedDecode(eng)
    head = sharded if (args.lm_shard and sharded) else None
    graph = head.capture(1) if head else eng.capture(1)
    torch.cuda.synchronize()
    hbm_peak, tf_burst, tf_sust, peak_kind = peaks()

    # ---- headline: the timed requests
    total_ms, decode_ms, prefill_ms, clocks = time_requests(eng, graph, prompts, args.warmup, args.steps, T, local)
    total_ms, decode_ms, prefill_ms = (max_over_ranks(x) for x in (total_ms, decode_ms, prefill_ms))
    value = R.aggregate_rate(args.steps * T, decode_ms / 1000.0, world)
    kv_bytes = 2 * dims.n_attn * dims.kv_heads * dims.head_dim * 2 * (P + T // 2)
    bytes_tok = dims.weight_bytes_per_token(headline_a8w8) + kv_bytes
    ttft_ms = prefill_ms / args.steps
    flops = prefill_flops(dims, P)
    roofline = gate_up_roofline(eng, dims, dev, hbm_peak, peak_kind, headline_a8w8)

    # ---- end to end through the public generate path (host prompt, per-token host reads)
    e2e_tok, e2e_time, e2e_ttft = 0, 0.0, []
    for i in range(2):
        host_prompt = make_prompt(dims, P, seed=50_000 + R.request_seed(rank, i))[0]
        toks, ttft, elapsed = (head or eng).generate(host_prompt, T + 1)
        e2e_tok += len(toks) - 1
        e2e_time += elapsed - ttft
        e2e_ttft.append(ttft)
    e2e_time = max_over_ranks(e2e_time)
    e2e_value = R.aggregate_rate(e2e_tok, e2e_time, world)

    # ---- A8W8 engine on the same workload (fewer requests)
    a8 = None
    if eng8 is not None:
        n8, w8 = min(args.steps, 10), min(args.warmup, 3)
        g8 = eng8.capture(1)
        t8, d8, p8, _ = time_requests(eng8, g8, prompts, w8, n8, T)
        d8, p8 = max_over_ranks(d8), max_over_ranks(p8)
        v8 = R.aggregate_rate(n8 * T, d8 / 1000.0, world)
        b8 = dims.weight_bytes_per_token(True) + kv_bytes
        toks8, ttft8, el8 = eng8.generate(make_prompt(dims, P, seed=70_000 + rank)[0], T + 1)
        e8 = R.aggregate_rate(len(toks8) - 1, max_over_ranks(el8 - ttft8), world)
        a8 = {"value": round(v8, 2), "unit": "tok/s", "steps": n8, "warmup": w8,
              "ttft_ms": round(p8 / n8, 3), "decode_ms_per_token": round(d8 / n8 / T, 4),
              "step_hbm": {"bytes_per_token": b8, "achieved_gbs": round(b8 * v8 / world / 1e9, 1),
                           "peak_gbs": hbm_peak, "frac": round(b8 * v8 / world / 1e9 / hbm_peak, 4),
                           "peak_kind": peak_kind},
              "roofline": gate_up_roofline(eng8, dims, dev, hbm_peak, peak_kind, True),
              "prefill_roofline": {"flops": flops, "achieved_tflops": round(flops / (p8 / n8 / 1e3) / 1e12, 1),
                                   "peak_tflops": tf_sust, "frac": round(flops / (p8 / n8 / 1e3) / 1e12 / tf_sust, 4),
                                   "note": "int8 projections (kind::i8); peak is the measured bf16 sustained rate"},
              "e2e": {"value": round(e8, 2), "unit": "tok/s", "path": "Qwen35Engine.generate (A8W8)"},
              "dtype": "int8 weights (M/F/L groups), per-token int8 activations, int32 accumulate; bf16 LM head"}
        del g8
        eng8._graphs.clear()

    # ---- lock-step decode with the vocab-sharded LM head (the mode with a data-path collective)
    shard = None
    if sharded is not None and head is None:
        import torch.distributed as dist

        from ppu_b200 import kernels as K

        ns, ws_ = min(args.steps, 10), min(args.warmup, 3)
        gs = sharded.capture(1)
        ts, ds, ps, _ = time_requests(eng, gs, prompts, ws_, ns, T)
        ds = max_over_ranks(ds)
        vs = R.aggregate_rate(ns * T, ds / 1000.0, world)
        # the per-token exchange alone: all-gather of the residuals + MAX all-reduce of the keys
        cg = torch.cuda.CUDAGraph()
        reps = 64
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.cuda.graph(cg, stream=side):
            for _ in range(reps):
                dist.all_gather_into_tensor(sharded.gathered, sharded.hidden)
                dist.all_reduce(sharded.keys, op=dist.ReduceOp.MAX)
        torch.cuda.current_stream(dev).wait_stream(side)
        cg.replay()
        torch.cuda.synchronize()
        R.barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        cg.replay()
        c1.record()
        torch.cuda.synchronize()
        coll_us = max_over_ranks(c0.elapsed_time(c1) * 1000.0 / reps)
        # the shard top-1 launch alone (world hiddens against this rank's 1/world of the table)
        kg = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side), torch.cuda.graph(kg, stream=side):
            for _ in range(reps):
                K.lm_head_shard_keys(sharded.gathered, sharded.shard, sharded.row0, sharded.vocab,
                                     norm_weight=eng.final_norm, eps=dims.eps, workspace=sharded.workspace,
                                     out=sharded.keys)
        torch.cuda.current_stream(dev).wait_stream(side)
        kg.replay()
        torch.cuda.synchronize()
        c0.record()
        kg.replay()
        c1.record()
        torch.cuda.synchronize()
        shard_us = max_over_ranks(c0.elapsed_time(c1) * 1000.0 / reps)
        shard_bytes = sharded.shard.numel() * 2
        toks_s, ttft_s, el_s = sharded.generate(make_prompt(dims, P, seed=80_000 + rank)[0], T + 1)
        es = R.aggregate_rate(len(toks_s) - 1, max_over_ranks(el_s - ttft_s), world)
        shard = {"value": round(vs, 2), "unit": "tok/s", "steps": ns, "warmup": ws_,
                 "decode_ms_per_token": round(ds / ns / T, 4),
                 "vs_replicas": round(vs / value, 4),
                 "collective_us_per_token": round(coll_us, 2),
                 "shard_top1_us": round(shard_us, 2),
                 "shard_top1_gbs": round(shard_bytes / (shard_us * 1e-6) / 1e9, 1),
                 "shard_rows": int(sharded.shard.shape[0]),
                 "limiter": "per token: NCCL all_gather (world x 4 KB) + int64 MAX all_reduce, measured alone as "
                            "collective_us_per_token, against the shard top-1 launch it shortens the LM head to",
                 "e2e": {"value": round(es, 2), "unit": "tok/s", "path": "ShardedDecode.generate"}}
        del gs, cg, kg
        sharded.release()

    # ---- config 5: the multimodal request stream (replicas; at N > 1 also lock-step with the
    # vocab-sharded LM head)
    batched = batched_decode_leg(engB, dims, dev, rank, world, args, hbm_peak, peak_kind) if engB else None
    mm = mm_batched = mm_shard = None
    if args.mm_requests > 0:
        vis = vision_engine(dev, max_images=engB.batch if engB is not None else 1)
        mm = multimodal_leg(eng, vis, None, dims, dev, rank, world, args, tf_sust, peak_kind)
        if engB is not None:
            mm_batched = multimodal_leg(engB, vis, None, dims, dev, rank, world, args, tf_sust, peak_kind)
        if sharded is not None and head is None:
            mm_shard = multimodal_leg(eng, vis, sharded.capture(1), dims, dev, rank, world, args, tf_sust, peak_kind)
            sharded.release()

    cpu = None
    if weights_cpu is not None:
        threads = len(os.sched_getaffinity(0))
        cpu_ttft, per_tok = cpu_reference_sample(dims, weights_cpu, P, args.cpu_tokens, threads)
        med = statistics.median(per_tok)
        cpu = {"value": round(1.0 / med, 3), "unit": "tok/s", "cores": threads, "kind": "hf-eager",
               "ttft_ms": round(cpu_ttft * 1000, 1),
               "sample": f"the reference's CPU path, Transformers eager Qwen3_5ForCausalLM (attn_implementation="
                         f"eager), bf16, same seeded weights, {threads} host threads: prefill {P} tokens, then "
                         f"{args.cpu_tokens} greedy decode tokens; value = 1 / median per-token time"}

    prefill_launches = 1 + 2 + dims.layers * 9 + 1 + (dims.layers * 4 if headline_a8w8 else 0)
    step_kernels = eng.kernels_per_step + (1 if head else 0)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8 (A8W8: int8 weights, per-token int8 activations, int32 accumulate)" if headline_a8w8
        else "bf16",
        "data": "synthetic: seeded random-init 2B-shape weights N(0,0.02), uniform-random prompt ids",
        "config": {
            "workload": f"config4: prefill {P} tokens + {T} greedy decode steps, batch 1 (one step = one request)",
            "model": "Qwen3.5-2B-shape text decoder (24 layers, 3xGatedDeltaNet:1xGQA, hidden 2048, vocab 248320)",
            "global_batch": world, "seq_len": P,
            "parallelism": (f"lock-step decode x{world}, LM head vocab-sharded {dims.vocab // world} rows/rank "
                            "(NCCL all_gather + int64 MAX all_reduce per token)") if head
            else f"request-parallel replicas x{world}",
            "a8w8": headline_a8w8, "pdl": not args.no_pdl, "cuda_graph": "1 decode step per replay",
            "decode_step": "persistent" if eng.persistent else "per-op kernels", "gemv": args.gemv,
            "gemv_ctas_per_sm": args.gemv_ctas or "all that fit",
            "prefill_delta": args.prefill_delta, "prefill_gemm": "tcgen05",
            "l2": "weights 3.8 GB per step >> 126 MB L2 (no flush needed)",
        },
        "per_gpu_value": round(value / world, 2),
        "ttft_ms": round(ttft_ms, 3),
        "decode_ms_per_token": round(decode_ms / args.steps / T, 4),
        "step_hbm": {"bytes_per_token": bytes_tok, "achieved_gbs": round(bytes_tok * value / world / 1e9, 1),
                     "peak_gbs": hbm_peak, "frac": round(bytes_tok * value / world / 1e9 / hbm_peak, 4),
                     "peak_kind": peak_kind},
        "roofline": roofline,
        "prefill_roofline": {"flops": flops, "achieved_tflops": round(flops / (ttft_ms / 1e3) / 1e12, 1),
                             "peak_tflops": tf_sust, "frac": round(flops / (ttft_ms / 1e3) / 1e12 / tf_sust, 4),
                             "bound": "tensor", "peak_kind": f"{peak_kind} bf16 sustained",
                             "what": "TTFT (prefill + first greedy token, device-timed) against all dense prefill "
                                     "FLOPs: projections, causal attention, DeltaNet chunk products, LM head"},
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": P * 8,
                "d2h_bytes_per_step": (T + 1) * 8, "ttft_ms": round(1000 * statistics.mean(e2e_ttft), 3),
                "path": ("ShardedDecode.generate" if head else "Qwen35Engine.generate")
                        + " (host ids -> H2D, prefill, per-token D2H read, graph replay)"},
        "gpu_launches": args.steps * (prefill_launches + T * step_kernels),
        "clocks": clocks,
    }
    if a8 is not None:
        line["a8w8"] = a8
    if shard is not None:
        line["lm_shard"] = shard
    if batched is not None:
        line["decode_batched"] = batched
    if mm is not None:
        line["multimodal"] = mm
    if mm_batched is not None:
        line["multimodal_batched"] = mm_batched
    if mm_shard is not None:
        line["multimodal_lm_shard"] = mm_shard
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        del graph
        eng._graphs.clear()
        if sharded:
            sharded.release()
        torch.cuda.synchronize()
        R.barrier()
        R.shutdown()
    return 0


if __name__ == "__main__":
    sys.exit(main())
