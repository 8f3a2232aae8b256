#!/usr/bin/env python3
"""Benchmark of the Qwen3.5-2B-shape fused decode path.

Workload per step (one request): prefill 1024 uniform-random token ids, then 32 greedy decode
steps with the fused LM-head top-1, batch 1, random-init 2B-shape weights (N(0, 0.02)), all
resident in HBM before the timed region. Metric: decode tokens/s (whole job, all ranks), timed
on the device with CUDA events; TTFT is reported beside it. One process per GPU; each rank is
an independent model replica on its own seeded requests (request-level data parallelism, no
collectives on the data path: "scaling": "weak").

``--impl reference`` times the reference's CPU path instead (the eager PyTorch restatement in
``oracle/``, the only CPU implementation of this path) on the host cores, rank 0 only.
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
    ap.add_argument("--a8w8", action="store_true", help="int8 weights / per-token int8 activations (M/F/L groups)")
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--gemv", default="registers", choices=["registers", "bulk"],
                    help="decode GEMV weight streaming: shared-memory bulk copies or register loads")
    ap.add_argument("--gemv-ctas", type=int, default=0, help="decode GEMV grid cap in CTAs per SM (0: all that fit)")
    ap.add_argument("--prefill-delta", default="chunked", choices=["chunked", "sequential"])
    ap.add_argument("--decode", default="kernels", choices=["kernels", "persistent"],
                    help="decode step: one persistent cooperative kernel (bf16) or the per-op kernels")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--lm-shard", action="store_true",
                    help="N > 1: lock-step decode with the LM head split over the vocabulary (NCCL all_gather of "
                         "the final residuals + int64 MAX all_reduce of the top-1 keys) instead of full replicas")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


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


def cpu_decode_baseline(weights_cpu, dims, prompt_len: int, decode_tokens: int, threads: int):
    """Decode tok/s of the reference's eager CPU path (oracle restatement) on the host cores."""
    from oracle.model import OracleDecoder

    torch.set_num_threads(threads)
    dec = OracleDecoder(weights_cpu, dims, max_cache_len=prompt_len + decode_tokens + 8)
    prompt = make_prompt(dims, prompt_len, seed=99)
    t0 = time.perf_counter()
    h = dec.forward(prompt)
    tok = dec.next_token(h[:, -1])
    ttft = time.perf_counter() - t0
    t1 = time.perf_counter()
    for _ in range(decode_tokens):
        h = dec.forward(tok)
        tok = dec.next_token(h[:, -1])
    dt = time.perf_counter() - t1
    return decode_tokens / dt, ttft


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    dims = Qwen35Dims()
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    weights = make_weights(dims, seed=0)
    from oracle.model import OracleDecoder

    dec = OracleDecoder(weights, dims, max_cache_len=args.prompt_len + 4 * (args.steps + args.warmup) + 8)
    prompt = make_prompt(dims, args.prompt_len, seed=1)
    t0 = time.perf_counter()
    h = dec.forward(prompt)
    tok = dec.next_token(h[:, -1])
    ttft = time.perf_counter() - t0
    per_step = 4  # decode tokens per step: a bounded sample of the 32-token workload
    for _ in range(args.warmup * per_step):
        h = dec.forward(tok)
        tok = dec.next_token(h[:, -1])
    t1 = time.perf_counter()
    for _ in range(args.steps * per_step):
        h = dec.forward(tok)
        tok = dec.next_token(h[:, -1])
    dt = time.perf_counter() - t1
    value = args.steps * per_step / dt
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1000 * dt / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights, "
        "uniform-random token ids)", "impl": "reference",
        "config": {"workload": "config4: prefill 1024 + greedy decode, 2B-shape decoder, batch 1",
                   "model": "Qwen3.5-2B-shape text decoder (random init)", "global_batch": 1,
                   "seq_len": args.prompt_len, "parallelism": "cpu", "decode_tokens_per_step": per_step},
        "ttft_ms": round(1000 * ttft, 1),
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"eager PyTorch restatement (oracle/), bf16, {threads} threads: prefill "
                                   f"{args.prompt_len} tokens once, then {per_step} greedy decode tokens per step"},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    from ppu_b200 import kernels as K
    from ppu_b200 import replicas as R
    from ppu_b200 import lib as L
    from ppu_b200.engine import Qwen35Engine, cache_bucket

    rank, world, local = R.dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    R.init("nccl", timeout_s=300, device=dev)  # request replicas: no collective on the data path
    barrier = R.barrier

    def max_over_ranks(x: float) -> float:
        return R.max_over_ranks(x, dev)

    dims = Qwen35Dims()
    P, T = args.prompt_len, args.new_tokens
    L.call("q35_set_gemv_variant", L.Q35_GEMV_BULK if args.gemv == "bulk" else L.Q35_GEMV_REGISTERS)
    L.call("q35_set_gemv_ctas_per_sm", args.gemv_ctas)
    weights = make_weights(dims, seed=0, device=dev)
    eng = Qwen35Engine(weights, dims, a8w8=args.a8w8, max_len=cache_bucket(P, T), max_prefill=P, device=dev,
                       use_pdl=not args.no_pdl, prefill_chunked=args.prefill_delta == "chunked",
                       persistent=(args.decode == "persistent" and not args.a8w8))
    gate_up_w = [t["gate_up"] for t in eng.layer_tensors]
    post_ln = [t["post_ln"] for t in eng.layer_tensors]
    gate_up_s = [t.get("gate_up_scale") for t in eng.layer_tensors]
    weights_cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        weights_cpu = {k: v.cpu() for k, v in weights.items()}
    del weights
    torch.cuda.empty_cache()

    n_req = args.warmup + args.steps
    prompts = [make_prompt(dims, P, seed=R.request_seed(rank, i))[0].to(dev) for i in range(n_req)]
    sharded = None
    if args.lm_shard and world > 1:
        from ppu_b200.vocab_shard import ShardedDecode
        sharded = ShardedDecode(eng)
    graph = sharded.capture(1) if sharded else eng.capture(1)
    torch.cuda.synchronize()

    def request(i, ev=None):
        if ev:
            ev[0].record()
        eng.prefill(prompts[i])
        if ev:
            ev[1].record()
        for _ in range(T):
            graph.replay()
        if ev:
            ev[2].record()

    for i in range(args.warmup):
        request(i)
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for s in range(args.steps):
            request(args.warmup + s, evs[s])
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
    total_ms = evs[0][0].elapsed_time(evs[-1][2])
    decode_ms = sum(e[1].elapsed_time(e[2]) for e in evs)
    prefill_ms = sum(e[0].elapsed_time(e[1]) for e in evs)
    total_ms, decode_ms, prefill_ms = (max_over_ranks(x) for x in (total_ms, decode_ms, prefill_ms))
    value = R.aggregate_rate(args.steps * T, decode_ms / 1000.0, world)
    bytes_tok = dims.weight_bytes_per_token(args.a8w8) + 2 * dims.n_attn * dims.kv_heads * dims.head_dim * 2 * (P + T // 2)
    hbm_peak, tf_peak, peak_kind = peaks()

    # ---- dominant kernel (gate/up GEMV with fused RMSNorm + SwiGLU), cold weights rotated over the 24 layers
    resid = torch.randn(dims.hidden, device=dev).to(torch.bfloat16)
    n_rep = 3

    def gate_up_launches():
        for j in range(len(gate_up_w)):
            K.fused_gemv(gate_up_w[j], resid, prologue=L.PRO_NORM, epilogue=L.EPI_SWIGLU, norm_weight=post_ln[j],
                         w_scale=gate_up_s[j])

    gate_up_launches()
    torch.cuda.synchronize()
    # captured once so host launch overhead does not pace the kernels; replayed on this stream
    kgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(kgraph):
        for _ in range(n_rep):
            gate_up_launches()
    kgraph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    kgraph.replay()
    e1.record()
    torch.cuda.synchronize()
    del kgraph
    kern_s = e0.elapsed_time(e1) / 1000.0 / (n_rep * len(gate_up_w))
    w_bytes = gate_up_w[0].numel() * gate_up_w[0].element_size() + (gate_up_w[0].shape[0] * 4 if args.a8w8 else 0)
    achieved = w_bytes / kern_s / 1e9
    traffic = None
    tfile = ROOT / "profiles" / ("gemv_swiglu_a8w8_traffic.json" if args.a8w8 else "gemv_swiglu_traffic.json")
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get("bytes_per_launch")

    # ---- end to end through the public generate path (host prompt, per-token host reads)
    e2e_tok, e2e_time, e2e_ttft = 0, 0.0, []
    for i in range(2):
        host_prompt = make_prompt(dims, P, seed=50_000 + R.request_seed(rank, i))[0]
        toks, ttft, elapsed = (sharded or eng).generate(host_prompt, T + 1)
        e2e_tok += len(toks) - 1
        e2e_time += elapsed - ttft
        e2e_ttft.append(ttft)
    e2e_time = max_over_ranks(e2e_time)
    e2e_value = R.aggregate_rate(e2e_tok, e2e_time, world)

    cpu = None
    if weights_cpu is not None:
        threads = len(os.sched_getaffinity(0))
        cpu_tps, cpu_ttft = cpu_decode_baseline(weights_cpu, dims, 128, 12, threads)
        cpu = {"value": round(cpu_tps, 3), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"oracle/ eager PyTorch restatement, bf16 on {threads} host threads: prefill 128 tokens, "
                         f"then 12 greedy decode tokens timed (TTFT of that 128-token prefill {cpu_ttft * 1000:.0f} ms)"}

    prefill_launches = 1 + 2 + dims.layers * 9 + 1 + (dims.layers * 4 if args.a8w8 else 0)
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
        "dtype": "int8 (A8W8: int8 weights, per-token int8 activations, int32 accumulate)" if args.a8w8 else "bf16",
        "data": "synthetic: seeded random-init 2B-shape weights N(0,0.02), uniform-random prompt ids",
        "config": {
            "workload": f"config4: prefill {P} tokens + {T} greedy decode steps, batch 1 (one step = one request)",
            "model": "Qwen3.5-2B-shape text decoder (24 layers, 3xGatedDeltaNet:1xGQA, hidden 2048, vocab 248320)",
            "global_batch": world, "seq_len": P,
            "parallelism": (f"lock-step decode x{world}, LM head vocab-sharded {dims.vocab // world} rows/rank "
                            "(NCCL all_gather + int64 MAX all_reduce per token)") if sharded
            else f"request-parallel replicas x{world}",
            "a8w8": args.a8w8, "pdl": not args.no_pdl, "cuda_graph": "1 decode step per replay",
            "decode_step": "persistent" if eng.persistent else "per-op kernels", "gemv": args.gemv,
            "gemv_ctas_per_sm": args.gemv_ctas or "all that fit",
            "prefill_delta": args.prefill_delta, "prefill_gemm": "tcgen05",
            "l2": "weights 3.8 GB per step >> 126 MB L2 (no flush needed)",
        },
        "ttft_ms": round(prefill_ms / args.steps, 3),
        "decode_ms_per_token": round(decode_ms / args.steps / T, 4),
        "step_hbm": {"bytes_per_token": bytes_tok, "achieved_gbs": round(bytes_tok * value / world / 1e9, 1),
                     "peak_gbs": hbm_peak, "frac": round(bytes_tok * value / world / 1e9 / hbm_peak, 4),
                     "peak_kind": peak_kind},
        "roofline": {"kernel": f"gemv_{args.gemv}<2048,NORM,SWIGLU> (gate/up + RMSNorm + SwiGLU)", "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
                     "algorithmic_bytes_per_launch": w_bytes, "avg_launch_us": round(kern_s * 1e6, 3),
                     "peak_kind": peak_kind},
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": P * 8,
                "d2h_bytes_per_step": (T + 1) * 8, "ttft_ms": round(1000 * statistics.mean(e2e_ttft), 3),
                "path": ("ShardedDecode.generate" if sharded else "Qwen35Engine.generate")
                        + " (host ids -> H2D, prefill, per-token D2H read, graph replay)"},
        "gpu_launches": args.steps * (prefill_launches + T * (eng.kernels_per_step + (1 if sharded else 0))),
        "clocks": clocks.summary(),
    }
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
