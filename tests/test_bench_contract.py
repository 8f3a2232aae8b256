"""bench.py's reference arm on the CPU: one JSON line with the contract's keys, timed on the host
cores through the reference's CPU path (Transformers eager Qwen3_5ForCausalLM at the 2B shape; a
16-token prompt and 2 decode tokens per step keep it short); ranks other than 0 exit without
work."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(*args, env=None):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, capture_output=True, text=True,
                          timeout=600, env=env)


def test_reference_arm_prints_one_contract_line():
    res = _run("--impl", "reference", "--prompt-len", "16", "--steps", "1", "--warmup", "1", "--cpu-tokens", "2")
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["kind"] == "hf-eager"
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work():
    env = {**os.environ, "RANK": "1", "WORLD_SIZE": "2"}
    res = _run("--impl", "reference", "--prompt-len", "16", "--steps", "1", "--warmup", "1", env=env)
    assert res.returncode == 0
    assert not [l for l in res.stdout.splitlines() if l.startswith("{")]


def test_cpu_baseline_model_is_the_reference_eager_path_on_the_seeded_weights():
    """The CPU baseline's Transformers eager model, built on the meta device and filled with the
    seeded weights, predicts the oracle's greedy tokens (a tiny shape, so it runs in seconds)."""
    import torch

    sys.path.insert(0, str(ROOT))
    import bench
    from oracle.model import OracleDecoder
    from ppu_b200.config import Qwen35Dims
    from ppu_b200.synthetic import make_prompt, make_weights

    dims = Qwen35Dims(vocab=1024, hidden=512, intermediate=1024, layers=4, q_heads=2, kv_heads=1, lin_heads=2)
    w = make_weights(dims, seed=12)
    prompt = make_prompt(dims, 24, seed=13)
    model = bench.hf_eager_model(w, dims)
    with torch.inference_mode():
        logits = model(input_ids=prompt).logits[0, -1].float()
    oracle = OracleDecoder(w, dims, max_cache_len=64)
    h = oracle.forward(prompt)[:, -1]
    ref = torch.nn.functional.linear(h, oracle.embed).float()[0]
    assert int(logits.argmax()) == int(ref.argmax())
    assert float((logits - ref).abs().max()) < 0.1
