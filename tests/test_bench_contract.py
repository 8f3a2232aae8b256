"""bench.py's reference arm on the CPU: one JSON line with the contract's keys, timed on the host
cores through the oracle's eager restatement (a tiny prompt keeps it to ~20 s); ranks other than
0 exit without work."""

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
    res = _run("--impl", "reference", "--prompt-len", "16", "--steps", "1", "--warmup", "1")
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work():
    env = {**os.environ, "RANK": "1", "WORLD_SIZE": "2"}
    res = _run("--impl", "reference", "--prompt-len", "16", "--steps", "1", "--warmup", "1", env=env)
    assert res.returncode == 0
    assert not [l for l in res.stdout.splitlines() if l.startswith("{")]
