"""CPU checks of bench.py's command-line contract.

The reference arm (`--impl reference`) times the CPU restatement of the
reference's gather-then-attention decode on the host cores, so it runs here:
one JSON line from rank 0 with the contract's keys, nothing from other ranks.
The GPU arm must fail loudly where there is no GPU, never fall back to a CPU
path and print a number.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _bench(args, env_extra=None, timeout=300):
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    env.pop("LOCAL_RANK", None)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=timeout)


def _json_lines(stdout):
    return [json.loads(l) for l in stdout.splitlines() if l.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    r = _bench(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    d = lines[0]
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 0
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_print_nothing():
    r = _bench(["--impl", "reference", "--steps", "1", "--warmup", "0"],
               {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert _json_lines(r.stdout) == []
    r0 = _bench(["--impl", "reference", "--steps", "1", "--warmup", "0"],
                {"RANK": "0", "WORLD_SIZE": "2", "LOCAL_RANK": "0"})
    assert r0.returncode == 0, r0.stderr[-2000:]
    lines = _json_lines(r0.stdout)
    assert len(lines) == 1 and lines[0]["n_gpus"] == 2


def test_gpu_arm_fails_loudly_without_a_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the GPU arm is covered by the bench runs")
    r = _bench(["--steps", "1", "--warmup", "0"])
    assert r.returncode != 0
    assert _json_lines(r.stdout) == []  # no number from a fallback path
