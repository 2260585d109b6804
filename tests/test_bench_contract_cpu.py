"""bench.py's reference arm on the host (no GPU needed): the JSON line the driver reads, and the
torchrun behaviour where only rank 0 runs and prints while the other ranks exit 0 without work."""

import json
import os
import subprocess
import sys

from conftest import REPO


def _run(env_extra, steps=1):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference",
                           "--steps", str(steps), "--warmup", "3"],
                          cwd=str(REPO), env=env, capture_output=True, text=True, timeout=900)


def test_reference_arm_line_carries_the_contract_keys():
    p = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"].startswith("BDH prefill tokens/s (config 2")
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("reference", "port")
    assert cb["cores"] >= 1 and "T=512" in cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_runs_on_rank_zero_only():
    p = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
