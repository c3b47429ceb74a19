"""bench.py's contract on a host without a GPU: the reference arm prints one
JSON line with the keys the driver reads, and our arm fails loudly instead of
falling back to a CPU path."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(*args, timeout=600):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, capture_output=True,
                          text=True, timeout=timeout)


def test_reference_arm_prints_one_contract_line():
    r = _run("--impl", "reference", "--workload", "cfg1", "--steps", "2", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["metric"] == "decode tokens/sec" and d["unit"] == "tokens/s"
    assert d["steps"] == 2 and d["warmup"] == 3 and d["higher_is_better"] is True
    assert d["value"] > 0 and d["value"] == d["cpu_baseline"]["value"] == d["e2e"]["value"]
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]


def test_our_arm_has_no_cpu_fallback():
    import torch

    if torch.cuda.is_available():
        return
    r = _run("--workload", "cfg1", "--steps", "2", "--warmup", "3")
    assert r.returncode != 0
    assert not any(ln.startswith("{") for ln in r.stdout.splitlines())
