"""bench.py's output contract, checked on the CPU through the reference arm (which runs the
oracle's CPU product and needs no GPU): one JSON line with the keys the driver reads, the arm's
`impl`, a `cpu_baseline` describing the run and an `e2e` with zero transfer bytes; argument
checks (warm-up below 3 is rejected)."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def _bench(*args: str, timeout: int = 300) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, str(REPO / "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, cwd=REPO)


def test_reference_arm_prints_one_contract_line():
    r = _bench("--impl", "reference", "--config", "c1", "--steps", "3", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3
    assert d["unit"] == "GFLOP/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["config_id"] == "c1" and d["config"]["nnz"] == 167686
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_warmup_below_three_is_rejected():
    r = _bench("--impl", "reference", "--config", "c1", "--steps", "1", "--warmup", "2", timeout=120)
    assert r.returncode != 0 and "warmup" in r.stderr
