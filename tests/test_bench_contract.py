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


def test_reference_arm_config_matches_our_arm():
    # Both arms print the same workload description (bench.config_dict); the reference arm builds
    # its inputs with the oracle's generators and maps no product library.
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_mod", REPO / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    r = _bench("--impl", "reference", "--config", "c2", "--steps", "3", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][0])
    assert d["config"] == bench.config_dict("c2", 678214, 1, True)
    assert set(d["config"]) == {"workload", "config_id", "nnz", "N", "rows", "cols", "parallelism", "l2"}


def test_parity_checker_catches_a_planted_mistake():
    # bench.parity_rows against rows computed by the oracle itself: equal rows pass; one element
    # changed by one ulp in a sampled row fails (the mistake is planted in the oracle's output).
    import importlib.util

    import numpy as np

    sys.path[:0] = [str(REPO), str(REPO / "sparse-matrix-multiplication_b200")]
    import spmm_b200 as S
    from oracle import oracle as O

    spec = importlib.util.spec_from_file_location("bench_mod", REPO / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    A = S.generate_uniform_csr(3000, 700, 0.02, 42)
    B = S.generate_dense(700, 40, 43)
    r0, r1 = 1000, 2600
    sl = S.row_slice(A, r0, r1)
    C = O.spmm_csr_f32(O.CSR(sl.rows, sl.cols, sl.row_ptr, sl.col_idx, sl.values), B)
    n, ok = bench.parity_rows(A, B, r0, r1, C, S.CSR_ROWWARP, 0)
    assert ok and n == bench.PARITY_ROWS
    rng = np.random.default_rng(1000 + r0)  # the checker's own sample of rows
    row = int(np.sort(rng.choice(r1 - r0, size=bench.PARITY_ROWS, replace=False))[7])
    bad = C.copy()
    bad[row, 3] = np.nextafter(bad[row, 3], np.float32(np.inf))
    assert bench.parity_rows(A, B, r0, r1, bad, S.CSR_ROWWARP, 0) == (bench.PARITY_ROWS, False)


def test_rank_slice_argument_is_checked():
    for bad in ("3/2", "x", "1/0"):
        r = _bench("--impl", "reference", "--config", "c1", "--steps", "3", "--rank-slice", bad, timeout=120)
        assert r.returncode != 0 and "rank-slice" in r.stderr
