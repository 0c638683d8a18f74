"""sweep.py on the CPU: the reference-format outputs of the B200 pattern sweep.

The pattern sweep writes the reference's tidy CSV (scripts/run_pattern_sweep.py:147 columns:
pattern,kernel,m,k,n,nnz,density,time_ms,gflops) over the reference's grid and generator
parameters (:46-51); --dry-run builds the matrices without a GPU. The roofline mode turns such a
CSV into the reference's roofline table (scripts/roofline.py:177-212, columns :236-239) with B200
ceilings. Both run here on a tiny grid."""
from __future__ import annotations

import csv
import subprocess
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent.parent
SWEEP = REPO / "sparse-matrix-multiplication_b200" / "sweep.py"

REF_SWEEP_COLUMNS = ["pattern", "kernel", "m", "k", "n", "nnz", "density", "time_ms", "gflops"]
REF_ROOFLINE_COLUMNS = ["kernel", "m", "density", "nnz", "gflops", "ai_flop_per_byte", "ceiling_gflops",
                        "pct_fp32_peak", "pct_roofline", "eff_dram_bw_gbs", "pct_dram_bw", "bound", "B_fits_L2"]


def _run(*args: str) -> subprocess.CompletedProcess:
    r = subprocess.run([sys.executable, str(SWEEP), *args], capture_output=True, text=True, timeout=300, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    return r


def test_pattern_sweep_dry_run_writes_reference_columns(tmp_path):
    out = tmp_path / "pattern_sweep.csv"
    _run("--pattern-sweep", "--dry-run", "--max-size", "1024", "--patterns", "banded", "block-diagonal", "--out",
         str(out))
    with open(out, newline="") as fh:
        reader = csv.DictReader(fh)
        assert reader.fieldnames == REF_SWEEP_COLUMNS
        rows = list(reader)
    assert [r["pattern"] for r in rows] == ["banded"] * 4 + ["block-diagonal"] * 4
    kernels = [r["kernel"] for r in rows]
    assert kernels[:3] == ["csr_rowwarp", "csr_merge", "bsr16_tc"] and kernels[3] == "hybrid[wmma]"
    # banded, bandwidth 32 (gen_matrices.py --bandwidth): |i - j| <= 32 inside 1024 x 1024
    i = np.arange(1024)
    band = int((np.minimum(1023, i + 32) - np.maximum(0, i - 32) + 1).sum())
    assert int(rows[0]["nnz"]) == band
    # block-diagonal, block 16: 64 dense 16 x 16 blocks
    assert int(rows[4]["nnz"]) == 1024 * 16
    for r in rows:
        assert (r["m"], r["k"], r["n"]) == ("1024", "1024", "256") and r["time_ms"] == "" and r["gflops"] == ""


def test_roofline_table_from_a_sweep_csv(tmp_path):
    src = tmp_path / "in.csv"
    with open(src, "w", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=REF_SWEEP_COLUMNS)
        w.writeheader()
        # config 5's shape: 17184511 nonzeros, N = 256, 0.951 ms
        w.writerow({"pattern": "uniform", "kernel": "csr_rowwarp", "m": 131072, "k": 131072, "n": 256,
                    "nnz": 17184511, "density": 0.001, "time_ms": 0.951, "gflops": 9251.0})
        w.writerow({"pattern": "uniform", "kernel": "csr_rowwarp", "m": 1024, "k": 1024, "n": 256, "nnz": 10529,
                    "density": 0.01, "time_ms": 0.0, "gflops": ""})  # untimed rows are skipped
    out = tmp_path / "roofline.csv"
    _run("--roofline-from", str(src), "--out", str(out))
    with open(out, newline="") as fh:
        reader = csv.DictReader(fh)
        assert reader.fieldnames == REF_ROOFLINE_COLUMNS
        rows = list(reader)
    assert len(rows) == 1
    r = rows[0]
    dram = 8 * 17184511 + 4 * 131073 + 4 * 131072 * 256 * 2
    ai = 2.0 * 17184511 * 256 / dram
    assert abs(float(r["ai_flop_per_byte"]) - ai) < 1e-9 * ai
    assert abs(float(r["eff_dram_bw_gbs"]) - dram / 0.951e6) < 1e-3
    assert r["bound"] == "compute/L2" and r["B_fits_L2"] == "False"  # AI 21.6 > ridge ~11.5; B 134 MB > L2
    assert float(r["pct_roofline"]) == float(r["pct_fp32_peak"])  # above the ridge the ceiling is the FP32 peak
