"""The drop-in proof: the reference's own drivers (src/bench/harness.cu -> spmm_bench,
src/bench/spmm_run.cu -> spmm_run), compiled unchanged against include/spmm/ and linked to
libspmm.so (oracle/Makefile target `dropin`), run on the GPU and verified by their own
cuSPARSE comparison. The build needs the reference checkout; the GPU tests use the prebuilt
binaries in oracle/_ref/dropin/ and skip when they were not built."""
from __future__ import annotations

import os
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import spmm_b200 as S
from oracle import oracle as O

REPO = Path(__file__).resolve().parent.parent
DROP = REPO / "oracle" / "_ref" / "dropin"
REF_SRC = O.ref_source()  # $SPMM_REF_SRC, or where the last `make -C oracle ref` found the reference
LINE = re.compile(r"(\w+)=([^\s]+)")


def parse(out: str, prefix: str) -> list[dict]:
    return [dict(LINE.findall(line)) for line in out.splitlines() if line.startswith(prefix)]


@pytest.mark.skipif(REF_SRC is None, reason="reference sources not found: set SPMM_REF_SRC=<reference>/src")
def test_reference_drivers_compile_unchanged_against_our_headers():
    subprocess.run(["make", "-s", "-C", str(REPO / "oracle"), "dropin", f"REF_SRC={REF_SRC}"], check=True)
    for exe in ("spmm_bench", "spmm_run"):
        p = DROP / exe
        assert p.exists()
        r = subprocess.run([str(p), "--help"], capture_output=True, text=True)
        assert r.returncode == 0 and "Usage" in r.stderr
        libs = subprocess.run(["ldd", str(p)], capture_output=True, text=True).stdout
        assert "libspmm.so" in libs and "libspmm_b200.so" in libs


needs_bins = pytest.mark.skipif(not (DROP / "spmm_bench").exists(), reason="drop-in binaries not built")


def run(args: list[str]) -> str:
    r = subprocess.run(args, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


@pytest.mark.gpu
@needs_bins
def test_spmm_bench_all_kernels_pass_cusparse_check(cuda):
    out = run([str(DROP / "spmm_bench"), "--m", "4096", "--k", "4096", "--n", "256", "--density", "0.01",
               "--kernel", "all", "--warmup", "2", "--iters", "5"])
    rows = parse(out, "kernel=")
    names = {r["kernel"] for r in rows}
    assert {"baseline", "memopt", "memopt_v2", "tiled", "tiled_v2", "tiled_v3", "tiled_v4", "wmma"} <= names
    for r in rows:
        assert int(r["nnz"]) == 167686
        bar = 1e-2 if r["kernel"].startswith(("wmma", "hybrid[wmma")) else 1e-4  # README.md:237
        assert float(r["rel_l2_err"]) < bar, r


@pytest.mark.gpu
@needs_bins
def test_spmm_run_modes_pass(cuda, tmp_path):
    for extra in ([], ["--unified"], ["--multi-gpu", "--gpus", "1"]):
        out = run([str(DROP / "spmm_run"), "--m", "2048", "--k", "2048", "--n", "128", "--iters", "3"] + extra)
        assert "[PASS]" in out, out
    # Banded input through --bin: the hybrid rule picks the tensor cores (fill-in 1.348).
    import spmm_patterns as SP

    A = SP.host_csr(8192, 8192, SP.banded_arrays(8192, 8192, 41, 42))
    f = tmp_path / "banded.bin"
    S.write_binary(A, f)
    out = run([str(DROP / "spmm_run"), "--bin", str(f), "--n", "128", "--iters", "3"])
    plan = parse(out, "plan ")[0]
    assert plan["backend"] == "wmma" and abs(float(plan["fill_in"]) - 1.35) < 0.01
    assert "[PASS]" in out


@pytest.mark.gpu
@needs_bins
def test_spmm_run_threshold_flag_selects_b200_routing(cuda, tmp_path):
    """The unchanged spmm_run always passes its own --threshold (default 2.0, the T4 cut-off,
    spmm_run.cu:35,189) to hybrid_choose, so the library's B200 default (6.0) never reaches it;
    B200 routing through that driver needs --threshold 6. Banded bandwidth 6 has fill-in 3.69:
    the T4 cut-off sends it to the CUDA cores, the B200 one to the tensor cores."""
    import spmm_patterns as SP

    A = SP.host_csr(8192, 8192, SP.banded_arrays(8192, 8192, 6, 42))
    f = tmp_path / "banded_bw6.bin"
    S.write_binary(A, f)
    base = [str(DROP / "spmm_run"), "--bin", str(f), "--n", "128", "--iters", "3"]
    plan = parse(run(base), "plan ")[0]
    assert plan["backend"] == "csr" and float(plan["threshold"]) == 2.0
    out = run(base + ["--threshold", "6"])
    plan = parse(out, "plan ")[0]
    assert plan["backend"] == "wmma" and float(plan["threshold"]) == 6.0
    assert abs(float(plan["fill_in"]) - 3.69) < 0.01
    assert "[PASS]" in out
    # Config 2 (banded 41, fill-in 1.35) stays on the tensor cores with the B200 cut-off.
    A2 = SP.host_csr(8192, 8192, SP.banded_arrays(8192, 8192, 41, 42))
    f2 = tmp_path / "banded_bw41.bin"
    S.write_binary(A2, f2)
    out = run([str(DROP / "spmm_run"), "--bin", str(f2), "--n", "128", "--iters", "3", "--threshold", "6"])
    assert parse(out, "plan ")[0]["backend"] == "wmma" and "[PASS]" in out
