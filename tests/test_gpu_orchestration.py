"""The host-buffer orchestration entry points on the GPU: hybrid dispatch (spmm_hybrid_run),
the managed-memory path (spmm_unified_run) and the multi-GPU row split (spmm_multigpu_run,
on every GPU the box shows), each checked against the CPU oracle."""
from __future__ import annotations

import numpy as np
import pytest

import _cases as K
import spmm_b200 as S
import spmm_patterns as SP
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def bits_equal(x, y) -> bool:
    return np.array_equal(np.asarray(x, np.float32).view(np.uint32), np.asarray(y, np.float32).view(np.uint32))


def split_oracle(A: S.HostCSR, B: np.ndarray) -> np.ndarray:
    """The engine's FP32 arithmetic for one launch over A (chunk as the library picks it)."""
    chunk = S.csr_chunk(A.view(), B.shape[1])
    return O.spmm_csr_f32_split(K.to_oracle(A), B, chunk)


def test_hybrid_picks_csr_for_uniform_and_matches(cuda):
    A, B = K.config("c1")
    plan = S.hybrid_choose(A, 64)
    assert plan["backend_name"] == "csr"
    C = np.empty((A.rows, 64), np.float32)
    ms = S.hybrid_run(plan, A, B, C, 64, 2, 5)
    assert ms > 0
    assert bits_equal(C, split_oracle(A, B))


def test_hybrid_picks_tensor_cores_for_banded_and_matches(cuda):
    A, B = K.config("c2")
    plan = S.hybrid_choose(A, 128)
    assert plan["backend_name"] == "wmma"
    C = np.empty((A.rows, 128), np.float32)
    S.hybrid_run(plan, A, B, C, 128, 2, 5)
    hb = S.csr_to_bsr16(A)
    ob = O.BSR(hb.rows, hb.cols, hb.block_rows, hb.block_cols, hb.row_ptr, hb.col_idx, hb.values, hb.nnz)
    ref = O.spmm_bsr_f64(ob, O.to_half_bits(B), 0)
    assert float(np.abs(C - ref).max()) / float(np.abs(ref).max()) <= 1e-5
    c32 = O.spmm_csr_f32(K.to_oracle(A), B)
    assert np.linalg.norm(C - c32) / np.linalg.norm(c32) <= 1e-2


def test_unified_memory_path(cuda):
    A, B = K.config("c1")
    C = np.empty((A.rows, 64), np.float32)
    assert S.unified_run(A, B, C, 64, 1, 3) > 0
    assert bits_equal(C, split_oracle(A, B))


@pytest.mark.parametrize("want_phases", [1, 3, 8, 32])
def test_unified_oversubscription_phases(cuda, want_phases):
    # B (16384 x 512 FP32 = 32 MiB) against a device budget that does not hold it: B's rows
    # move to the device one column phase at a time, the chain carries over in C. Rows are
    # ragged (one long row), and one row is unsorted (its phases cut positions, not columns).
    rng = np.random.default_rng(want_phases)
    lens = rng.integers(0, 70, size=3000)
    lens[17] = 5000
    A = K.random_csr(3000, 16384, lens, seed=3)
    s, e = A.row_ptr[5], A.row_ptr[6]
    A.col_idx[s:e] = A.col_idx[s:e][::-1].copy()
    B = K.dense(16384, 512, 4)
    C = np.full((A.rows, 512), np.nan, np.float32)
    rest = 4 * (A.rows + 1) + 8 * A.nnz + 4 * A.rows * 512 + 4 * 32 * A.rows + (64 << 20)
    b_bytes = B.nbytes
    budget = 0 if want_phases == 1 else rest + -(-b_bytes // want_phases)  # room for 1/P of B
    ms, phases = S.unified_run_ex(A, B, C, 512, budget, 1, 2)
    assert ms > 0 and phases == want_phases
    if want_phases > 1:
        assert bits_equal(C, O.spmm_csr_f32(K.to_oracle(A), B))


@pytest.mark.parametrize("gpus", [1, 2, 8])
def test_multigpu_row_split(cuda, gpus):
    A = S.generate_uniform_csr(8192, 8192, 0.01, 42)
    B = S.generate_dense(8192, 256, 43)
    C = np.full((A.rows, 256), np.nan, np.float32)
    r = S.multigpu_run(A, B, C, 256, gpus, 1, 3)
    g = r["num_gpus"]
    assert g == min(gpus, S.gpu_count())
    bounds = S.nnz_balanced_bounds(A.row_ptr, A.rows, A.nnz, g)
    assert r["rows"] == np.diff(bounds).tolist()
    for k in range(g):
        sl = S.row_slice(A, int(bounds[k]), int(bounds[k + 1]))
        assert r["nnz"][k] == sl.nnz
        # Every device runs the per-rank path, whose plan takes one warp per row for this
        # uniform matrix: the reference's sequential FMA chain for every element.
        assert bits_equal(C[bounds[k]:bounds[k + 1]], O.spmm_csr_f32(K.to_oracle(sl), B))
    if g > 1:
        assert r["bcast_ms"] > 0
