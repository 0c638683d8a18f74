"""The per-rank multi-GPU path (spmm_comm_* / spmm_rank_* of include/spmm_c.h) on the GPU.

Every rank holds the whole host A and B, takes the reference's nnz-balanced row range
(spmm_multigpu.cu:26-40), receives B by an NCCL all-gather of per-rank shares, and returns its
rows of C. The bar is bit equality with the CPU oracle's FP32 arithmetic: the sequential FMA
chain per element for one-warp-per-row plans, the merge-path cut for merge plans.

A world of one runs in this process. Worlds of two run as spawned child processes, one GPU
each, and are skipped on a box with fewer GPUs. The lost-rank test needs one GPU: a child joins
a two-rank communicator that nobody else joins and must get SPMM_ERR_TIMEOUT back from the
library's bounded wait (the failure is made on the host; nothing waits on the GPU).
"""
from __future__ import annotations

import ctypes
import os
import pickle
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest

import _cases as K
import spmm_b200 as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parent.parent


def bits_equal(x, y) -> bool:
    return np.array_equal(np.asarray(x, np.float32).view(np.uint32), np.asarray(y, np.float32).view(np.uint32))


def expected_rows(A: S.HostCSR, B: np.ndarray, r0: int, r1: int, algo: int) -> np.ndarray:
    sl = S.row_slice(A, r0, r1)
    if algo == S.CSR_MERGE:
        chunk = S.csr_chunk(sl.view(), B.shape[1], S.CSR_MERGE)
        return O.spmm_csr_f32_split(K.to_oracle(sl), B, chunk)
    return O.spmm_csr_f32(K.to_oracle(sl), B)


def device_rows(torch, ptr: int, rows: int, N: int) -> np.ndarray:
    """Copy `rows` x N floats from a device pointer the plan owns (cudaMemcpy of the CUDA runtime
    torch loaded)."""
    out = np.empty((rows, N), np.float32)
    if rows * N == 0:
        return out
    torch.cuda.synchronize()
    rt = ctypes.CDLL("libcudart.so.12")
    rc = rt.cudaMemcpy(ctypes.c_void_p(out.ctypes.data), ctypes.c_void_p(ptr), ctypes.c_size_t(out.nbytes), 2)
    assert rc == 0, f"cudaMemcpy failed: {rc}"
    return out


@pytest.mark.parametrize("case", ["c1", "c2", "c4", "ragged"])
def test_world_of_one_matches_oracle(cuda, case):
    torch = cuda
    if case == "ragged":
        # Empty rows, one long row, N that is not a multiple of 4 (scalar B loads).
        lens = np.random.default_rng(7).integers(0, 40, size=5000)
        lens[::97] = 0
        lens[123] = 3000
        A = K.random_csr(5000, 7000, lens, seed=11)
        B = K.dense(7000, 37, 5)
    else:
        A, B = K.config(case)
    N = B.shape[1]
    plan = S.RankPlan(None, A, N)
    assert (plan.row_begin, plan.row_end, plan.nnz) == (0, A.rows, A.nnz)
    assert (plan.b_row_begin, plan.b_row_end) == (0, A.cols)
    want = expected_rows(A, B, 0, A.rows, plan.algo)
    for call in range(2):
        C = np.full((A.rows, N), np.nan, np.float32)
        plan.run(A, B, C)
        assert bits_equal(C, want), f"run {call}"
    # The kernels alone on the resident operands give the same bits.
    plan.execute()
    assert bits_equal(device_rows(torch, plan.d_C, A.rows, N), want)
    code, detail = S.device_error(0)
    assert code == 0, f"device error {code} at {detail}"
    plan.close()


def test_submitted_runs_overlap_and_each_matches(cuda):
    # Four runs submitted back to back (new B, new values of A, both), each into its own
    # C, then one wait: every C must be its own product, bit for bit; then a synchronous run.
    A, B = K.config("c2")
    N = B.shape[1]
    A2 = S.HostCSR(A.rows, A.cols, A.row_ptr, A.col_idx, (A.values * -0.5).astype(np.float32))
    B2 = (B * 3.0).astype(np.float32)
    plan = S.RankPlan(None, A, N)
    jobs = [(A, B), (A, B2), (A2, B), (A2, B2)]
    outs = [np.full((A.rows, N), np.nan, np.float32) for _ in jobs]
    for (a, b), c in zip(jobs, outs):
        plan.submit(a, b, c)
    plan.wait()
    for (a, b), c in zip(jobs, outs):
        assert bits_equal(c, expected_rows(a, b, 0, a.rows, plan.algo))
    C = np.full((A.rows, N), np.nan, np.float32)
    plan.run(A, B2, C)
    assert bits_equal(C, outs[1])
    plan.wait()  # nothing left in flight: returns at once
    code, detail = S.device_error(0)
    assert code == 0, f"device error {code} at {detail}"
    plan.close()


def test_execute_after_submit_waits_on_the_device(cuda):
    # A submitted run (new B) and, on another stream with no host wait between, the kernels
    # alone: they start after the run's copies back, so the device C is the new product.
    torch = cuda
    A, B = K.config("c2")
    N = B.shape[1]
    plan = S.RankPlan(None, A, N)
    C0 = np.full((A.rows, N), np.nan, np.float32)
    plan.run(A, B, C0)
    B2 = (B * 3.0).astype(np.float32)
    want = expected_rows(A, B2, 0, A.rows, plan.algo)
    C1 = np.full((A.rows, N), np.nan, np.float32)
    plan.submit(A, B2, C1)
    other = torch.cuda.Stream()
    plan.execute(other)
    other.synchronize()
    plan.wait()
    assert bits_equal(C1, want)
    assert bits_equal(device_rows(torch, plan.d_C, A.rows, N), want)
    code, detail = S.device_error(0)
    assert code == 0, f"device error {code} at {detail}"
    plan.close()


@pytest.mark.parametrize("after", ["run", "submit"])
def test_execute_captures_in_a_cuda_graph(cuda, after):
    # The kernels alone captured in a CUDA graph, after a synchronous run (nothing to wait for)
    # or after a submitted run still in flight (the wait becomes an external-event node);
    # replayed into a NaN-filled device C they give the run's product.
    torch = cuda
    A, B = K.config("c2")
    N = B.shape[1]
    plan = S.RankPlan(None, A, N)
    C0 = np.full((A.rows, N), np.nan, np.float32)
    if after == "run":
        plan.run(A, B, C0)
    else:
        plan.submit(A, B, C0)
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        plan.execute(side)
    plan.wait()
    want = expected_rows(A, B, 0, A.rows, plan.algo)
    assert bits_equal(C0, want)
    rt = ctypes.CDLL("libcudart.so.12")
    assert rt.cudaMemset(ctypes.c_void_p(plan.d_C), 0xFF, ctypes.c_size_t(4 * A.rows * N)) == 0
    graph.replay()
    torch.cuda.synchronize()
    assert bits_equal(device_rows(torch, plan.d_C, A.rows, N), want)
    code, detail = S.device_error(0)
    assert code == 0, f"device error {code} at {detail}"
    del graph
    plan.close()


def test_phased_plan_runs_pipelined_and_matches(cuda):
    # B of 128 MiB (131072 x 256, about the L2) and 4.3 GB of gathers: the plan takes 3 column
    # phases for the resident launches; the pipelined end-to-end run launches its row groups
    # unphased. Both must give the reference's chain bit for bit.
    torch = cuda
    A = S.generate_uniform_csr_fast(32768, 131072, 0.001, 42)
    B = K.dense(131072, 256, 9)
    plan = S.RankPlan(None, A, 256)
    assert plan.algo == S.CSR_ROWWARP and plan.launches == 3
    C = np.full((A.rows, 256), np.nan, np.float32)
    plan.run(A, B, C)
    for r0 in (0, 16384, 32768 - 512):
        sl = S.row_slice(A, r0, r0 + 512)
        assert bits_equal(C[r0:r0 + 512], O.spmm_csr_f32(K.to_oracle(sl), B)), r0
    plan.execute()
    assert bits_equal(device_rows(torch, plan.d_C, A.rows, 256), C)
    code, detail = S.device_error(0)
    assert code == 0, f"device error {code} at {detail}"
    plan.close()


def test_rank_slice_plans_match_reference_partition(cuda):
    # A world of one on each rank's slice gives that rank's rows: the split the multi-GPU path
    # takes is the reference's nnz-balanced one.
    A = S.generate_uniform_csr(6000, 3000, 0.01, 42)
    B = S.generate_dense(3000, 64, 43)
    bounds = S.nnz_balanced_bounds(A.row_ptr, A.rows, A.nnz, 3)
    assert np.array_equal(bounds, O.nnz_balanced_bounds(K.to_oracle(A), 3))
    for r in range(3):
        sl = S.row_slice(A, int(bounds[r]), int(bounds[r + 1]))
        plan = S.RankPlan(None, sl, 64)
        C = np.empty((sl.rows, 64), np.float32)
        plan.run(sl, B, C)
        assert bits_equal(C, expected_rows(A, B, int(bounds[r]), int(bounds[r + 1]), plan.algo))
        plan.close()


def test_run_refuses_a_different_matrix(cuda):
    A, B = K.config("c1")
    plan = S.RankPlan(None, A, 64)
    other = S.generate_uniform_csr(4096, 4096, 0.02, 7)
    C = np.empty((A.rows, 64), np.float32)
    with pytest.raises(S.SpmmError) as e:
        plan.run(other, B, C)
    assert e.value.status == -1  # SPMM_ERR_INVALID_ARG
    # New values with the same structure are fine.
    A2 = S.HostCSR(A.rows, A.cols, A.row_ptr, A.col_idx, (A.values * 0.5).astype(np.float32))
    plan.run(A2, B, C)
    assert bits_equal(C, O.spmm_csr_f32(K.to_oracle(A2), B))
    plan.close()


# ------------------------------------------------------------------ child processes

_CHILD = textwrap.dedent("""
    import pickle, sys
    sys.path[:0] = [{repo!r}, {repo!r} + "/sparse-matrix-multiplication_b200"]
    import numpy as np, torch
    import spmm_b200 as S
    rank, world, dev, out = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), sys.argv[4]
    job = pickle.load(open(sys.argv[5], "rb"))
    torch.cuda.set_device(dev)
    res = {{}}
    try:
        comm = S.RankComm(job["id"], world, rank, timeout_ms=job["timeout_ms"])
    except S.SpmmError as e:
        res["init_status"] = e.status
        pickle.dump(res, open(out, "wb"))
        sys.exit(0)
    A, B = job["A"], job["B"]
    plan = S.RankPlan(comm, A, B.shape[1])
    C = np.full((max(plan.rows, 1), B.shape[1]), np.nan, np.float32)
    for _ in range(2):
        plan.run(A, B, C)
    res.update(rows=(plan.row_begin, plan.row_end), share=(plan.b_row_begin, plan.b_row_end), algo=plan.algo,
               C=C[:plan.rows])
    # Two runs submitted back to back (B, then 2 B), one wait.
    C1 = np.full_like(C, np.nan)
    C2 = np.full_like(C, np.nan)
    B2 = (B * 2.0).astype(np.float32)
    plan.submit(A, B, C1)
    plan.submit(A, B2, C2)
    plan.wait()
    res.update(C1=C1[:plan.rows], C2=C2[:plan.rows])
    plan.gather_b()
    plan.execute()
    torch.cuda.synchronize()
    plan.close()
    comm.close()
    pickle.dump(res, open(out, "wb"))
""")


def _spawn(tmp_path, world: int, devices, job: dict, timeout: int = 240, pieces: int = 1):
    job_path = tmp_path / "job.pkl"
    job_path.write_bytes(pickle.dumps(job))
    script = tmp_path / "child.py"
    script.write_text(_CHILD.format(repo=str(REPO)))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SPMM_B200_B_PIECES=str(pieces))
    procs = [subprocess.Popen([sys.executable, str(script), str(r), str(world), str(devices[r]),
                               str(tmp_path / f"out{r}.pkl"), str(job_path)], env=env)
             for r in range(len(devices))]
    for p in procs:
        p.wait(timeout=timeout)
        assert p.returncode == 0
    return [pickle.loads((tmp_path / f"out{r}.pkl").read_bytes()) for r in range(len(devices))]


@pytest.mark.parametrize("K_rows,pieces", [(4096, 1), (4093, 1), (4096, 4), (4093, 3)])
def test_two_ranks_gather_b_and_return_their_rows(cuda, tmp_path, K_rows, pieces):
    if S.gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    # K_rows = 4093 gives unequal B shares (grouped send/recv instead of ncclAllGather); pieces > 1
    # exchanges each share piece by piece while the next piece is being copied.
    A = S.generate_uniform_csr(8192, K_rows, 0.01, 42)
    B = S.generate_dense(K_rows, 128, 43)
    res = _spawn(tmp_path, 2, [0, 1], {"id": S.comm_unique_id(), "timeout_ms": 120000, "A": A, "B": B},
                 pieces=pieces)
    bounds = S.nnz_balanced_bounds(A.row_ptr, A.rows, A.nnz, 2)
    for r, d in enumerate(res):
        assert d["rows"] == (int(bounds[r]), int(bounds[r + 1]))
        assert d["share"] == (K_rows * r // 2, K_rows * (r + 1) // 2)
        want = expected_rows(A, B, *d["rows"], d["algo"])
        assert bits_equal(d["C"], want) and bits_equal(d["C1"], want)
        assert bits_equal(d["C2"], expected_rows(A, (B * 2.0).astype(np.float32), *d["rows"], d["algo"]))


def test_rank_that_never_joins_gives_timeout(cuda, tmp_path):
    # Rank 1 of a two-rank communicator never joins: the one that does must come back with
    # SPMM_ERR_TIMEOUT after its 3 s bound instead of waiting for ever.
    A = S.generate_uniform_csr(64, 64, 0.1, 1)
    B = S.generate_dense(64, 16, 2)
    res = _spawn(tmp_path, 2, [0], {"id": S.comm_unique_id(), "timeout_ms": 3000, "A": A, "B": B}, timeout=120)
    assert res[0].get("init_status") == -5  # SPMM_ERR_TIMEOUT
