"""The data flow of the per-rank multi-GPU path (spmm_rank_run) on CPU ranks (gloo, world_size 2
and 3): every rank builds the same A and B, takes the reference's nnz-balanced row range, holds
only its share of B's rows (rows K*r/world .. K*(r+1)/world, the library's split; unequal when
world does not divide K), the ranks all-gather the shares into the whole B, each computes its
rows (the CPU oracle stands in for the GPU kernel here) and the gathered rows equal the
single-process product bit for bit. A second test drops a rank before the exchange and checks
the survivor gets an error from the short process-group timeout instead of hanging."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_worker(rank: int, world: int, port: int, out_dir: str):
    import sys

    sys.path[:0] = [out_dir.rsplit("|", 1)[1], out_dir.rsplit("|", 1)[1] + "/sparse-matrix-multiplication_b200"]
    out_dir = out_dir.rsplit("|", 1)[0]
    import torch
    import torch.distributed as dist

    import spmm_b200 as S
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    A = S.generate_uniform_csr(3000, 2000, 0.01, 42)
    K = 2000
    full_b = S.generate_dense(K, 48, 43)
    # This rank's share of B's rows, then an all-gather of the shares (padded to the largest
    # share, as gloo's all_gather wants equal sizes) into the whole B.
    share = [K * r // world for r in range(world + 1)]
    mine = torch.zeros(max(share[r + 1] - share[r] for r in range(world)), 48)
    mine[: share[rank + 1] - share[rank]] = torch.from_numpy(full_b[share[rank]:share[rank + 1]])
    parts_b = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(parts_b, mine)
    B = torch.cat([parts_b[r][: share[r + 1] - share[r]] for r in range(world)])
    assert np.array_equal(B.numpy(), full_b)
    bounds = S.nnz_balanced_bounds(A.row_ptr, A.rows, A.nnz, world)
    sl = S.row_slice(A, int(bounds[rank]), int(bounds[rank + 1]))
    Cr = O.spmm_csr_f32(O.CSR(sl.rows, sl.cols, sl.row_ptr, sl.col_idx, sl.values), B.numpy())
    rows = torch.tensor([sl.rows])
    all_rows = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(all_rows, rows)
    mx = int(max(int(r) for r in all_rows))
    pad = torch.zeros(mx, 48)
    pad[: sl.rows] = torch.from_numpy(Cr)
    parts = [torch.zeros(mx, 48) for _ in range(world)]
    dist.all_gather(parts, pad)
    if rank == 0:
        C = torch.cat([p[: int(r)] for p, r in zip(parts, all_rows)]).numpy()
        np.save(os.path.join(out_dir, "C.npy"), C)
        np.save(os.path.join(out_dir, "bounds.npy"), bounds)
    dist.barrier()
    dist.destroy_process_group()


def _drop_worker(rank: int, world: int, port: int, out_dir: str):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the broadcast
    B = torch.ones(10)
    try:
        dist.broadcast(B, src=0)
        dist.barrier()
        msg = "no error"
    except Exception as e:  # noqa: BLE001 - any error from the timed-out collective
        msg = f"error: {type(e).__name__}"
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(msg)
    os._exit(0)


@pytest.mark.parametrize("world", [2, 3])
def test_row_split_gather_equals_single_process(tmp_path, world):
    import torch.multiprocessing as mp

    import spmm_b200 as S
    from oracle import oracle as O

    repo = str(__import__("pathlib").Path(__file__).resolve().parent.parent)
    mp.spawn(_shard_worker, args=(world, _free_port(), f"{tmp_path}|{repo}"), nprocs=world, join=True)
    A = S.generate_uniform_csr(3000, 2000, 0.01, 42)
    B = S.generate_dense(2000, 48, 43)
    want = O.spmm_csr_f32(O.CSR(A.rows, A.cols, A.row_ptr, A.col_idx, A.values), B)
    got = np.load(tmp_path / "C.npy")
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(np.load(tmp_path / "bounds.npy"), S.nnz_balanced_bounds(A.row_ptr, A.rows, A.nnz, world))


def test_lost_rank_is_detected_by_timeout(tmp_path):
    import torch.multiprocessing as mp

    ctx = mp.start_processes(_drop_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(120)
        assert not p.is_alive()
    assert (tmp_path / "rank0.txt").read_text().startswith("error")
