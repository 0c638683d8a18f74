#!/usr/bin/env python3
"""Benchmark of the B200 SpMM engine on BASELINE config 5 (the metric's 1/2/4/8-GPU config).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5|c1|c2|c3|c4] [--impl ours|reference]
                    [--rank-slice R/G]

Workload (default c5): A = generate_uniform_random_csr(131072, 131072, 0.001, seed 42)
(~17.2M nnz, the reference generator's exact matrix), B = 131072 x 256 FP32 U(-1,1) from
mt19937(43), C = A @ B in FP32. At N GPUs (one process per GPU, torchrun) every rank runs the
library's per-rank multi-GPU path (spmm_rank_plan_* / spmm_rank_run of include/spmm_c.h): A is
split into the reference's nnz-balanced row ranges, B reaches every GPU by an NCCL all-gather
over NVLink, and each rank computes its rows of C -- the total work is fixed ("strong" scaling).

One step = one SpMM of the rank's row range, inputs resident in HBM (spmm_rank_execute). `value`
is whole-job GFLOP/s, 2*nnz*N / (max over ranks of the device time of the K timed steps / K).
The inputs (406 MB at N=1) are larger than the 126 MB L2, so no flush is needed between steps.
`e2e` is the same metric from pinned host buffers: per step, every rank copies its rows of A and
its 1/N share of B's rows in, the ranks all-gather B over NVLink, the kernels run and each rank's
rows of C come back -- pipelined inside the library. Its `value` submits the steps back to back
(spmm_rank_submit, one spmm_rank_wait at the end: a step's copy back overlaps the next step's
copies in); `e2e.sync` times one synchronous spmm_rank_run per step. All are timed with CUDA
events on the launching stream, max over ranks. `e2e.host_link` is the roofline of the end-to-end
figure: each rank's bytes of a step moved as plain pinned copies, in and out at once, on all ranks
together (`floor_ms`), and `frac` = floor_ms / ms_per_step.

After the timed regions every rank checks its rows of C from the last end-to-end step against the
CPU oracle (sampled rows, bit for bit) and the line carries `parity`.

`roofline` carries the HBM fraction of the compulsory bytes (the reference's roofline model)
and, for the CSR kernels, `gather_ceiling`: the rate at which the kernel pulls B rows into the
SMs against a load-only probe of random row fetches of B's width (N = 256 or 128) from an
L2-resident part of B.

`--rank-slice R/G` runs rank R's rows of a G-way split alone on one GPU (the same kernel launch
that rank runs at G GPUs), to profile a rank's launch with ncu on a single GPU.

`--impl reference` times the reference's CSR x dense semantics on the host cores (the
oracle's OpenMP port: the reference ships no CPU SpMM of its own) on rank 0 only, on inputs made
by the oracle's own generators.

`--impl reference-gpu` is a same-box comparison on one GPU: the reference's own CUDA kernels,
compiled unchanged for sm_100a from its sources into oracle/_ref/libref.so (tiled_v3, the kernel
its multi-GPU path runs, for the CSR configs; spmm_wmma for config 3), against this engine's
kernels on the same inputs with the same CUDA events; both outputs are compared.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
PKG = REPO / "sparse-matrix-multiplication_b200"
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(PKG))

METRIC = "SpMM GFLOP/s (2*nnz*N/t)"
UNIT = "GFLOP/s"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
CONFIGS = {
    "c5": "multi-GPU uniform CSR 131072^2 p=0.001 (seed 42), N=256, FP32",
    "c1": "uniform CSR 4096^2 p=0.01 (seed 42), N=64, FP32",
    "c2": "banded CSR 8192^2 |i-j|<=41, N=128, FP32",
    "c3": "block-diagonal 8192^2 (64 dense 128^2 blocks) BSR-16 FP16, N=256, FP32 accumulate",
    "c4": "power-law CSR 16384^2 mean 164 alpha 1.8, N=128, FP32",
}
# (rows, cols, N) of every config, for the config dict both arms print.
SHAPES = {"c1": (4096, 4096, 64), "c2": (8192, 8192, 128), "c3": (8192, 8192, 256), "c4": (16384, 16384, 128),
          "c5": (131072, 131072, 256)}
PARITY_ROWS = 1024  # sampled rows per rank checked against the oracle after timing


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", default="c5", choices=sorted(CONFIGS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"])
    p.add_argument("--rank-slice", default=None, help="R/G: rank R's rows of a G-way split, alone on one GPU")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-clocks", action="store_true")
    a = p.parse_args()
    if a.warmup < 3:
        p.error("--warmup must be >= 3")
    if a.steps is None:
        a.steps = 400 if a.config == "c5" else 200
    if a.rank_slice is not None:
        try:
            r, g = (int(x) for x in a.rank_slice.split("/"))
        except ValueError:
            p.error("--rank-slice wants R/G")
        if not (0 <= r < g) or a.config == "c3":
            p.error("--rank-slice wants 0 <= R < G and a CSR config")
        a.rank_slice = (r, g)
    return a


def peaks():
    f = REPO / "MEASURED_PEAKS.json"
    if f.exists():
        try:
            d = json.loads(f.read_text())
            return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
        except (ValueError, KeyError):
            pass
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def config_dict(cfg: str, nnz: int, world: int, small: bool, rank_slice=None) -> dict:
    """The workload description; both arms print the same dict."""
    rows, cols, n = SHAPES[cfg]
    par = f"row-split x{world} (nnz-balanced)"
    if rank_slice is not None:
        par = f"rank {rank_slice[0]} of a {rank_slice[1]}-way row split, alone on one GPU"
    return {"workload": CONFIGS[cfg], "config_id": cfg, "nnz": int(nnz), "N": n, "rows": rows, "cols": cols,
            "parallelism": par, "l2": "L2 flushed between steps" if small else "inputs larger than L2"}


# ------------------------------------------------------------------------ inputs


def build_inputs(cfg: str):
    """Host A (HostCSR) and B (K x N float32) of a config (the product's own generators)."""
    import spmm_patterns

    return spmm_patterns.config(cfg)


# ------------------------------------------------------------------------ clocks


class Clocks:
    """nvidia-smi sampling of SM clock and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, enabled: bool = True):
        self.index = index
        self.proc = None
        self.path = None
        self.enabled = enabled

    def start(self):
        if not self.enabled:
            return
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------ gather ceiling


def gather_ceiling(torch, b_ptr: int, n_cols: int, rows: int, fetches: int, stream) -> float | None:
    """Random whole-row gather rate (GB/s) of this GPU over the first `rows` rows of the device B
    at b_ptr (N = 256 or 128: 1 KB or 512-byte rows): lib/libspmm_probe.so, same residency and
    load width as the CSR kernels, no arithmetic. The median of 5 launches of `fetches` rows."""
    import ctypes as C

    so = PKG / "lib" / "libspmm_probe.so"
    if n_cols not in (128, 256) or not so.exists() or fetches < 8:
        return None
    lib = C.CDLL(str(so))
    lib.spmm_probe_gather_rows.argtypes = [C.c_void_p, C.c_int, C.c_uint32, C.c_longlong, C.c_uint32, C.c_void_p,
                                           C.c_void_p]
    ctas = C.c_int()
    if lib.spmm_probe_ctas(C.byref(ctas)) != 0:
        return None
    out = torch.empty(ctas.value * 256, dtype=torch.float32, device="cuda")
    fetches -= fetches % 8
    ts = []
    for i in range(7):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        rc = lib.spmm_probe_gather_rows(C.c_void_p(b_ptr), n_cols, rows, fetches, i, C.c_void_p(out.data_ptr()),
                                        C.c_void_p(stream.cuda_stream))
        b.record(stream)
        torch.cuda.synchronize()
        if rc != 0:
            return None
        if i >= 2:
            ts.append(a.elapsed_time(b))
    return fetches * 4.0 * n_cols / (statistics.median(ts) * 1e-3) / 1e9


# ------------------------------------------------------------------------ CPU baseline and checker


def cpu_baseline_run(A, B, steps: int, warmup: int):
    """The reference's CSR x dense semantics on all host cores (oracle port)."""
    from oracle import oracle as O

    oa = O.CSR(A.rows, A.cols, A.row_ptr, A.col_idx, A.values)
    threads = os.cpu_count() or 1
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        O.spmm_csr_f32(oa, B, threads=threads, dynamic=False)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    flops = 2.0 * A.nnz * B.shape[1]
    med = statistics.median(times)
    return flops / med / 1e9, threads, med


def parity_rows(A, B: np.ndarray, r0: int, r1: int, C_rows: np.ndarray, algo: int, chunk: int) -> tuple[int, bool]:
    """Checker, run after the timed regions: this rank's rows of C against the CPU oracle, bit
    for bit. One-warp-per-row plans follow the reference's sequential FMA chain per element
    (spmm_baseline.cu:19-24), so PARITY_ROWS sampled rows are compared with oracle.spmm_csr_f32;
    merge-path plans cut long rows at chunk boundaries of the launch, so all its rows are
    compared with oracle.spmm_csr_f32_split. Returns (rows checked, all equal)."""
    from oracle import oracle as O

    import spmm_b200 as S

    rows = r1 - r0
    if rows == 0:
        return 0, True
    if algo == S.CSR_MERGE:
        sl = S.row_slice(A, r0, r1)
        want = O.spmm_csr_f32_split(O.CSR(sl.rows, sl.cols, sl.row_ptr, sl.col_idx, sl.values), B, chunk)
        return rows, bool(np.array_equal(C_rows.view(np.uint32), want.view(np.uint32)))
    rng = np.random.default_rng(1000 + r0)
    k = min(PARITY_ROWS, rows)
    idx = np.sort(rng.choice(rows, size=k, replace=False)) + r0
    starts, ends = A.row_ptr[idx].astype(np.int64), A.row_ptr[idx + 1].astype(np.int64)
    lens = ends - starts
    sub_rp = np.zeros(k + 1, np.int32)
    np.cumsum(lens, out=sub_rp[1:])
    sel = (np.repeat(starts - sub_rp[:-1], lens) + np.arange(int(lens.sum()))).astype(np.int64)
    sub = O.CSR(k, A.cols, sub_rp, np.ascontiguousarray(A.col_idx[sel]), np.ascontiguousarray(A.values[sel]))
    want = O.spmm_csr_f32(sub, B)
    got = np.ascontiguousarray(C_rows[idx - r0])
    return k, bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))


# ------------------------------------------------------------------------ main


def host_link(torch, h2d: int, d2h: int, R, reps: int = 5) -> dict:
    """The host link's floor for one end-to-end step: `h2d` bytes in and `d2h` bytes out between
    pinned host memory and this GPU, each direction alone and both at once (the in-copies in 16
    pieces on one stream, the out-copies in 8 on another, as a step issues them), every rank at
    the same time so that ranks sharing a PCIe switch or a host socket share it here too. Plain
    copies, no kernels; median of `reps`, max over ranks."""
    dev = torch.device("cuda", torch.cuda.current_device())
    h_in = torch.empty(max(h2d, 1), dtype=torch.uint8).pin_memory()
    h_out = torch.empty(max(d2h, 1), dtype=torch.uint8).pin_memory()
    d_in = torch.empty(max(h2d, 1), dtype=torch.uint8, device=dev)
    d_out = torch.empty(max(d2h, 1), dtype=torch.uint8, device=dev)
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    cur = torch.cuda.current_stream()

    def issue(do_in: bool, do_out: bool):
        ev = torch.cuda.Event()
        ev.record(cur)
        for s, on, n, pieces, dst, src in ((s_in, do_in, h2d, 16, d_in, h_in), (s_out, do_out, d2h, 8, h_out, d_out)):
            s.wait_event(ev)
            if not on or n == 0:
                continue
            with torch.cuda.stream(s):
                cut = [n * j // pieces for j in range(pieces + 1)]
                for a, b in zip(cut, cut[1:]):
                    dst[a:b].copy_(src[a:b], non_blocking=True)
            done = torch.cuda.Event()
            done.record(s)
            cur.wait_event(done)

    def timed(do_in: bool, do_out: bool) -> float:
        ts = []
        for _ in range(reps + 1):
            R.barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(cur)
            issue(do_in, do_out)
            b.record(cur)
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return R.max(statistics.median(ts[1:]))

    t_in, t_out, t_both = timed(True, False), timed(False, True), timed(True, True)
    del h_in, h_out, d_in, d_out
    return {"h2d_gbs": round(h2d / (t_in * 1e-3) / 1e9, 2), "d2h_gbs": round(d2h / (t_out * 1e-3) / 1e9, 2),
            "both_ms": round(t_both, 4)}


class Ranks:
    """torch.distributed helpers: barrier, max / sum / min over ranks (no-ops at one rank)."""

    def __init__(self, torch, dist, world: int):
        self.torch, self.dist, self.world = torch, dist, world

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def _reduce(self, x: float, op) -> float:
        if self.world == 1:
            return x
        t = self.torch.tensor([x], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=op)
        return float(t.item())

    def max(self, x: float) -> float:
        return self._reduce(x, self.dist.ReduceOp.MAX)

    def sum(self, x: float) -> float:
        return self._reduce(x, self.dist.ReduceOp.SUM)

    def min(self, x: float) -> float:
        return self._reduce(x, self.dist.ReduceOp.MIN)


def time_steps(torch, step, K: int, stream, flush, R: Ranks):
    """K steps on `stream`, each bracketed by CUDA events; the region bracketed by a barrier and
    a synchronize on both sides. Returns (ms per step: region / K, or the sum of the per-step
    times when an L2 flush runs between steps; average per-step ms)."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    R.barrier()
    torch.cuda.synchronize()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(K):
        if flush is not None:
            flush.fill_(float(i))  # L2 flush between steps (inputs smaller than L2)
        evs[i][0].record(stream)
        step()
        evs[i][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    R.barrier()
    per = [a.elapsed_time(b) for a, b in evs]
    region = sum(per) if flush is not None else t_start.elapsed_time(t_end)
    return region / K, sum(per) / K


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        print(f"WORLD_SIZE={world} but --gpus={args.gpus}", file=sys.stderr)
    cfg_name = args.config
    if world > 1 and cfg_name != "c5":
        raise SystemExit("only config c5 is sharded across GPUs")
    if world > 1 and args.rank_slice is not None:
        raise SystemExit("--rank-slice runs on one GPU")

    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.impl == "reference-gpu":
        return run_reference_gpu(args, rank, world)

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    R = Ranks(torch, dist, world)
    try:
        line = (run_bsr if cfg_name == "c3" else run_csr)(args, torch, dist, R, rank, world, local)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


def run_csr(args, torch, dist, R: Ranks, rank: int, world: int, local: int) -> dict:
    import spmm_b200 as S

    cfg_name = args.config
    A, Bh = build_inputs(cfg_name)
    full_nnz = A.nnz
    if args.rank_slice is not None:
        sr, sg = args.rank_slice
        b = S.nnz_balanced_bounds(A.row_ptr, A.rows, A.nnz, sg)
        A = S.row_slice(A, int(b[sr]), int(b[sr + 1]))
    N = Bh.shape[1]
    flops_total = 2.0 * A.nnz * N
    hbm_peak, tc_peak, peak_src = peaks()
    stream = torch.cuda.current_stream()
    small = cfg_name != "c5"

    # Pinned host operands: A's arrays, B, and this rank's rows of C.
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()  # noqa: E731
    hA = S.HostCSR(A.rows, A.cols, pin(A.row_ptr), pin(A.col_idx), pin(A.values))
    hB = pin(Bh)

    # ---- the library's per-rank path: communicator (N > 1), plan, one end-to-end run to load
    comm = None
    if world > 1:
        obj = [S.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = S.RankComm(obj[0], world, rank, timeout_ms=120000)
    plan = S.RankPlan(comm, hA, N, stream)
    r0, r1 = plan.row_begin, plan.row_end
    rows_r = r1 - r0
    hC = torch.empty((max(rows_r, 1), N), dtype=torch.float32).pin_memory().numpy()
    plan.run(hA, hB, hC, stream)
    torch.cuda.synchronize()
    kernel_name = "csr_rowwarp_kernel" if plan.algo == S.CSR_ROWWARP else "csr_merge_kernel"
    chunk = S.csr_chunk(S.CsrView(rows_r, A.cols, plan.nnz, 0, 0, 0), N) if plan.algo == S.CSR_MERGE else 0

    gather_ms = None
    if world > 1:
        ts = []
        for i in range(6):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            R.barrier()
            a.record(stream)
            plan.gather_b(stream)
            b.record(stream)
            torch.cuda.synchronize()
            if i:
                ts.append(a.elapsed_time(b))
        gather_ms = R.max(statistics.median(ts))

    def step(s=None):
        plan.execute(s or stream)

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda") if small else None
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    code, detail = S.device_error(local)
    if code != 0:
        raise SystemExit(f"device error {code} ({detail}) during warm-up")

    # ---- timed region: kernels on resident operands
    clocks = Clocks(local, enabled=not args.no_clocks)
    clocks.start()
    K = args.steps
    ms_rank, avg_step_ms = time_steps(torch, step, K, stream, flush, R)
    clk = clocks.stop()
    ms_step = R.max(ms_rank)
    code, detail = S.device_error(local)
    if code != 0:
        raise SystemExit(f"device error {code} ({detail}) in the timed region")
    total_flops = 2.0 * R.sum(float(plan.nnz)) * N
    value = total_flops / (ms_step * 1e-3) / 1e9

    # ---- end to end from host buffers (copies inside the timed region). Throughput: ke steps
    # submitted back to back (spmm_rank_submit, alternating between two pinned C buffers), one
    # wait, so a step's copy back of C shares the host link with the next step's copies in;
    # latency: ke synchronous spmm_rank_run calls.
    e2e = None
    if not args.no_e2e:
        hC2 = torch.empty((max(rows_r, 1), N), dtype=torch.float32).pin_memory().numpy()
        for _ in range(2):
            plan.run(hA, hB, hC, stream)
        ke = max(3, min(K, 20))
        ms_sync_rank, _ = time_steps(torch, lambda: plan.run(hA, hB, hC, stream), ke, stream, None, R)
        bufs = (hC2, hC)  # the last submitted step writes hC, which the parity check reads
        hC.fill(np.nan)
        R.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(ke):
            plan.submit(hA, hB, bufs[(i + ke) % 2], stream)
        plan.wait(stream)
        t1.record(stream)
        torch.cuda.synchronize()
        R.barrier()
        e2e_ms = R.max(t0.elapsed_time(t1) / ke)
        sync_ms = R.max(ms_sync_rank)
        h2d_rank = 4 * (rows_r + 1) + 8 * plan.nnz + 4 * (plan.b_row_end - plan.b_row_begin) * N
        d2h_rank = 4 * rows_r * N
        h2d, d2h = R.sum(float(h2d_rank)), R.sum(float(d2h_rank))
        # The floor the host link sets: this rank's bytes of a step, in and out at once, on every
        # rank together (after the timed region)
        link = host_link(torch, h2d_rank, d2h_rank, R)
        e2e = {"value": round(total_flops / (e2e_ms * 1e-3) / 1e9, 3), "unit": UNIT, "ms_per_step": round(e2e_ms, 4),
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "api": "spmm_rank_submit x steps + spmm_rank_wait (C ABI; per rank and step: its A rows and 1/N of "
                      "B's rows H2D from pinned buffers, NCCL all-gather of B over NVLink, kernels, its C rows D2H; "
                      "pipelined in row groups, consecutive steps overlapped)",
               "sync": {"value": round(total_flops / (sync_ms * 1e-3) / 1e9, 3), "ms_per_step": round(sync_ms, 4),
                        "api": "spmm_rank_run per step (returns when the step's C is on the host)"},
               "host_link": {**link, "floor_ms": link["both_ms"], "frac": round(link["both_ms"] / e2e_ms, 4),
                             "probe": "each rank's step bytes as plain pinned copies, in and out at once, all ranks "
                                      "together (in: 16 pieces, out: 8); frac = floor_ms / ms_per_step"}}
    else:
        plan.run(hA, hB, hC, stream)
    torch.cuda.synchronize()

    # ---- parity of this rank's rows (checker, after timing)
    checked, ok = parity_rows(A, Bh, r0, r1, hC[:rows_r], plan.algo, chunk)
    parity = {"rows_checked": int(R.sum(float(checked))), "ok": bool(R.min(1.0 if ok else 0.0) == 1.0),
              "ranks": world, "bitwise": True,
              "oracle": ("oracle.spmm_csr_f32 (sequential FMA chain per element), sampled rows per rank"
                         if plan.algo == S.CSR_ROWWARP else "oracle.spmm_csr_f32_split (merge-path cut), all rows"),
              "source": "C rows of the last end-to-end step (host)"}

    # ---- roofline of the dominant kernel, per step (one pass over the rank's rows: `launches`
    # launches of it when the plan cuts A's columns into phases), this rank; rank 0 reports
    alg_bytes = 8 * plan.nnz + 4 * (rows_r + 1) + 4 * A.cols * N + 4 * rows_r * N
    launches = max(plan.launches, 1)
    achieved = alg_bytes / (avg_step_ms * 1e-3) / 1e9
    gpus_key = args.rank_slice[1] if args.rank_slice is not None else world
    traffic = None
    prof = REPO / "profiles" / f"{kernel_name}_config{cfg_name[1:]}.md"
    if prof.exists():
        key = f"dram_bytes_per_step_gpus{gpus_key}:"
        for ln in prof.read_text().splitlines():
            if ln.startswith(key):
                traffic = int(ln.split(":", 1)[1].strip())
    roofline = {"bound": "hbm", "kernel": kernel_name, "achieved": round(achieved, 1), "peak": hbm_peak,
                "unit": "GB/s", "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else peak_src,
                "alg_bytes_per_step": int(alg_bytes), "avg_step_ms": round(avg_step_ms, 5),
                "launches_per_step": launches, "per": "step (one pass over the rank's rows)"}
    gathered = 4.0 * plan.nnz * N  # B-row bytes the gather moves through L2 per step
    gather_gbs = gathered / (avg_step_ms * 1e-3) / 1e9
    roofline["l2_gather_gbs"] = round(gather_gbs, 1)
    # The ceiling that bounds a gather of whole B rows: a load-only probe that pulls random
    # rows of B's width into the SMs from an L2-resident part of B (at most 32 MB), and the same
    # probe over B's whole footprint (uniformly random rows, so it misses L2 more often than the
    # kernel, whose warps walk their sorted columns together).
    res_rows = min(A.cols, (32 << 20) // (4 * max(N, 1)))
    resident = gather_ceiling(torch, plan.d_B, N, res_rows, plan.nnz, stream)
    same = gather_ceiling(torch, plan.d_B, N, A.cols, plan.nnz, stream)
    if resident:
        roofline["gather_ceiling"] = {
            "achieved_gbs": round(gather_gbs, 1), "ceiling_gbs": round(resident, 1),
            "frac": round(gather_gbs / resident, 4), "same_footprint_probe_gbs": round(same or 0.0, 1),
            "probe": f"load-only random {4 * N}-byte B-row fetches, L2-resident {res_rows * 4 * N / 2**20:.0f} MB "
                     "(lib/libspmm_probe.so)"}

    graph = graph_batch(torch, step, flops_total, S, local) if small and world == 1 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.rank_slice is None:
        gf, threads, med = cpu_baseline_run(A, Bh, steps=3, warmup=1)
        cpu = {"value": round(gf, 3), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"full {cfg_name} product, median of 3 (OpenMP static over rows, {med*1e3:.0f} ms each)"}

    path = {"api": "spmm_rank_plan_create / spmm_rank_execute (C ABI)", "kernel": kernel_name,
            "algo": "rowwarp" if plan.algo == S.CSR_ROWWARP else "merge", "rows_this_rank": rows_r,
            "b_allgather_ms": round(gather_ms, 4) if gather_ms is not None else None}
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (reference generators, fixed seeds)",
        "config": config_dict(cfg_name, A.nnz if args.rank_slice else full_nnz, world, small, args.rank_slice),
        "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk, "gpu_launches": K * launches,
        "parity": parity, "path": path, "graph_batch": graph,
    }
    plan.close()
    if comm is not None:
        comm.close()
    return line


def graph_batch(torch, step, flops_total: float, S, local: int):
    """µs-scale configs: a CUDA graph of 100 back-to-back launches (no flush in between, so the
    inputs stay in L2), the launch-overhead-free figure for kernels of a few µs."""
    try:
        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cap):
            step(cap)  # warm the capture stream
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=cap):
            for _ in range(100):
                step(torch.cuda.current_stream())
        torch.cuda.synchronize()
        ts = []
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b) / 100)
        us = statistics.median(ts) * 1e3
        out = {"launches": 100, "us_per_launch": round(us, 3), "value": round(flops_total / (us * 1e-6) / 1e9, 1),
               "unit": UNIT, "l2": "warm (no flush between launches)"}
        del g
    except Exception as e:  # noqa: BLE001 - reported, not fatal
        out = {"error": str(e)[:200]}
    code, detail = S.device_error(local)
    if code != 0:
        raise SystemExit(f"device error {code} ({detail}) in the graph batch")
    return out


def run_bsr(args, torch, dist, R: Ranks, rank: int, world: int, local: int) -> dict:
    """Config 3: BSR-16 FP16 on the tensor cores (spmm_bsr16_plan_*), one GPU."""
    import spmm_b200 as S

    A, Bh = build_inputs("c3")
    N = Bh.shape[1]
    flops_total = 2.0 * A.nnz * N
    hbm_peak, tc_peak, peak_src = peaks()
    stream = torch.cuda.current_stream()
    dev = torch.device("cuda", local)
    Ah = S.csr_to_bsr16(A, S.DTYPE_F16)
    brp = torch.from_numpy(Ah.row_ptr).to(dev)
    bci = torch.from_numpy(Ah.col_idx).to(dev)
    bva = torch.from_numpy(Ah.values.view(np.int16)).to(dev)
    Bd = torch.from_numpy(Bh).to(dev)
    B16 = torch.empty((A.cols, N), dtype=torch.float16, device=dev)
    S.convert_f32(Bd, B16, A.cols * N, S.DTYPE_F16, stream)
    Cd = torch.empty((A.rows, N), dtype=torch.float32, device=dev)
    bview = S.BsrView(Ah.rows, Ah.cols, Ah.block_rows, Ah.block_cols, Ah.num_blocks, Ah.nnz, S.ptr(brp),
                      S.ptr(bci), S.ptr(bva), S.DTYPE_F16)
    bplan = S.BsrPlan(bview, N, stream=stream)  # the per-CTA schedule, made once

    def step(s=None):
        bplan.execute(B16, Cd, s or stream)

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    code, detail = S.device_error(local)
    if code != 0:
        raise SystemExit(f"device error {code} ({detail}) during warm-up")
    clocks = Clocks(local, enabled=not args.no_clocks)
    clocks.start()
    K = args.steps
    ms_step, avg_launch_ms = time_steps(torch, step, K, stream, flush, R)
    clk = clocks.stop()
    code, detail = S.device_error(local)
    if code != 0:
        raise SystemExit(f"device error {code} ({detail}) in the timed region")
    value = flops_total / (ms_step * 1e-3) / 1e9

    # Checker (after timing): the whole C against the FP64 oracle on the same FP16 inputs.
    from oracle import oracle as O

    ob = O.BSR(Ah.rows, Ah.cols, Ah.block_rows, Ah.block_cols, Ah.row_ptr, Ah.col_idx, Ah.values, Ah.nnz)
    ref = O.spmm_bsr_f64(ob, B16.cpu().numpy().view(np.uint16), 0)
    err = float(np.abs(Cd.cpu().numpy() - ref).max() / max(np.abs(ref).max(), 1e-30))
    parity = {"rows_checked": A.rows, "ok": err <= 1e-5, "max_abs_err_over_max_ref": err, "bitwise": False,
              "oracle": "oracle.spmm_bsr_f64 on the same FP16 inputs (tolerance 1e-5 of max |ref|)", "ranks": 1}

    alg_bytes = 512 * Ah.num_blocks + 4 * Ah.num_blocks + 4 * (Ah.block_rows + 1) + 2 * A.cols * N + 4 * A.rows * N
    kernel_name = "bsr_tcgen05_kernel"
    achieved = alg_bytes / (avg_launch_ms * 1e-3) / 1e9
    traffic = None
    prof = REPO / "profiles" / f"{kernel_name}_config3.md"
    if prof.exists():
        for ln in prof.read_text().splitlines():
            if ln.startswith("dram_bytes_per_launch_gpus1:"):
                traffic = int(ln.split(":", 1)[1].strip())
    tflops = 2.0 * A.nnz * N / (avg_launch_ms * 1e-3) / 1e12
    roofline = {"bound": "hbm", "kernel": kernel_name, "achieved": round(achieved, 1), "peak": hbm_peak,
                "unit": "GB/s", "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else peak_src,
                "alg_bytes_per_launch": int(alg_bytes), "avg_launch_ms": round(avg_launch_ms, 5),
                "tensor": {"achieved_tflops": round(tflops, 2), "peak_tflops": tc_peak,
                           "frac": round(tflops / tc_peak, 4)}}
    graph = graph_batch(torch, step, flops_total, S, local)
    cpu = None
    if not args.no_cpu_baseline:
        gf, threads, med = cpu_baseline_run(A, Bh, steps=3, warmup=1)
        cpu = {"value": round(gf, 3), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"full c3 product in FP32, median of 3 (OpenMP static over rows, {med*1e3:.0f} ms each)"}
    bplan.close()
    return {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (reference generators, fixed seeds)", "config": config_dict("c3", A.nnz, world, True),
        "e2e": None, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk, "gpu_launches": K,
        "parity": parity, "path": {"api": "spmm_bsr16_plan_execute (C ABI)", "kernel": kernel_name},
        "graph_batch": graph,
    }


# ------------------------------------------------------------------------ reference arm


def oracle_inputs(cfg: str, rows_prefix: int | None = None):
    """Inputs made by the oracle's own generators (no product code): A as oracle.CSR, B float32.
    For the uniform configs `rows_prefix` builds only the leading rows, which are the same rows
    the full generator makes (the mt19937 Bernoulli scan runs row by row)."""
    from oracle import oracle as O
    from oracle import patterns as P

    rows, cols, n = SHAPES[cfg]
    if cfg in ("c1", "c5"):
        d = 0.01 if cfg == "c1" else 0.001
        A = O.gen_uniform_csr(rows if rows_prefix is None else rows_prefix, cols, d, 42)
    else:
        pat = {"c2": ("banded", {"bandwidth": 41}), "c3": ("block-diagonal", {"block": 128}),
               "c4": ("power-law", {"mean_deg": 164.0, "alpha": 1.8})}[cfg]
        rp, ci, v = P.make(pat[0], rows, cols, 42, **pat[1])
        A = O.CSR(rows, cols, np.ascontiguousarray(rp, np.int32), np.ascontiguousarray(ci, np.int32),
                  np.ascontiguousarray(v, np.float32))
    return A, O.gen_dense(cols, n, 43)


# nnz of every config's full matrix (the generators' outputs at seed 42), for the reference arm's
# config dict when it builds only a sample of the rows.
NNZ = {"c1": 167686, "c2": 678214, "c3": 1048576, "c4": 2686981, "c5": 17184511}


def run_reference(args, rank: int, world: int):
    """The reference semantics on the host cores; rank 0 only. Each step is the CSR x dense
    product of a bounded sample of the workload (the leading rows, sized so that the whole run
    stays within about a minute of CPU time); the rate (GFLOP/s) is the metric."""
    if rank != 0:
        return
    from oracle import oracle as O

    cfg = args.config
    rows, cols, n = SHAPES[cfg]
    budget = 60.0
    if cfg == "c5":
        # Rate on a 4096-row prefix, then as many leading rows as the budget allows.
        A, Bh = oracle_inputs(cfg, 4096)
        _, threads, one = cpu_baseline_run(A, Bh, steps=1, warmup=1)
        want = int(4096 * budget / ((args.steps + args.warmup) * max(one, 1e-6)))
        take = max(1024, min(rows, want))
        if take != 4096:
            A = oracle_inputs(cfg, take)[0]
        full_nnz = None
    else:
        A, Bh = oracle_inputs(cfg)
        full_nnz = A.nnz
        _, threads, one = cpu_baseline_run(A, Bh, steps=1, warmup=0)
        take = rows
        if (args.steps + args.warmup) * one > budget:
            take = max(1, int(rows * budget / ((args.steps + args.warmup) * one)))
            A = O.row_slice(A, 0, take)
    sample = (f"rows 0..{take} of {cfg} ({100.0 * take / rows:.1f} % of the product) per step"
              if take < rows else f"full {cfg} product per step")
    sample += ", OpenMP static over rows; inputs from the oracle's generators"
    gf, threads, med = cpu_baseline_run(A, Bh, steps=args.steps, warmup=args.warmup)
    nnz = full_nnz if full_nnz is not None else NNZ[cfg]
    line = {
        "metric": METRIC, "value": round(gf, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(med * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp16" if cfg == "c3" else "f32",
        "data": "synthetic (reference generators, fixed seeds)",
        "config": config_dict(cfg, nnz, world, cfg != "c5"),
        "impl": "reference",
        "cpu_baseline": {"value": round(gf, 3), "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(gf, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_gpu(args, rank: int, world: int):
    """Same-box GPU comparison (rank 0, one GPU): the reference's kernels recompiled for sm_100a
    (oracle/_ref/libref.so, built from the reference's sources by oracle/Makefile) against this
    engine's, on inputs from the oracle's generators, timed with the same CUDA events."""
    if rank != 0:
        return
    from oracle import oracle as O

    cfg = args.config
    rows, cols, n = SHAPES[cfg]
    base = {"metric": METRIC, "unit": UNIT, "impl": "reference-gpu", "n_gpus": 1,
            "config": config_dict(cfg, NNZ[cfg], 1, cfg != "c5")}
    if not O.ref_available():
        print(json.dumps({**base, "unavailable": "oracle/_ref/libref.so not built (make -C oracle ref)"}), flush=True)
        return
    import ctypes as C

    import torch

    import spmm_b200 as S

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    R = O.ref()
    A, Bh = oracle_inputs(cfg)
    N = Bh.shape[1]
    flops = 2.0 * A.nnz * N
    K = args.steps
    to_dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)  # noqa: E731
    rp, ci, va = to_dev(A.row_ptr), to_dev(A.col_idx), to_dev(A.values)
    stream = torch.cuda.current_stream()  # the legacy default stream, where the reference launches

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(K):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / K

    vp = C.c_void_p
    if cfg == "c3":
        Ab = O.bsr_from_csr(A)
        B16 = O.to_half_bits(Bh)
        brp, bci, bva = to_dev(Ab.row_ptr), to_dev(Ab.col_idx), to_dev(Ab.values.view(np.int16))
        Bd16 = to_dev(B16.view(np.int16))
        C_ref = torch.zeros((rows, N), dtype=torch.float32, device=dev)
        C_our = torch.zeros((rows, N), dtype=torch.float32, device=dev)

        def ref_step():
            R.ref_spmm_wmma_device(rows, cols, Ab.block_rows, Ab.block_cols, Ab.num_blocks, A.nnz, vp(brp.data_ptr()),
                                   vp(bci.data_ptr()), vp(bva.data_ptr()), vp(Bd16.data_ptr()), vp(C_ref.data_ptr()), N)

        view = S.BsrView(rows, cols, Ab.block_rows, Ab.block_cols, Ab.num_blocks, A.nnz, S.ptr(brp), S.ptr(bci),
                         S.ptr(bva), S.DTYPE_F16)
        plan = S.BsrPlan(view, N, stream=stream)
        ms_ref = timed(ref_step)
        ms_our = timed(lambda: plan.execute(Bd16, C_our, stream))
        ref64 = O.spmm_bsr_f64(Ab, B16, 0)
        scale = max(float(np.abs(ref64).max()), 1e-30)
        e_ref = float(np.abs(C_ref.cpu().numpy() - ref64).max()) / scale
        e_our = float(np.abs(C_our.cpu().numpy() - ref64).max()) / scale
        parity = {"max_err_over_max_ref": {"reference": e_ref, "ours": e_our}, "ok": e_our <= 1e-5,
                  "oracle": "oracle.spmm_bsr_f64 on the same FP16 inputs"}
        names = ("spmm_wmma (reference, nvcuda::wmma)", "bsr_tcgen05_kernel (planned)")
        plan.close()
    else:
        Bd = to_dev(Bh)
        C_ref = torch.zeros((rows, N), dtype=torch.float32, device=dev)

        def ref_step():
            R.ref_spmm_csr_device(5, rows, cols, A.nnz, vp(rp.data_ptr()), vp(ci.data_ptr()), vp(va.data_ptr()),
                                  vp(Bd.data_ptr()), vp(C_ref.data_ptr()), N)

        hA = S.HostCSR(rows, cols, A.row_ptr, A.col_idx, A.values)
        plan = S.RankPlan(None, hA, N, stream)
        hC = np.empty((rows, N), np.float32)
        plan.run(hA, Bh, hC, stream)
        ms_ref = timed(ref_step)
        ms_our = timed(lambda: plan.execute(stream))
        plan.run(hA, Bh, hC, stream)
        got_ref = C_ref.cpu().numpy()
        same = bool(np.array_equal(got_ref.view(np.uint32), hC.view(np.uint32)))
        parity = {"bit_identical_to_reference_kernel": same, "ok": same or plan.algo == S.CSR_MERGE,
                  "compare_vs_reference": list(O.compare(hC, got_ref))}
        names = ("spmm_tiled_v3 (reference)",
                 "csr_rowwarp_kernel" if plan.algo == S.CSR_ROWWARP else "csr_merge_kernel")
        plan.close()
    line = {**base, "value": round(flops / (ms_ref * 1e-3) / 1e9, 3), "ms_per_step": round(ms_ref, 5),
            "steps": K, "warmup": args.warmup, "higher_is_better": True, "reference_kernel": names[0],
            "ours": {"kernel": names[1], "ms_per_step": round(ms_our, 5),
                     "value": round(flops / (ms_our * 1e-3) / 1e9, 3)},
            "speedup_ours_over_reference": round(ms_ref / ms_our, 3), "parity": parity,
            "data": "synthetic (the oracle's generators, fixed seeds)", "gpu": torch.cuda.get_device_name(0)}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
