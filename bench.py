#!/usr/bin/env python3
"""Benchmark of the B200 SpMM engine on BASELINE config 5 (the metric's 1/2/4/8-GPU config).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5|c1|c2|c3|c4] [--impl ours|reference]

Workload (default c5): A = generate_uniform_random_csr(131072, 131072, 0.001, seed 42)
(~17.2M nnz, the reference generator's exact matrix), B = 131072 x 256 FP32 U(-1,1) from
mt19937(43), C = A @ B in FP32. At N GPUs (one process per GPU, torchrun) A is split into
nnz-balanced row ranges (the reference's partition), B is broadcast once from rank 0 with
NCCL, and each rank computes its rows of C -- the total work is fixed ("strong" scaling).

One step = one SpMM of the rank's row range, inputs resident in HBM. `value` is whole-job
GFLOP/s, 2*nnz*N / (max over ranks of the device time of the K timed steps / K). The inputs
(406 MB at N=1) are larger than the 126 MB L2, so no flush is needed between steps.
`e2e` repeats the measurement from pinned host buffers. At one GPU through the host-buffer
C entry point (spmm_csr_f32_host): per step, host->device copies of A and B, the kernel, and
the device->host copy of C. At N GPUs: per step every rank copies its A rows in, B crosses the
host links once in total (each rank copies 1/N of its rows, then an NCCL all-gather over
NVLink), every rank runs its plan and copies its C rows out.

`roofline` carries the HBM fraction of the compulsory bytes (the reference's roofline model)
and, for the CSR kernels, `gather_ceiling`: the rate at which the kernel pulls B rows into the
SMs against a load-only probe of random 1 KB row fetches from an L2-resident part of B.

`--impl reference` times the reference's CSR x dense semantics on the host cores (the
oracle's OpenMP port: the reference ships no CPU SpMM of its own) on rank 0 only.
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


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", default="c5", choices=sorted(CONFIGS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-clocks", action="store_true")
    a = p.parse_args()
    if a.warmup < 3:
        p.error("--warmup must be >= 3")
    if a.steps is None:
        a.steps = 400 if a.config == "c5" else 200
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


def gather_ceiling(torch, Bd, rows: int, fetches: int, stream) -> float | None:
    """Random whole-row gather rate (GB/s) of this GPU over the first `rows` rows of Bd
    (N = 256 only): lib/libspmm_probe.so, same residency and load width as the CSR kernels,
    no arithmetic. The median of 5 launches of `fetches` 1 KB rows each."""
    import ctypes as C

    so = PKG / "lib" / "libspmm_probe.so"
    if Bd.shape[1] != 256 or not so.exists() or fetches < 4:
        return None
    lib = C.CDLL(str(so))
    lib.spmm_probe_gather.argtypes = [C.c_void_p, C.c_uint32, C.c_longlong, C.c_uint32, C.c_void_p, C.c_void_p]
    ctas = C.c_int()
    if lib.spmm_probe_ctas(C.byref(ctas)) != 0:
        return None
    out = torch.empty(ctas.value * 256, dtype=torch.float32, device=Bd.device)
    fetches -= fetches % 4
    ts = []
    for i in range(7):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        rc = lib.spmm_probe_gather(C.c_void_p(Bd.data_ptr()), rows, fetches, i, C.c_void_p(out.data_ptr()),
                                   C.c_void_p(stream.cuda_stream))
        b.record()
        torch.cuda.synchronize()
        if rc != 0:
            return None
        if i >= 2:
            ts.append(a.elapsed_time(b))
    return fetches * 1024.0 / (statistics.median(ts) * 1e-3) / 1e9


# ------------------------------------------------------------------------ CPU baseline


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


# ------------------------------------------------------------------------ main


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

    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist

    import spmm_b200 as S

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    A, Bh = build_inputs(cfg_name)
    N = Bh.shape[1]
    total_nnz = A.nnz
    flops_total = 2.0 * total_nnz * N
    hbm_peak, tc_peak, peak_src = peaks()
    stream = torch.cuda.current_stream()

    # ---- this rank's rows: the reference's nnz-balanced partition
    bounds = S.nnz_balanced_bounds(A.row_ptr, A.rows, A.nnz, world)
    r0, r1 = int(bounds[rank]), int(bounds[rank + 1])
    Ar = S.row_slice(A, r0, r1)
    rows_r = r1 - r0

    dev = torch.device("cuda", local)
    rp = torch.from_numpy(Ar.row_ptr).to(dev)
    ci = torch.from_numpy(Ar.col_idx).to(dev)
    va = torch.from_numpy(Ar.values).to(dev)
    # B: host -> rank 0, then NCCL broadcast over NVLink (timed separately, outside `value`).
    Bd = torch.empty((A.cols, N), dtype=torch.float32, device=dev)
    if rank == 0:
        Bd.copy_(torch.from_numpy(Bh))
    torch.cuda.synchronize()
    bcast_ms = 0.0
    if world > 1:
        warm = torch.zeros(1024, dtype=torch.float32, device=dev)
        dist.broadcast(warm, src=0)  # communicator set-up stays out of the timed broadcast
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dist.broadcast(Bd, src=0)
        e1.record()
        torch.cuda.synchronize()
        bcast_ms = max_over_ranks(e0.elapsed_time(e1))
    Cd = torch.empty((max(rows_r, 1), N), dtype=torch.float32, device=dev)
    view = S.device_view(rows_r, A.cols, rp, ci, va)
    small = cfg_name != "c5"

    # ---- kernel step
    if cfg_name == "c3":
        Ah = S.csr_to_bsr16(A, S.DTYPE_F16)
        brp = torch.from_numpy(Ah.row_ptr).to(dev)
        bci = torch.from_numpy(Ah.col_idx).to(dev)
        bva = torch.from_numpy(Ah.values.view(np.int16)).to(dev)
        B16 = torch.empty((A.cols, N), dtype=torch.float16, device=dev)
        S.convert_f32(Bd, B16, A.cols * N, S.DTYPE_F16, stream)
        bview = S.BsrView(Ah.rows, Ah.cols, Ah.block_rows, Ah.block_cols, Ah.num_blocks, Ah.nnz, S.ptr(brp),
                          S.ptr(bci), S.ptr(bva), S.DTYPE_F16)

        # Inspect A once (the per-CTA schedule of the tensor-core kernel).
        bplan = S.BsrPlan(bview, N, stream=stream)

        def step(s=None):
            bplan.execute(B16, Cd, s or stream)

        launches = 1

        alg_bytes = 512 * Ah.num_blocks + 4 * Ah.num_blocks + 4 * (Ah.block_rows + 1) + 2 * A.cols * N + 4 * A.rows * N
        kernel_name = "bsr_tcgen05_kernel"
    else:
        # Inspect the rank's rows once (picks the work distribution, owns the workspace).
        plan = S.CsrPlan(view, N, stream=stream)
        csr_algo = plan.algo
        launches = plan.k_phases  # kernel launches per step

        def step(s=None):
            plan.execute(Bd, Cd, s or stream)

        # Compulsory bytes of one launch (this rank): A rows + row_ptr + all of B + C rows.
        alg_bytes = 8 * Ar.nnz + 4 * (rows_r + 1) + 4 * A.cols * N + 4 * rows_r * N
        kernel_name = "csr_rowwarp_kernel" if csr_algo == S.CSR_ROWWARP else "csr_merge_kernel"

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev) if small else None

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    code, detail = S.device_error(local)
    if code != 0:
        raise SystemExit(f"device error {code} ({detail}) during warm-up")

    # ---- timed region
    clocks = Clocks(local, enabled=not args.no_clocks)
    clocks.start()
    K = args.steps
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    barrier()
    torch.cuda.synchronize()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record()
    for i in range(K):
        if flush is not None:
            flush.fill_(float(i))  # L2 flush between steps (inputs smaller than L2)
        evs[i][0].record()
        step()
        evs[i][1].record()
    t_end.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    per_launch = [a.elapsed_time(b) for a, b in evs]
    if small:
        region_ms = sum(per_launch)  # flushes excluded
    else:
        region_ms = t_start.elapsed_time(t_end)
    ms_step = max_over_ranks(region_ms / K)
    avg_launch_ms = sum(per_launch) / K
    code, detail = S.device_error(local)
    if code != 0:
        raise SystemExit(f"device error {code} ({detail}) in the timed region")
    value = flops_total / (ms_step * 1e-3) / 1e9

    # ---- end to end through the host-buffer entry point
    e2e = None
    if not args.no_e2e and cfg_name != "c3" and world > 1:
        # Multi-GPU end to end: every rank copies its A rows host -> device; B crosses the
        # host links once in total -- each rank copies 1/N of B's rows and NCCL all-gathers
        # them over NVLink (when N divides B's rows; else rank 0 copies B and broadcasts it,
        # as spmm_multigpu does); every rank runs its plan (spmm_csr_plan_execute) and copies
        # its C rows back.
        pin = lambda a: torch.from_numpy(a).pin_memory()  # noqa: E731
        h_rp, h_ci, h_va = pin(Ar.row_ptr), pin(Ar.col_idx), pin(Ar.values)
        gather_b = A.cols % world == 0
        if gather_b:
            kb = A.cols // world
            h_b = pin(np.ascontiguousarray(Bh[rank * kb:(rank + 1) * kb]))
            b_part = Bd[rank * kb:(rank + 1) * kb]
        else:
            h_b = pin(Bh) if rank == 0 else None
        h_c = torch.empty((max(rows_r, 1), N), dtype=torch.float32).pin_memory()

        def e2e_step():
            rp.copy_(h_rp, non_blocking=True)
            ci.copy_(h_ci, non_blocking=True)
            va.copy_(h_va, non_blocking=True)
            if gather_b:
                b_part.copy_(h_b, non_blocking=True)
                dist.all_gather_into_tensor(Bd, b_part)
            else:
                if rank == 0:
                    Bd.copy_(h_b, non_blocking=True)
                dist.broadcast(Bd, src=0)
            plan.execute(Bd, Cd, stream)
            h_c.copy_(Cd, non_blocking=True)
            torch.cuda.synchronize()

        for _ in range(2):
            e2e_step()
        ke = max(3, min(K, 20))
        barrier()
        t0 = time.perf_counter()
        for _ in range(ke):
            e2e_step()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / ke
        barrier()
        e2e_ms = max_over_ranks(e2e_ms)
        h2d = sum_over_ranks(float(Ar.row_ptr.nbytes + Ar.col_idx.nbytes + Ar.values.nbytes)) + Bh.nbytes
        d2h = sum_over_ranks(float(rows_r * N * 4))
        how = "1/N of B's rows H2D + NCCL all-gather" if gather_b else "B H2D on rank 0 + NCCL broadcast"
        e2e = {"value": round(flops_total / (e2e_ms * 1e-3) / 1e9, 3), "unit": UNIT, "ms_per_step": round(e2e_ms, 4),
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "api": f"per rank: A rows H2D, {how}, spmm_csr_plan_execute, C rows D2H"}
    elif not args.no_e2e and cfg_name != "c3":
        pin = lambda a: torch.from_numpy(a).pin_memory()  # noqa: E731
        hA = S.HostCSR(Ar.rows, Ar.cols, pin(Ar.row_ptr).numpy(), pin(Ar.col_idx).numpy(), pin(Ar.values).numpy())
        hB = pin(Bh).numpy()
        hC = torch.empty((max(rows_r, 1), N), dtype=torch.float32).pin_memory().numpy()
        for _ in range(2):
            S.csr_f32_host(hA, hB, hC, N, csr_algo, stream)
        ke = max(3, min(K, 20))
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(ke):
            S.csr_f32_host(hA, hB, hC, N, csr_algo, stream)
        torch.cuda.synchronize()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / ke
        barrier()
        e2e_ms = max_over_ranks(e2e_ms)
        h2d = sum_over_ranks(float(Ar.row_ptr.nbytes + Ar.col_idx.nbytes + Ar.values.nbytes + Bh.nbytes))
        d2h = sum_over_ranks(float(rows_r * N * 4))
        e2e = {"value": round(flops_total / (e2e_ms * 1e-3) / 1e9, 3), "unit": UNIT, "ms_per_step": round(e2e_ms, 4),
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "api": "spmm_csr_f32_host (C ABI, pinned host buffers)"}

    # ---- roofline of the dominant kernel (per launch, this rank; rank 0 reports)
    achieved = alg_bytes / (avg_launch_ms * 1e-3) / 1e9
    # DRAM bytes per launch from the committed ncu summary of this kernel and config, for this
    # GPU count (a line "dram_bytes_per_launch_gpus<N>: <bytes>"); null when not captured.
    traffic = None
    prof = REPO / "profiles" / f"{kernel_name}_config{cfg_name[1:]}.md"
    if prof.exists():
        key = f"dram_bytes_per_launch_gpus{world}:"
        for line in prof.read_text().splitlines():
            if line.startswith(key):
                traffic = int(line.split(":", 1)[1].strip())
    roofline = {"bound": "hbm", "kernel": kernel_name, "achieved": round(achieved, 1), "peak": hbm_peak,
                "unit": "GB/s", "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else peak_src,
                "alg_bytes_per_launch": int(alg_bytes), "avg_launch_ms": round(avg_launch_ms, 5)}
    if cfg_name == "c3":
        tflops = 2.0 * A.nnz * N / (avg_launch_ms * 1e-3) / 1e12
        roofline["tensor"] = {"achieved_tflops": round(tflops, 2), "peak_tflops": tc_peak,
                              "frac": round(tflops / tc_peak, 4)}
    else:
        gathered = 4.0 * Ar.nnz * N  # B-row bytes the gather moves through L2 per launch
        gather_gbs = gathered / (avg_launch_ms * 1e-3) / 1e9
        roofline["l2_gather_gbs"] = round(gather_gbs, 1)
        # The ceiling that bounds a gather of whole B rows: a load-only probe that pulls random
        # 1 KB rows into the SMs from an L2-resident 32 MB part of B (the fastest any gather can
        # go), and the same probe over B's whole footprint (uniformly random rows, so it misses
        # L2 more often than the kernel, whose warps walk their sorted columns together).
        resident = gather_ceiling(torch, Bd, min(A.cols, 32768), Ar.nnz, stream)
        same = gather_ceiling(torch, Bd, A.cols, Ar.nnz, stream)
        if resident:
            roofline["gather_ceiling"] = {
                "achieved_gbs": round(gather_gbs, 1), "ceiling_gbs": round(resident, 1),
                "frac": round(gather_gbs / resident, 4), "same_footprint_probe_gbs": round(same or 0.0, 1),
                "probe": "load-only random 1 KB B-row fetches, L2-resident 32 MB (lib/libspmm_probe.so)"}

    # ---- µs-scale configs: a CUDA graph of 100 back-to-back launches (no flush in between, so
    # the inputs stay in L2), the launch-overhead-free figure for kernels of a few µs.
    graph = None
    if small and world == 1:
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
            graph = {"launches": 100, "us_per_launch": round(us, 3),
                     "value": round(flops_total / (us * 1e-6) / 1e9, 1), "unit": UNIT,
                     "l2": "warm (no flush between launches)"}
            del g
        except Exception as e:  # noqa: BLE001 - reported, not fatal
            graph = {"error": str(e)[:200]}
        code, detail = S.device_error(local)
        if code != 0:
            raise SystemExit(f"device error {code} ({detail}) in the graph batch")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gf, threads, med = cpu_baseline_run(A, Bh, steps=3, warmup=1)
        cpu = {"value": round(gf, 3), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"full {cfg_name} product, median of 3 (OpenMP static over rows, {med*1e3:.0f} ms each)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp16" if cfg_name == "c3" else "f32",
            "data": "synthetic (reference generators, fixed seeds)",
            "config": {"workload": CONFIGS[cfg_name], "config_id": cfg_name, "nnz": total_nnz, "N": N,
                       "rows": A.rows, "cols": A.cols, "parallelism": f"row-split x{world} (nnz-balanced)",
                       "kernel": kernel_name,
                       "l2": "inputs larger than L2" if not small else "L2 flushed between steps",
                       "b_broadcast_ms": round(bcast_ms, 4)},
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk, "gpu_launches": K * launches,
            "graph_batch": graph,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args, rank: int, world: int):
    """The reference semantics on the host cores; rank 0 only."""
    if rank != 0:
        return
    A, Bh = build_inputs(args.config)
    # Keep the whole run within ~150 s of CPU time: time one full product, and if the requested
    # steps would exceed that, time each step on the leading rows only (same rate metric).
    import spmm_b200 as S

    _, threads, one = cpu_baseline_run(A, Bh, steps=1, warmup=0)
    sample = f"full {args.config} product per step (OpenMP static over rows)"
    budget = 150.0
    if (args.steps + args.warmup) * one > budget:
        frac = max(budget / ((args.steps + args.warmup) * one), 1e-3)
        rows = max(1, int(A.rows * frac))
        A = S.row_slice(A, 0, rows)
        sample = f"rows 0..{rows} of {args.config} ({100 * frac:.1f} % of the product) per step, OpenMP static"
    gf, threads, med = cpu_baseline_run(A, Bh, steps=args.steps, warmup=args.warmup)
    line = {
        "metric": METRIC, "value": round(gf, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(med * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (reference generators, fixed seeds)",
        "config": {"workload": CONFIGS[args.config], "config_id": args.config, "nnz": A.nnz, "N": Bh.shape[1]},
        "impl": "reference",
        "cpu_baseline": {"value": round(gf, 3), "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(gf, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
