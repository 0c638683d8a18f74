#!/usr/bin/env python3
"""B200 pattern x size sweep of the SpMM engine (the B200 counterpart of the reference's
scripts/run_pattern_sweep.py:46-151 and scripts/roofline.py:177-212).

For every case it times the CUDA-core CSR kernel (both work distributions) and the
tensor-core BSR kernel on the same matrix, records the BSR fill-in, the hybrid rule's choice
at the given threshold, GFLOP/s = 2*nnz*N/t, and the fraction of the HBM roofline under the
reference's compulsory-byte model (8*nnz + 4(M+1) + 4*K*N + 4*M*N for CSR; 516*blocks +
4(block_rows+1) + 2*K*N + 4*M*N for BSR), against the measured B200 peak. The measured
CSR/TC crossover in fill-in is what the hybrid threshold is set from.

    python sparse-matrix-multiplication_b200/sweep.py --out sweep.csv [--quick] [--n 256]

Times are CUDA-event medians of single launches with a 256 MiB L2 flush in between.

    python sparse-matrix-multiplication_b200/sweep.py --pattern-sweep --out pattern_sweep.csv [--dry-run]

runs the reference's own cross-pattern grid (scripts/run_pattern_sweep.py: uniform d=0.01,
banded bandwidth 32, block-diagonal block 16, power-law mean degree 32 alpha 2.5; m = 1024, 4096,
8192, 16384; N = 256; seed 42, the same generator call sequence) and writes the reference's tidy
CSV, one row per (pattern, size, kernel) with exactly its columns
(pattern,kernel,m,k,n,nnz,density,time_ms,gflops). Kernels: csr_rowwarp, csr_merge, bsr16_tc
(tcgen05, FP16) and hybrid[<choice>] (the hybrid rule's pick at --threshold). --dry-run builds
the matrices on the CPU and writes the rows without timings.

    python sparse-matrix-multiplication_b200/sweep.py --roofline-from pattern_sweep.csv --out roofline.csv

turns such a CSV into the reference's roofline table (scripts/roofline.py:177-212: compulsory
DRAM bytes 8*nnz + 4(m+1) + 4*k*n + 4*m*n, AI, ceiling min(FP32 peak, AI * DRAM bandwidth), % of
FP32 peak, % of the ceiling, effective DRAM bandwidth, bound, B_fits_L2) with B200 ceilings: the
measured HBM bandwidth (MEASURED_PEAKS.json), the FP32 CUDA-core peak (148 SMs x 128 lanes x
2 FLOP x the maximum SM clock) and the 126 MB L2. CPU only.

    python sparse-matrix-multiplication_b200/sweep.py --gather-footprints --out gather.csv

instead measures the gather ceiling that bounds the FP32 CSR kernels: for B footprints from 8 MB
to 512 MB (N = 256, so one B row is 1 KB) it times the load-only random-row probe
(lib/libspmm_probe.so) and the planned CSR kernel on a 131072-row uniform matrix with 131
nonzeros per row over that many columns (the fast generator), and reports both as GB/s of
gathered B rows.
"""
from __future__ import annotations

import argparse
import csv
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import spmm_b200 as S  # noqa: E402
import spmm_patterns as SP  # noqa: E402


def peak_hbm_gbs() -> float:
    f = HERE.parent / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(f.read_text())["hbm_gbs"])
    except (OSError, ValueError, KeyError):
        return 6650.0


def cases(quick: bool):
    sizes = (4096, 8192) if quick else (1024, 4096, 8192, 16384)
    for m in sizes:  # the reference's uniform sweep grid (scripts/roofline.py:59-154)
        for d in (0.05, 0.01, 0.001):
            if quick and d == 0.05 and m > 4096:
                continue
            yield f"uniform_{m}_d{d}", lambda m=m, d=d: S.generate_uniform_csr(m, m, d, 42)
    for bw in ((2, 8, 41) if quick else (1, 2, 4, 8, 16, 41, 64)):
        yield f"banded_8192_bw{bw}", lambda bw=bw: SP.host_csr(8192, 8192, SP.banded_arrays(8192, 8192, bw, 42))
    for blk in ((8, 16, 128) if quick else (4, 8, 12, 16, 32, 64, 128)):
        yield f"blockdiag_8192_b{blk}", lambda blk=blk: SP.host_csr(8192, 8192, SP.block_diagonal_arrays(8192, 8192, blk, 42))
    yield "powerlaw_16384", lambda: SP.host_csr(16384, 16384, SP.power_law_arrays(16384, 16384, 164.0, 1.8, 42))


# The reference's cross-pattern grid (scripts/run_pattern_sweep.py:46-51 generator parameters,
# :92-93 sizes, :94 N) and its CSV columns (:147); the roofline table's columns
# (scripts/roofline.py:236-239).
PATTERN_PARAMS = {"uniform": {"density": 0.01}, "banded": {"bandwidth": 32}, "block-diagonal": {"block": 16},
                  "power-law": {"mean_deg": 32.0, "alpha": 2.5}}
PATTERN_SIZES = (1024, 4096, 8192, 16384)
PATTERN_SWEEP_COLUMNS = ["pattern", "kernel", "m", "k", "n", "nnz", "density", "time_ms", "gflops"]
ROOFLINE_COLUMNS = ["kernel", "m", "density", "nnz", "gflops", "ai_flop_per_byte", "ceiling_gflops", "pct_fp32_peak",
                    "pct_roofline", "eff_dram_bw_gbs", "pct_dram_bw", "bound", "B_fits_L2"]
B200_SMS = 148
B200_L2_BYTES = 126 * 1024 * 1024
FP32_LANES_PER_SM = 128


def pattern_matrix(pattern: str, m: int, seed: int = 42) -> S.HostCSR:
    """An m x m matrix of one of the reference's sweep patterns (gen_matrices.py's call sequence)."""
    kw = PATTERN_PARAMS[pattern]
    if pattern == "uniform":
        arrays = SP.uniform_mask_arrays(m, m, kw["density"], seed)
    elif pattern == "banded":
        arrays = SP.banded_arrays(m, m, kw["bandwidth"], seed)
    elif pattern == "block-diagonal":
        arrays = SP.block_diagonal_arrays(m, m, kw["block"], seed)
    else:
        arrays = SP.power_law_arrays(m, m, kw["mean_deg"], kw["alpha"], seed)
    return SP.host_csr(m, m, arrays)


def b200_ceilings() -> tuple[float, float, int]:
    """(FP32 CUDA-core peak GFLOP/s, DRAM GB/s, L2 bytes): the peak from the SM count and the
    maximum SM clock, the bandwidth measured by the driver (MEASURED_PEAKS.json)."""
    mhz = 1965.0
    try:
        mhz = float(json.loads((HERE.parent / "MEASURED_PEAKS.json").read_text()).get("sm_max_mhz", mhz))
    except (OSError, ValueError):
        pass
    return B200_SMS * FP32_LANES_PER_SM * 2 * mhz / 1e3, peak_hbm_gbs(), B200_L2_BYTES


def roofline_rows(rows, fp32_gflops: float, dram_gbs: float, l2_bytes: int) -> list[dict]:
    """The reference's roofline analysis (scripts/roofline.py:177-212) of sweep rows with the
    given ceilings: compulsory bytes, AI, min(peak, AI * bandwidth), the percentages, the bound."""
    ridge = fp32_gflops / dram_gbs
    out = []
    for r in rows:
        m, k, n, nnz = int(r["m"]), int(r["k"]), int(r["n"]), int(r["nnz"])
        t = float(r["time_ms"])
        gflops = float(r["gflops"])
        flops = 2.0 * nnz * n
        dram = 8 * nnz + 4 * (m + 1) + 4 * k * n + 4 * m * n
        ai = flops / dram
        ceiling = min(fp32_gflops, ai * dram_gbs)
        eff = dram / (t * 1e6)
        out.append({"kernel": r["kernel"], "m": m, "density": float(r.get("density") or nnz / (m * k)), "nnz": nnz,
                    "gflops": gflops, "ai_flop_per_byte": ai, "ceiling_gflops": ceiling,
                    "pct_fp32_peak": 100.0 * gflops / fp32_gflops, "pct_roofline": 100.0 * gflops / ceiling,
                    "eff_dram_bw_gbs": eff, "pct_dram_bw": 100.0 * eff / dram_gbs,
                    "bound": "compute/L2" if ai > ridge else "memory", "B_fits_L2": 4 * k * n <= l2_bytes,
                    "pattern": r.get("pattern", "")})
    return out


def roofline_from(args) -> None:
    with open(args.roofline_from, newline="") as fh:
        # Timed rows only (a dry run leaves time_ms and gflops empty).
        rows = [r for r in csv.DictReader(fh) if r.get("time_ms") and r.get("gflops") and float(r["time_ms"]) > 0]
    fp32, dram, l2 = b200_ceilings()
    res = roofline_rows(rows, fp32, dram, l2)
    with open(args.out, "w", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=ROOFLINE_COLUMNS, extrasaction="ignore")
        w.writeheader()
        w.writerows(res)
    print(f"B200 ceilings: FP32 {fp32:.0f} GFLOP/s | DRAM {dram:.0f} GB/s | ridge {fp32 / dram:.1f} FLOP/byte | "
          f"L2 {l2 // (1024 * 1024)} MB")
    for r in res:
        print(f"{r['pattern']:>15} {r['kernel']:>14} m={r['m']:<6d} AI {r['ai_flop_per_byte']:6.1f} "
              f"{r['gflops']:9.1f} GFLOP/s  {r['pct_roofline']:5.1f}% of roof  {r['pct_dram_bw']:5.1f}% of DRAM")


def pattern_sweep(args) -> None:
    """The reference's cross-pattern grid on this engine (see the module docstring)."""
    rows = []
    timer = None
    if not args.dry_run:
        import torch

        torch.cuda.set_device(0)
        dev = torch.device("cuda", 0)
        stream = torch.cuda.current_stream()
        flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
        timer = (torch, dev, stream, flush)
    N = args.n
    sizes = [m for m in PATTERN_SIZES if m <= args.max_size]
    with open(args.out, "w", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=PATTERN_SWEEP_COLUMNS, extrasaction="ignore")
        w.writeheader()
        for pattern in args.patterns or list(PATTERN_PARAMS):
            for m in sizes:
                A = pattern_matrix(pattern, m)
                base = {"pattern": pattern, "m": m, "k": m, "n": N, "nnz": A.nnz, "density": A.nnz / (m * m)}
                choice = S.hybrid_choose(A, N, args.threshold)["backend_name"]
                if timer is None:
                    times = {"csr_rowwarp": None, "csr_merge": None, "bsr16_tc": None}
                else:
                    times = time_pattern_case(timer, A, N, args.reps)
                times[f"hybrid[{choice}]"] = (times["bsr16_tc"] if choice == "wmma"
                                              else min(times["csr_rowwarp"], times["csr_merge"])
                                              if times["csr_rowwarp"] is not None else None)
                for kernel, t in times.items():
                    row = {**base, "kernel": kernel, "time_ms": "" if t is None else round(t, 5),
                           "gflops": "" if t is None else round(2.0 * A.nnz * N / (t * 1e-3) / 1e9, 2)}
                    rows.append(row)
                    w.writerow(row)
                fh.flush()
                print(json.dumps({k: base[k] for k in ("pattern", "m", "nnz")} | {"times_ms": times}), flush=True)
    if timer is not None:
        code, detail = S.device_error(0)
        if code:
            raise SystemExit(f"device error {code} ({detail})")


def time_pattern_case(timer, A: S.HostCSR, N: int, reps: int) -> dict:
    torch, dev, stream, flush = timer
    M, K = A.rows, A.cols
    Bh = S.generate_dense(K, N, 43)
    rp, ci, v = (torch.from_numpy(x).to(dev) for x in (A.row_ptr, A.col_idx, A.values))
    B = torch.from_numpy(Bh).to(dev)
    C = torch.empty((M, N), device=dev)
    view = S.device_view(M, K, rp, ci, v)
    out = {"csr_rowwarp": time_ms(torch, lambda: S.csr_f32(view, B, C, N, S.CSR_ROWWARP, stream), reps, flush),
           "csr_merge": time_ms(torch, lambda: S.csr_f32(view, B, C, N, S.CSR_MERGE, stream), reps, flush)}
    bview, keep = S.csr_to_bsr16_device(view, S.DTYPE_F16, stream)
    B16 = torch.empty((K, N), dtype=torch.float16, device=dev)
    S.convert_f32(B, B16, K * N, S.DTYPE_F16, stream)
    bplan = S.BsrPlan(bview, N, stream=stream)
    out["bsr16_tc"] = time_ms(torch, lambda: bplan.execute(B16, C, stream), reps, flush)
    bplan.close()
    del keep
    return out


def time_ms(torch, fn, reps: int, flush) -> float:
    fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        flush.fill_(1.0)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return float(np.median(ts))


def gather_footprints(args) -> None:
    import ctypes as C

    import torch

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream()
    probe = C.CDLL(str(HERE / "lib" / "libspmm_probe.so"))
    probe.spmm_probe_gather.argtypes = [C.c_void_p, C.c_uint32, C.c_longlong, C.c_uint32, C.c_void_p, C.c_void_p]
    ctas = C.c_int()
    if probe.spmm_probe_ctas(C.byref(ctas)) != 0:
        raise SystemExit("spmm_probe_ctas failed")
    out = torch.empty(ctas.value * 256, dtype=torch.float32, device=dev)
    M, N, per_row = 131072, 256, 131
    fields = ["footprint_mb", "cols", "nnz", "probe_ms", "probe_gbs", "csr_ms", "csr_gbs", "csr_frac_of_probe",
              "csr_gflops", "k_phases", "phased_k", "phased_ms"]
    with open(args.out, "w", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=fields)
        w.writeheader()
        for mb in (8, 16, 32, 48, 64, 80, 96, 112, 128, 160, 256, 512):
            K = mb * 1024
            A = S.generate_uniform_csr_fast(M, K, per_row / K, 42)
            Bd = torch.empty((K, N), dtype=torch.float32, device=dev).uniform_(-1, 1)
            rp, ci, v = (torch.from_numpy(x).to(dev) for x in (A.row_ptr, A.col_idx, A.values))
            Cd = torch.empty((M, N), dtype=torch.float32, device=dev)
            view = S.device_view(M, K, rp, ci, v)
            plan = S.CsrPlan(view, N, stream=stream)

            def run_probe(i=[0]):
                i[0] += 1
                rc = probe.spmm_probe_gather(C.c_void_p(Bd.data_ptr()), K, A.nnz - A.nnz % 4, i[0],
                                             C.c_void_p(out.data_ptr()), C.c_void_p(stream.cuda_stream))
                if rc:
                    raise SystemExit(f"probe failed ({rc})")

            def back_to_back(fn, reps=9):
                fn()
                torch.cuda.synchronize()
                ts = []
                for _ in range(reps):
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    fn()
                    b.record()
                    torch.cuda.synchronize()
                    ts.append(a.elapsed_time(b))
                return float(np.median(ts))

            pm = back_to_back(run_probe)
            cm = back_to_back(lambda: plan.execute(Bd, Cd, stream))
            ph, phm = 1, None
            if mb > 96:  # column phases sized to ~64 MB of B each
                ph = min(8, -(-mb // 64))
                pplan = S.CsrPlan(view, N, tuning=S.CsrTuning(k_phases=ph), stream=stream)
                phm = back_to_back(lambda: pplan.execute(Bd, Cd, stream))
                pplan.close()
            pg = (A.nnz - A.nnz % 4) * 1024 / (pm * 1e-3) / 1e9
            cg = A.nnz * 1024 / (cm * 1e-3) / 1e9
            row = {"footprint_mb": mb, "cols": K, "nnz": A.nnz, "probe_ms": round(pm, 4), "probe_gbs": round(pg, 1),
                   "csr_ms": round(cm, 4), "csr_gbs": round(cg, 1), "csr_frac_of_probe": round(cg / pg, 4),
                   "csr_gflops": round(2.0 * A.nnz * N / (cm * 1e-3) / 1e9, 1), "k_phases": plan.k_phases,
                   "phased_k": ph, "phased_ms": round(phm, 4) if phm else ""}
            w.writerow(row)
            fh.flush()
            print(json.dumps(row), flush=True)
            plan.close()
            del Bd, Cd, rp, ci, v
    code, detail = S.device_error(0)
    if code:
        raise SystemExit(f"device error {code} ({detail})")


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out", type=Path, required=True)
    ap.add_argument("--n", type=int, default=256)
    ap.add_argument("--reps", type=int, default=15)
    ap.add_argument("--threshold", type=float, default=0.0, help="hybrid fill-in threshold (0 = library default)")
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--gather-footprints", action="store_true",
                    help="probe vs CSR kernel gather rate over B footprints (see above)")
    ap.add_argument("--pattern-sweep", action="store_true", help="the reference's cross-pattern grid (see above)")
    ap.add_argument("--patterns", nargs="+", default=None, choices=sorted(PATTERN_PARAMS))
    ap.add_argument("--max-size", type=int, default=max(PATTERN_SIZES), help="largest m of the pattern grid")
    ap.add_argument("--dry-run", action="store_true", help="pattern sweep: build the matrices, no GPU, no timings")
    ap.add_argument("--roofline-from", type=Path, default=None, help="pattern-sweep CSV to analyse (CPU only)")
    args = ap.parse_args()
    if args.gather_footprints:
        gather_footprints(args)
        return
    if args.roofline_from is not None:
        roofline_from(args)
        return
    if args.pattern_sweep:
        pattern_sweep(args)
        return

    import torch

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream()
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    hbm = peak_hbm_gbs()
    N = args.n
    fields = ["case", "rows", "cols", "n", "nnz", "fill_in", "block_density", "num_blocks", "hybrid_choice",
              "csr_merge_ms", "csr_rowwarp_ms", "tc_ms", "csr_gflops", "tc_gflops", "csr_pct_hbm_roofline",
              "tc_pct_hbm_roofline", "tc_rel_l2_vs_csr", "faster"]
    with open(args.out, "w", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=fields)
        w.writeheader()
        for name, make in cases(args.quick):
            A = make()
            M, K = A.rows, A.cols
            Bh = S.generate_dense(K, N, 43)
            rp, ci, v = (torch.from_numpy(x).to(dev) for x in (A.row_ptr, A.col_idx, A.values))
            B = torch.from_numpy(Bh).to(dev)
            C = torch.empty((M, N), device=dev)
            view = S.device_view(M, K, rp, ci, v)
            merge = time_ms(torch, lambda: S.csr_f32(view, B, C, N, S.CSR_MERGE, stream), args.reps, flush)
            rowwarp = time_ms(torch, lambda: S.csr_f32(view, B, C, N, S.CSR_ROWWARP, stream), args.reps, flush)
            Ccsr = C.clone()
            bview, keep = S.csr_to_bsr16_device(view, S.DTYPE_F16, stream)
            B16 = torch.empty((K, N), dtype=torch.float16, device=dev)
            S.convert_f32(B, B16, K * N, S.DTYPE_F16, stream)
            bplan = S.BsrPlan(bview, N, stream=stream)  # the hybrid times the planned kernel
            tc = time_ms(torch, lambda: bplan.execute(B16, C, stream), args.reps, flush)
            bplan.close()
            rel = float(torch.linalg.norm(C - Ccsr) / max(float(torch.linalg.norm(Ccsr)), 1e-30))
            nb = bview.num_blocks
            plan = S.hybrid_choose(A, N, args.threshold)
            flops = 2.0 * A.nnz * N
            csr_ms = min(merge, rowwarp)
            csr_bytes = 8 * A.nnz + 4 * (M + 1) + 4 * K * N + 4 * M * N
            tc_bytes = 516 * nb + 4 * ((M + 15) // 16 + 1) + 2 * K * N + 4 * M * N
            row = {"case": name, "rows": M, "cols": K, "n": N, "nnz": A.nnz,
                   "fill_in": round(256.0 * nb / max(A.nnz, 1), 4), "block_density": round(plan["block_density"], 5),
                   "num_blocks": nb, "hybrid_choice": plan["backend_name"], "csr_merge_ms": round(merge, 5),
                   "csr_rowwarp_ms": round(rowwarp, 5), "tc_ms": round(tc, 5),
                   "csr_gflops": round(flops / csr_ms / 1e6, 1), "tc_gflops": round(flops / tc / 1e6, 1),
                   "csr_pct_hbm_roofline": round(100 * csr_bytes / (csr_ms * 1e-3) / 1e9 / hbm, 2),
                   "tc_pct_hbm_roofline": round(100 * tc_bytes / (tc * 1e-3) / 1e9 / hbm, 2),
                   "tc_rel_l2_vs_csr": f"{rel:.3e}", "faster": "tc" if tc < csr_ms else "csr"}
            w.writerow(row)
            fh.flush()
            print(json.dumps(row), flush=True)
            del keep
    code, detail = S.device_error(0)
    if code:
        raise SystemExit(f"device error {code} ({detail})")


if __name__ == "__main__":
    main()
