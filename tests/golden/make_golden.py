#!/usr/bin/env python3
"""Regenerates tests/golden/golden.json from the reference itself (build container only).

Sources, none of which exist on the GPU box (the JSON is committed instead):
  * the reference's scripts/gen_matrices.py, imported read-only (no bytecode is written
    next to it), for the pattern configs C2-C4 and small pattern cases;
  * the reference's own C++ host code compiled into oracle/_ref/libref.so (csr.cu
    generator, bsr.cu conversion, nnz_balanced_bounds, harness generate_dense_row_major);
  * the known-answer tables the reference publishes in its docs (copied as numbers):
    scripts/roofline.py:59-154 (nnz per sweep cell), reports/tensor_core_wmma.md:43-56
    (BSR block counts), README.md:233 (4096^2 d=0.01 -> 167686).

Usage:  python tests/golden/make_golden.py --ref <reference checkout>
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.dont_write_bytecode = True

# Known answers published by the reference (seed 42, m = k, n = 256).
SWEEP_NNZ = {  # scripts/roofline.py:59-154
    "1024/0.05": 52260, "1024/0.01": 10388, "1024/0.001": 1044,
    "4096/0.05": 839236, "4096/0.01": 167686, "4096/0.001": 16935,
    "8192/0.05": 3354625, "8192/0.01": 671114, "8192/0.001": 67137,
    "16384/0.05": 13421456, "16384/0.01": 2684748, "16384/0.001": 268160,
}
BSR_TABLE = {  # reports/tensor_core_wmma.md:43-56: blocks, stored elements, fill-in, block density
    "1024/0.05": [4096, 1048576, 20.1, 1.000], "1024/0.01": [3761, 962816, 92.7, 0.918],
    "1024/0.001": [917, 234752, 224.9, 0.224], "4096/0.05": [65536, 16777216, 20.0, 1.000],
    "4096/0.01": [60630, 15521280, 92.6, 0.925], "4096/0.001": [14924, 3820544, 225.6, 0.228],
    "8192/0.05": [262144, 67108864, 20.0, 1.000], "8192/0.01": [242248, 62015488, 92.4, 0.924],
    "8192/0.001": [59324, 15186944, 226.2, 0.226], "16384/0.05": [1048574, 268434944, 20.0, 1.000],
    "16384/0.01": [968648, 247973888, 92.4, 0.924], "16384/0.001": [236629, 60577024, 225.9, 0.226],
}


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def load_gen_matrices(ref: Path):
    spec = importlib.util.spec_from_file_location("ref_gen_matrices", ref / "scripts" / "gen_matrices.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


PATTERN_CASES = {
    # name: (pattern, rows, cols, kwargs) -- C2, C3, C4 and small variants with ragged edges
    "c2_banded_8192_bw41": ("banded", 8192, 8192, {"bandwidth": 41}),
    "c3_blockdiag_8192_b128": ("block-diagonal", 8192, 8192, {"block": 128}),
    "c4_powerlaw_16384_m164_a1.8": ("power-law", 16384, 16384, {"mean_deg": 164.0, "alpha": 1.8}),
    "banded_1000x900_bw7": ("banded", 1000, 900, {"bandwidth": 7}),
    "blockdiag_300x250_b32": ("block-diagonal", 300, 250, {"block": 32}),
    "powerlaw_777x512_m9_a2.5": ("power-law", 777, 512, {"mean_deg": 9.0, "alpha": 2.5}),
    "uniform_mask_300x200_d0.05": ("uniform", 300, 200, {"density": 0.05}),
}


def pattern_csr(gm, pattern, rows, cols, kw, seed=42):
    rng = np.random.default_rng(seed)
    if pattern == "banded":
        r, c, v = gm.gen_banded(rows, cols, kw["bandwidth"], rng)
    elif pattern == "block-diagonal":
        r, c, v = gm.gen_block_diagonal(rows, cols, kw["block"], rng)
    elif pattern == "power-law":
        r, c, v = gm.gen_power_law(rows, cols, kw["mean_deg"], kw["alpha"], rng)
    else:
        r, c, v = gm.gen_uniform(rows, cols, kw["density"], rng)
    return gm.coo_to_csr(rows, cols, r, c, v)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", type=Path, required=True, help="the reference checkout (its top directory)")
    args = ap.parse_args()
    gm = load_gen_matrices(args.ref)
    from oracle import oracle as O

    out = {"sweep_nnz": SWEEP_NNZ, "bsr_table": BSR_TABLE, "readme_nnz_4096_0.01": 167686, "patterns": {},
           "uniform_csr": {}, "dense": {}, "bounds": {}, "bsr": {}, "small_product": {}}

    for name, (pattern, rows, cols, kw) in PATTERN_CASES.items():
        rp, ci, v = pattern_csr(gm, pattern, rows, cols, kw)
        out["patterns"][name] = {"pattern": pattern, "rows": rows, "cols": cols, "kw": kw, "seed": 42,
                                 "nnz": int(v.size), "max_row": int(np.diff(rp).max()),
                                 "sha256": digest(rp.astype("<i4"), ci.astype("<i4"), v.astype("<f4"))}

    if not O.ref_available():
        raise SystemExit("oracle/_ref/libref.so is missing: run `make -C oracle ref` first")
    for rows, cols, d, seed in [(4096, 4096, 0.01, 42), (1000, 777, 0.03, 7), (64, 64, 1.0, 1), (50, 80, 0.0, 3),
                                (3000, 5000, 0.002, 42)]:
        A = O.ref_gen_uniform_csr(rows, cols, d, seed)
        out["uniform_csr"][f"{rows}x{cols}/{d}/{seed}"] = {
            "nnz": A.nnz, "sha256": digest(A.row_ptr, A.col_idx, A.values)}
        if rows == 4096:
            for G in (1, 2, 3, 4, 5, 7, 8):
                out["bounds"][f"4096x4096/0.01/42/G{G}"] = O.ref_nnz_balanced_bounds(A, G).tolist()
            b, st = O.ref_bsr_from_csr(A)
            out["bsr"]["4096x4096/0.01/42"] = {"stats": st, "sha256": digest(b.row_ptr, b.col_idx, b.values)}
    for name in ("banded_1000x900_bw7", "blockdiag_300x250_b32", "powerlaw_777x512_m9_a2.5"):
        pattern, rows, cols, kw = PATTERN_CASES[name]
        rp, ci, v = pattern_csr(gm, pattern, rows, cols, kw)
        b, st = O.ref_bsr_from_csr(O.CSR(rows, cols, rp.astype(np.int32), ci.astype(np.int32), v.astype(np.float32)))
        out["bsr"][name] = {"stats": st, "sha256": digest(b.row_ptr, b.col_idx, b.values)}
    for rows, cols, seed in [(4096, 64, 43), (8192, 128, 43), (123, 45, 9)]:
        out["dense"][f"{rows}x{cols}/{seed}"] = digest(O.ref_gen_dense(rows, cols, seed))

    # A small product fixture: A (40 x 30, d = 0.2, seed 7), B (30 x 8, seed 8), C.
    A = O.ref_gen_uniform_csr(40, 30, 0.2, 7)
    B = O.ref_gen_dense(30, 8, 8)
    Cm = O.spmm_csr_f32(A, B)
    out["small_product"] = {"rows": 40, "cols": 30, "N": 8, "row_ptr": A.row_ptr.tolist(),
                            "col_idx": A.col_idx.tolist(), "values_hex": [float(x).hex() for x in A.values],
                            "B_hex": [float(x).hex() for x in B.ravel()],
                            "C_hex": [float(x).hex() for x in Cm.ravel()]}
    (HERE / "golden.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print(f"wrote {HERE / 'golden.json'}")


if __name__ == "__main__":
    main()
