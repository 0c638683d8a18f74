"""TEST INFRASTRUCTURE ONLY -- not part of the product.

Seeded sparsity-pattern generators used to build the BASELINE configs C2-C4 (and small
parity cases). They restate the generators of the reference's ``scripts/gen_matrices.py``
(banded :37-48, block-diagonal :51-63, power-law :66-81, dense-mask uniform :30-34) and its
COO->CSR step (:84-91): the same numpy ``Generator`` calls in the same order, so a given
seed yields the same matrix. Only tests/, ``__graft_entry__.smoke()`` and bench.py's setup
may import this module; the product never does.

Pinned by tests/test_oracle_golden.py against SHA-256 digests of the reference script's own
output (tests/golden/make_golden.py imports the reference script in the build container and
records the digests).
"""
from __future__ import annotations

import numpy as np


def _csr_from_triplets(rows: int, r: np.ndarray, c: np.ndarray, v: np.ndarray):
    """Sort triplets by (row, col) with a stable lexsort and build row_ptr by counting."""
    order = np.lexsort((c, r))
    r = r[order]
    c = c[order].astype(np.int32)
    v = v[order].astype(np.float32)
    counts = np.bincount(r, minlength=rows)[:rows]
    row_ptr = np.zeros(rows + 1, dtype=np.int32)
    np.cumsum(counts, out=row_ptr[1:])
    return row_ptr, c, v


def uniform_mask(rows: int, cols: int, density: float, seed: int):
    """Dense Bernoulli mask (only feasible for small shapes)."""
    rng = np.random.default_rng(seed)
    keep = rng.random((rows, cols)) < density
    r, c = np.nonzero(keep)
    v = rng.uniform(-1.0, 1.0, size=r.size).astype(np.float32)
    return _csr_from_triplets(rows, r.astype(np.int64), c.astype(np.int32), v)


def banded(rows: int, cols: int, bandwidth: int, seed: int):
    """Nonzeros exactly where |i - j| <= bandwidth; values U(-1, 1) in row-major order."""
    rng = np.random.default_rng(seed)
    i = np.arange(rows, dtype=np.int64)
    lo = np.maximum(0, i - bandwidth)
    hi = np.minimum(cols, i + bandwidth + 1)
    lens = np.maximum(hi - lo, 0)
    r = np.repeat(i, lens)
    starts = np.repeat(lo - np.concatenate(([0], np.cumsum(lens)[:-1])), lens)
    c = (np.arange(r.size, dtype=np.int64) + starts).astype(np.int32)
    v = rng.uniform(-1.0, 1.0, size=r.size).astype(np.float32)
    return _csr_from_triplets(rows, r, c, v)


def block_diagonal(rows: int, cols: int, block: int, seed: int):
    """min(rows, cols) // block dense block x block squares on the diagonal."""
    rng = np.random.default_rng(seed)
    nblk = min(rows, cols) // block
    local = np.arange(block, dtype=np.int64)
    rr, cc = np.meshgrid(local, local, indexing="ij")
    base = (np.arange(nblk, dtype=np.int64) * block)[:, None]
    r = (base + rr.ravel()[None, :]).ravel()
    c = (base + cc.ravel()[None, :]).ravel().astype(np.int32)
    v = rng.uniform(-1.0, 1.0, size=r.size).astype(np.float32)
    return _csr_from_triplets(rows, r, c, v)


def power_law(rows: int, cols: int, mean_deg: float, alpha: float, seed: int):
    """Pareto(alpha)+1 degrees rescaled to mean_deg, rounded and clipped to [1, cols];
    each row picks its columns uniformly without replacement (one ``choice`` per row, in
    row order); values U(-1, 1) drawn last, in generation order."""
    rng = np.random.default_rng(seed)
    raw = rng.pareto(alpha, size=rows) + 1.0
    raw = raw * (mean_deg / raw.mean())
    deg = np.clip(np.round(raw).astype(np.int64), 1, cols)
    picks = [rng.choice(cols, size=int(d), replace=False) for d in deg]
    r = np.repeat(np.arange(rows, dtype=np.int64), deg)
    c = np.concatenate(picks).astype(np.int32) if picks else np.zeros(0, np.int32)
    v = rng.uniform(-1.0, 1.0, size=r.size).astype(np.float32)
    return _csr_from_triplets(rows, r, c, v)


def make(pattern: str, rows: int, cols: int, seed: int = 42, **kw):
    if pattern == "uniform":
        return uniform_mask(rows, cols, kw.get("density", 0.01), seed)
    if pattern == "banded":
        return banded(rows, cols, kw.get("bandwidth", 16), seed)
    if pattern == "block-diagonal":
        return block_diagonal(rows, cols, kw.get("block", 32), seed)
    if pattern == "power-law":
        return power_law(rows, cols, kw.get("mean_deg", 16.0), kw.get("alpha", 2.5), seed)
    raise ValueError(f"unknown pattern {pattern!r}")
