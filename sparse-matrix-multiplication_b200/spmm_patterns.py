"""Seeded sparsity patterns of the engine's benchmark configs (product side).

Produces the same matrices as the reference's scripts/gen_matrices.py for a given seed --
banded (:37-48), block-diagonal (:51-63), power-law (:66-81), dense-mask uniform (:30-34),
COO->CSR (:84-91) -- because BASELINE configs 2-4 are defined by that script. The numpy
Generator call sequence is the one the script makes (it decides the values); the index
construction is vectorised. The mt19937 uniform generator of configs 1 and 5 is the C entry
point spmm_generate_uniform_csr.

Returns HostCSR objects of spmm_b200 and, for tests, plain arrays.
"""
from __future__ import annotations

import numpy as np


def _to_csr(rows: int, r: np.ndarray, c: np.ndarray, v: np.ndarray):
    # Stable sort by (row, col), then row counts -> row_ptr.
    order = np.lexsort((c, r))
    r, c, v = r[order], c[order], v[order]
    row_ptr = np.concatenate(([0], np.cumsum(np.bincount(r, minlength=rows)[:rows]))).astype(np.int32)
    return row_ptr, c.astype(np.int32), v.astype(np.float32)


def banded_arrays(rows: int, cols: int, bandwidth: int, seed: int):
    rng = np.random.default_rng(seed)
    lo = np.clip(np.arange(rows) - bandwidth, 0, None)
    hi = np.minimum(cols, np.arange(rows) + bandwidth + 1)
    n = np.maximum(hi - lo, 0)
    r = np.repeat(np.arange(rows), n)
    first = np.repeat(np.cumsum(n) - n, n)
    c = np.repeat(lo, n) + (np.arange(r.size) - first)
    v = rng.uniform(-1.0, 1.0, size=r.size).astype(np.float32)
    return _to_csr(rows, r, c, v)


def block_diagonal_arrays(rows: int, cols: int, block: int, seed: int):
    rng = np.random.default_rng(seed)
    nb = min(rows, cols) // block
    e = np.arange(nb * block * block)
    b, rem = np.divmod(e, block * block)
    r = b * block + rem // block
    c = b * block + rem % block
    v = rng.uniform(-1.0, 1.0, size=r.size).astype(np.float32)
    return _to_csr(rows, r, c, v)


def power_law_arrays(rows: int, cols: int, mean_deg: float, alpha: float, seed: int):
    rng = np.random.default_rng(seed)
    deg = rng.pareto(alpha, size=rows) + 1.0
    deg = np.clip(np.round(deg * (mean_deg / deg.mean())).astype(np.int64), 1, cols)
    c = np.concatenate([rng.choice(cols, size=int(d), replace=False) for d in deg])
    r = np.repeat(np.arange(rows), deg)
    v = rng.uniform(-1.0, 1.0, size=r.size).astype(np.float32)
    return _to_csr(rows, r, c, v)


def uniform_mask_arrays(rows: int, cols: int, density: float, seed: int):
    rng = np.random.default_rng(seed)
    r, c = np.nonzero(rng.random((rows, cols)) < density)
    v = rng.uniform(-1.0, 1.0, size=r.size).astype(np.float32)
    return _to_csr(rows, r, c, v)


def host_csr(rows: int, cols: int, arrays):
    import spmm_b200 as S

    rp, ci, v = arrays
    return S.HostCSR(rows, cols, rp, ci, v)


def config(name: str):
    """(A, B) of a BASELINE config c1 .. c5: A a HostCSR (FP32), B a float32 K x N array."""
    import spmm_b200 as S

    if name == "c1":
        return S.generate_uniform_csr(4096, 4096, 0.01, 42), S.generate_dense(4096, 64, 43)
    if name == "c2":
        return host_csr(8192, 8192, banded_arrays(8192, 8192, 41, 42)), S.generate_dense(8192, 128, 43)
    if name == "c3":
        return host_csr(8192, 8192, block_diagonal_arrays(8192, 8192, 128, 42)), S.generate_dense(8192, 256, 43)
    if name == "c4":
        return (host_csr(16384, 16384, power_law_arrays(16384, 16384, 164.0, 1.8, 42)),
                S.generate_dense(16384, 128, 43))
    if name == "c5":
        return S.generate_uniform_csr(131072, 131072, 0.001, 42), S.generate_dense(131072, 256, 43)
    raise KeyError(name)
