"""Seeded inputs for the parity tests: the BASELINE configs and small edge cases.

C1 and C5 use the reference's own C++ generator semantics (through the product's
bit-identical generator), C2-C4 the reference's pattern generators (oracle/patterns.py)."""
from __future__ import annotations

import numpy as np

import spmm_b200 as S
from oracle import oracle as O
from oracle import patterns as P


def to_oracle(A: S.HostCSR) -> O.CSR:
    return O.CSR(A.rows, A.cols, A.row_ptr, A.col_idx, A.values)


def from_arrays(rows: int, cols: int, rp, ci, v) -> S.HostCSR:
    return S.HostCSR(rows, cols, np.ascontiguousarray(rp, np.int32), np.ascontiguousarray(ci, np.int32),
                     np.ascontiguousarray(v, np.float32))


def config(name: str) -> tuple[S.HostCSR, np.ndarray]:
    """(A, B) of a BASELINE config: c1 .. c5 (c3's A is FP32 before the BSR rounding)."""
    if name == "c1":
        return S.generate_uniform_csr(4096, 4096, 0.01, 42), S.generate_dense(4096, 64, 43)
    if name == "c2":
        return from_arrays(8192, 8192, *P.banded(8192, 8192, 41, 42)), S.generate_dense(8192, 128, 43)
    if name == "c3":
        return from_arrays(8192, 8192, *P.block_diagonal(8192, 8192, 128, 42)), S.generate_dense(8192, 256, 43)
    if name == "c4":
        return from_arrays(16384, 16384, *P.power_law(16384, 16384, 164.0, 1.8, 42)), S.generate_dense(16384, 128, 43)
    if name == "c5":
        return S.generate_uniform_csr(131072, 131072, 0.001, 42), S.generate_dense(131072, 256, 43)
    raise KeyError(name)


def random_csr(rows: int, cols: int, lens, seed: int) -> S.HostCSR:
    """CSR with the given per-row lengths, distinct sorted random columns, U(-1,1) values."""
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, dtype=np.int64)
    rp = np.zeros(rows + 1, np.int64)
    np.cumsum(lens, out=rp[1:])
    cols_all = []
    for n in lens:
        n = int(min(n, cols))
        cols_all.append(np.sort(rng.choice(cols, size=n, replace=False)) if n else np.zeros(0, np.int64))
    ci = np.concatenate(cols_all) if cols_all else np.zeros(0, np.int64)
    lens = np.array([c.size for c in cols_all], dtype=np.int64)
    rp = np.zeros(rows + 1, np.int64)
    np.cumsum(lens, out=rp[1:])
    v = rng.uniform(-1.0, 1.0, size=ci.size).astype(np.float32)
    return from_arrays(rows, cols, rp, ci, v)


def dense(rows: int, cols: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).uniform(-1.0, 1.0, size=(rows, cols)).astype(np.float32)
