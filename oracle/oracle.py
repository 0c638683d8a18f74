"""TEST INFRASTRUCTURE ONLY -- ctypes front end of the CPU oracle (oracle/spmm_oracle.cpp)
and of the reference's own host code built into oracle/_ref/libref.so.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's ``cpu_baseline`` / ``--impl
reference`` legs may import this module. The product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_BUILD = HERE / "_build"
_REF = HERE / "_ref" / "libref.so"

_i32p = C.POINTER(C.c_int)
_f32p = C.POINTER(C.c_float)
_u16p = C.POINTER(C.c_uint16)


def _cpu_has_v3() -> bool:
    try:
        flags = Path("/proc/cpuinfo").read_text()
    except OSError:
        return False
    return all(f in flags for f in (" avx2", " fma", " bmi2"))


def build() -> None:
    """Compile the oracle (and, when the reference checkout is present, oracle/_ref)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    ref_src = ref_source()
    if ref_src is not None:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF_SRC={ref_src}"], check=True)


def ref_source() -> Path | None:
    """The reference's src/ directory: $SPMM_REF_SRC, else the location the last `make ref`
    recorded in oracle/_ref/REF_SRC; None when neither names an existing directory (the
    reference is only present where the fixtures are made, never on the GPU box)."""
    env = os.environ.get("SPMM_REF_SRC")
    rec = HERE / "_ref" / "REF_SRC"
    cand = env if env else (rec.read_text().strip() if rec.exists() else "")
    return Path(cand) if cand and Path(cand).is_dir() else None


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        name = "liboracle_v3.so" if _cpu_has_v3() else "liboracle.so"
        path = _BUILD / name
        if not path.exists():
            build()
        L = C.CDLL(str(path))
        L.orc_free.argtypes = [C.c_void_p]
        L.orc_gen_uniform_csr.argtypes = [C.c_int, C.c_int, C.c_float, C.c_int, C.POINTER(_i32p),
                                          C.POINTER(_i32p), C.POINTER(_f32p), _i32p]
        L.orc_gen_dense.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p]
        L.orc_csr_from_coo.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                       C.POINTER(_i32p), C.POINTER(_i32p), C.POINTER(_f32p)]
        L.orc_row_slice.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                    C.POINTER(_i32p), C.POINTER(_i32p), C.POINTER(_f32p), _i32p]
        L.orc_bsr_from_csr.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, _i32p, _i32p,
                                       _i32p, C.POINTER(_i32p), C.POINTER(_i32p), C.POINTER(_u16p)]
        L.orc_bsr_stats.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_long),
                                    C.POINTER(C.c_double), C.POINTER(C.c_double)]
        L.orc_nnz_balanced_bounds.argtypes = [C.c_void_p, C.c_int, C.c_long, C.c_int, C.c_void_p]
        L.orc_spmm_csr_f32.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_int, C.c_int]
        L.orc_spmm_csr_f64.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_int]
        L.orc_spmm_csr_f32_split.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                             C.c_void_p, C.c_int, C.c_int]
        L.orc_spmm_bsr_f64.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int]
        L.orc_compare.argtypes = [C.c_void_p, C.c_void_p, C.c_long, _f32p, _f32p, _f32p]
        L.orc_convert_f32.argtypes = [C.c_void_p, C.c_void_p, C.c_long, C.c_int]
        L.orc_max_threads.restype = C.c_int
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


def _take(L, p, n, dtype) -> np.ndarray:
    """Copy a malloc'd C array into numpy and free it."""
    if n > 0:
        out = np.ctypeslib.as_array(p, shape=(n,)).astype(dtype, copy=True)
    else:
        out = np.zeros(0, dtype=dtype)
    L.orc_free(C.cast(p, C.c_void_p))
    return out


@dataclass
class CSR:
    rows: int
    cols: int
    row_ptr: np.ndarray
    col_idx: np.ndarray
    values: np.ndarray

    @property
    def nnz(self) -> int:
        return int(self.col_idx.size)


@dataclass
class BSR:
    rows: int
    cols: int
    block_rows: int
    block_cols: int
    row_ptr: np.ndarray
    col_idx: np.ndarray
    values: np.ndarray  # uint16 bits, num_blocks*256
    nnz: int

    @property
    def num_blocks(self) -> int:
        return int(self.col_idx.size)


def gen_uniform_csr(rows: int, cols: int, density: float, seed: int) -> CSR:
    L = lib()
    rp, ci, v, n = _i32p(), _i32p(), _f32p(), C.c_int()
    rc = L.orc_gen_uniform_csr(rows, cols, C.c_float(density), seed, C.byref(rp), C.byref(ci), C.byref(v),
                               C.byref(n))
    if rc != 0:
        raise ValueError("orc_gen_uniform_csr: invalid density")
    nnz = n.value
    return CSR(rows, cols, _take(L, rp, rows + 1, np.int32), _take(L, ci, nnz, np.int32),
               _take(L, v, nnz, np.float32))


def gen_dense(rows: int, cols: int, seed: int) -> np.ndarray:
    out = np.empty((rows, cols), dtype=np.float32)
    lib().orc_gen_dense(rows, cols, seed, _ptr(out))
    return out


def csr_from_coo(rows: int, cols: int, r, c, v) -> CSR:
    L = lib()
    r = np.ascontiguousarray(r, np.int32)
    c = np.ascontiguousarray(c, np.int32)
    v = np.ascontiguousarray(v, np.float32)
    rp, ci, vo = _i32p(), _i32p(), _f32p()
    L.orc_csr_from_coo(rows, cols, int(v.size), _ptr(r), _ptr(c), _ptr(v), C.byref(rp), C.byref(ci), C.byref(vo))
    return CSR(rows, cols, _take(L, rp, rows + 1, np.int32), _take(L, ci, v.size, np.int32),
               _take(L, vo, v.size, np.float32))


def row_slice(A: CSR, b: int, e: int) -> CSR:
    L = lib()
    rp, ci, v, n = _i32p(), _i32p(), _f32p(), C.c_int()
    L.orc_row_slice(_ptr(A.row_ptr), _ptr(A.col_idx), _ptr(A.values), b, e, C.byref(rp), C.byref(ci), C.byref(v),
                    C.byref(n))
    return CSR(e - b, A.cols, _take(L, rp, e - b + 1, np.int32), _take(L, ci, n.value, np.int32),
               _take(L, v, n.value, np.float32))


def bsr_from_csr(A: CSR) -> BSR:
    L = lib()
    br, bc, nb = C.c_int(), C.c_int(), C.c_int()
    rp, ci, bv = _i32p(), _i32p(), _u16p()
    L.orc_bsr_from_csr(A.rows, A.cols, _ptr(A.row_ptr), _ptr(A.col_idx), _ptr(A.values), C.byref(br), C.byref(bc),
                       C.byref(nb), C.byref(rp), C.byref(ci), C.byref(bv))
    return BSR(A.rows, A.cols, br.value, bc.value, _take(L, rp, br.value + 1, np.int32),
               _take(L, ci, nb.value, np.int32), _take(L, bv, nb.value * 256, np.uint16), A.nnz)


def bsr_stats(B: BSR):
    stored, fill, dens = C.c_long(), C.c_double(), C.c_double()
    lib().orc_bsr_stats(B.num_blocks, B.nnz, B.block_rows, B.block_cols, C.byref(stored), C.byref(fill),
                        C.byref(dens))
    return {"num_blocks": B.num_blocks, "stored_elements": stored.value, "original_nnz": B.nnz,
            "fill_in_ratio": fill.value, "block_density": dens.value}


def nnz_balanced_bounds(A: CSR, G: int) -> np.ndarray:
    out = np.zeros(G + 1, dtype=np.int32)
    lib().orc_nnz_balanced_bounds(_ptr(A.row_ptr), A.rows, A.nnz, G, _ptr(out))
    return out


def spmm_csr_f32(A: CSR, B: np.ndarray, threads: int = 0, dynamic: bool = False) -> np.ndarray:
    B = np.ascontiguousarray(B, np.float32)
    N = B.shape[1]
    out = np.empty((A.rows, N), dtype=np.float32)
    lib().orc_spmm_csr_f32(A.rows, N, _ptr(A.row_ptr), _ptr(A.col_idx), _ptr(A.values), _ptr(B), _ptr(out),
                           threads, int(dynamic))
    return out


def spmm_csr_f32_split(A: CSR, B: np.ndarray, S: int, threads: int = 0) -> np.ndarray:
    """FP32 reference semantics with long rows (> S nonzeros) cut at multiples of S in
    row + nonzero index, pieces added left to right (the engine's merge-path arithmetic)."""
    B = np.ascontiguousarray(B, np.float32)
    N = B.shape[1]
    out = np.empty((A.rows, N), dtype=np.float32)
    lib().orc_spmm_csr_f32_split(A.rows, N, _ptr(A.row_ptr), _ptr(A.col_idx), _ptr(A.values), _ptr(B), _ptr(out),
                                 S, threads)
    return out


def spmm_csr_f64(A: CSR, B: np.ndarray, threads: int = 0) -> np.ndarray:
    B = np.ascontiguousarray(B, np.float32)
    N = B.shape[1]
    out = np.empty((A.rows, N), dtype=np.float64)
    lib().orc_spmm_csr_f64(A.rows, N, _ptr(A.row_ptr), _ptr(A.col_idx), _ptr(A.values), _ptr(B), _ptr(out), threads)
    return out


def spmm_bsr_f64(A: BSR, B16: np.ndarray, dtype: int = 0, threads: int = 0) -> np.ndarray:
    B16 = np.ascontiguousarray(B16, np.uint16)
    N = B16.shape[1]
    out = np.zeros((A.rows, N), dtype=np.float64)
    lib().orc_spmm_bsr_f64(A.rows, A.cols, N, A.block_rows, _ptr(A.row_ptr), _ptr(A.col_idx), _ptr(A.values),
                           _ptr(B16), dtype, _ptr(out), threads)
    return out


def to_half_bits(x: np.ndarray, bf16: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_convert_f32(_ptr(x), _ptr(out), x.size, int(bf16))
    return out


def compare(ours: np.ndarray, ref: np.ndarray):
    """harness.cu-style metrics: (max_abs, filtered max_rel, rel_l2)."""
    a = np.ascontiguousarray(ours, np.float32).ravel()
    b = np.ascontiguousarray(ref, np.float32).ravel()
    ma, mr, l2 = C.c_float(), C.c_float(), C.c_float()
    lib().orc_compare(_ptr(a), _ptr(b), a.size, C.byref(ma), C.byref(mr), C.byref(l2))
    return ma.value, mr.value, l2.value


def max_rel_vs_f64(ours: np.ndarray, ref64: np.ndarray) -> float:
    """compare()'s filtered max relative error measured against an FP64 reference."""
    ref = np.asarray(ref64, np.float64)
    d = np.abs(np.asarray(ours, np.float64) - ref)
    a = np.abs(ref)
    if a.size == 0:
        return 0.0
    keep = a > 1e-3 * a.max()
    return float((d[keep] / a[keep]).max()) if keep.any() else 0.0


def max_threads() -> int:
    return int(lib().orc_max_threads())


# ----------------------------------------------------------------------------------------
# The reference's own host code (oracle/_ref/libref.so), when it has been built.
# ----------------------------------------------------------------------------------------
_ref = None


def ref_available() -> bool:
    return _REF.exists()


def ref() -> C.CDLL:
    global _ref
    if _ref is None:
        L = C.CDLL(str(_REF))
        L.ref_free.argtypes = [C.c_void_p]
        L.ref_gen_uniform_csr.argtypes = [C.c_int, C.c_int, C.c_float, C.c_int, C.POINTER(_i32p),
                                          C.POINTER(_i32p), C.POINTER(_f32p), _i32p]
        L.ref_gen_dense.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p]
        L.ref_csr_from_coo.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                       C.POINTER(_i32p), C.POINTER(_i32p), C.POINTER(_f32p)]
        L.ref_bsr_from_csr.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, _i32p, _i32p,
                                       _i32p, C.POINTER(_i32p), C.POINTER(_i32p), C.POINTER(_u16p),
                                       C.POINTER(C.c_long), C.POINTER(C.c_double), C.POINTER(C.c_double)]
        L.ref_nnz_balanced_bounds.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p]
        L.ref_compare.argtypes = [C.c_void_p, C.c_void_p, C.c_long, _f32p, _f32p, _f32p]
        L.ref_spmm_csr_device.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_void_p, C.c_int]
        L.ref_spmm_wmma_device.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                           C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        _ref = L
    return _ref


def _rtake(L, p, n, dtype):
    out = np.ctypeslib.as_array(p, shape=(n,)).astype(dtype, copy=True) if n > 0 else np.zeros(0, dtype)
    L.ref_free(C.cast(p, C.c_void_p))
    return out


def ref_gen_uniform_csr(rows: int, cols: int, density: float, seed: int) -> CSR:
    L = ref()
    rp, ci, v, n = _i32p(), _i32p(), _f32p(), C.c_int()
    L.ref_gen_uniform_csr(rows, cols, C.c_float(density), seed, C.byref(rp), C.byref(ci), C.byref(v), C.byref(n))
    return CSR(rows, cols, _rtake(L, rp, rows + 1, np.int32), _rtake(L, ci, n.value, np.int32),
               _rtake(L, v, n.value, np.float32))


def ref_gen_dense(rows: int, cols: int, seed: int) -> np.ndarray:
    out = np.empty((rows, cols), dtype=np.float32)
    ref().ref_gen_dense(rows, cols, seed, _ptr(out))
    return out


def ref_csr_from_coo(rows: int, cols: int, r, c, v) -> CSR:
    L = ref()
    r = np.ascontiguousarray(r, np.int32)
    c = np.ascontiguousarray(c, np.int32)
    v = np.ascontiguousarray(v, np.float32)
    rp, ci, vo = _i32p(), _i32p(), _f32p()
    L.ref_csr_from_coo(rows, cols, int(v.size), _ptr(r), _ptr(c), _ptr(v), C.byref(rp), C.byref(ci), C.byref(vo))
    return CSR(rows, cols, _rtake(L, rp, rows + 1, np.int32), _rtake(L, ci, v.size, np.int32),
               _rtake(L, vo, v.size, np.float32))


def ref_bsr_from_csr(A: CSR):
    L = ref()
    br, bc, nb = C.c_int(), C.c_int(), C.c_int()
    rp, ci, bv = _i32p(), _i32p(), _u16p()
    stored, fill, dens = C.c_long(), C.c_double(), C.c_double()
    L.ref_bsr_from_csr(A.rows, A.cols, A.nnz, _ptr(A.row_ptr), _ptr(A.col_idx), _ptr(A.values), C.byref(br),
                       C.byref(bc), C.byref(nb), C.byref(rp), C.byref(ci), C.byref(bv), C.byref(stored),
                       C.byref(fill), C.byref(dens))
    b = BSR(A.rows, A.cols, br.value, bc.value, _rtake(L, rp, br.value + 1, np.int32),
            _rtake(L, ci, nb.value, np.int32), _rtake(L, bv, nb.value * 256, np.uint16), A.nnz)
    stats = {"num_blocks": nb.value, "stored_elements": stored.value, "original_nnz": A.nnz,
             "fill_in_ratio": fill.value, "block_density": dens.value}
    return b, stats


def ref_nnz_balanced_bounds(A: CSR, G: int) -> np.ndarray:
    out = np.zeros(G + 1, dtype=np.int32)
    ref().ref_nnz_balanced_bounds(A.rows, A.nnz, _ptr(A.row_ptr), G, _ptr(out))
    return out


def ref_compare(ours: np.ndarray, refv: np.ndarray):
    a = np.ascontiguousarray(ours, np.float32).ravel()
    b = np.ascontiguousarray(refv, np.float32).ravel()
    ma, mr, l2 = C.c_float(), C.c_float(), C.c_float()
    ref().ref_compare(_ptr(a), _ptr(b), a.size, C.byref(ma), C.byref(mr), C.byref(l2))
    return ma.value, mr.value, l2.value
