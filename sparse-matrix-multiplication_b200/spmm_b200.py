"""Python binding of the B200 SpMM engine's C ABI (include/spmm_c.h, lib/libspmm_b200.so).

ctypes only: device buffers are passed as raw pointers (torch tensors are accepted and must
live on the current CUDA device), host buffers as numpy arrays. There is no fallback: if the
shared library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "lib" / "libspmm_b200.so"
CXX_LIB_PATH = HERE / "lib" / "libspmm.so"

OK = 0
ERR = {
    -1: "SPMM_ERR_INVALID_ARG", -2: "SPMM_ERR_MISALIGNED", -3: "SPMM_ERR_CUDA", -4: "SPMM_ERR_NCCL",
    -5: "SPMM_ERR_TIMEOUT", -6: "SPMM_ERR_UNSUPPORTED", -7: "SPMM_ERR_NO_MEMORY", -8: "SPMM_ERR_BAD_INDEX",
    -9: "SPMM_ERR_IO", -10: "SPMM_ERR_TOO_LARGE",
}
CSR_AUTO, CSR_ROWWARP, CSR_MERGE = 0, 1, 2
DTYPE_F16, DTYPE_BF16 = 0, 1
BACKEND_CSR, BACKEND_TC = 0, 1

# Every symbol include/spmm_c.h declares (checked by the CPU test suite).
EXPORTS = [
    "spmm_status_string", "spmm_version", "spmm_csr_host_alloc", "spmm_csr_host_free", "spmm_csr_from_coo_host",
    "spmm_generate_uniform_csr", "spmm_generate_uniform_csr_fast", "spmm_generate_dense", "spmm_csr_row_slice_host", "spmm_csr_read_binary",
    "spmm_csr_write_binary", "spmm_csr_validate_host", "spmm_csr_to_bsr16_host", "spmm_bsr_host_free",
    "spmm_bsr_compute_stats", "spmm_nnz_balanced_bounds", "spmm_csr_f32", "spmm_csr_f32_workspace_size",
    "spmm_csr_f32_ws", "spmm_csr_f32_chunk", "spmm_csr_f32_host", "spmm_convert_f32", "spmm_bsr16",
    "spmm_bsr16_algo", "spmm_device_error", "spmm_hybrid_default_threshold", "spmm_hybrid_choose",
    "spmm_backend_name", "spmm_hybrid_run", "spmm_gpu_count", "spmm_multigpu_run", "spmm_unified_run",
    "spmm_unified_run_ex", "spmm_bsr16_plan_create", "spmm_bsr16_plan_execute", "spmm_bsr16_plan_info",
    "spmm_bsr16_plan_destroy", "spmm_bsr16_plan_a_stride",
    "spmm_csr_f32_noalloc", "spmm_csr_to_bsr16_device_count", "spmm_csr_to_bsr16_device_fill",
    "spmm_csr_plan_create", "spmm_csr_plan_execute", "spmm_csr_plan_info", "spmm_csr_plan_destroy",
    "spmm_csr_plan_k_phases", "spmm_csr_plan_launches",
    "spmm_comm_unique_id", "spmm_comm_init", "spmm_comm_wrap", "spmm_comm_info", "spmm_comm_destroy",
    "spmm_rank_plan_create", "spmm_rank_plan_info", "spmm_rank_run", "spmm_rank_submit", "spmm_rank_wait",
    "spmm_rank_execute", "spmm_rank_gather_b",
    "spmm_rank_plan_buffers", "spmm_rank_plan_destroy",
]


class SpmmError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {ERR.get(status, status)} ({status_string(status)})")


class CsrView(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("nnz", C.c_int32), ("row_ptr", C.c_void_p),
                ("col_idx", C.c_void_p), ("values", C.c_void_p)]


class CsrHost(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("nnz", C.c_int32), ("row_ptr", C.POINTER(C.c_int32)),
                ("col_idx", C.POINTER(C.c_int32)), ("values", C.POINTER(C.c_float))]


class BsrView(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("block_rows", C.c_int32), ("block_cols", C.c_int32),
                ("num_blocks", C.c_int32), ("nnz", C.c_int32), ("row_ptr", C.c_void_p), ("col_idx", C.c_void_p),
                ("values", C.c_void_p), ("dtype", C.c_int32)]


class BsrHost(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("block_rows", C.c_int32), ("block_cols", C.c_int32),
                ("num_blocks", C.c_int32), ("nnz", C.c_int32), ("dtype", C.c_int32),
                ("row_ptr", C.POINTER(C.c_int32)), ("col_idx", C.POINTER(C.c_int32)),
                ("values", C.POINTER(C.c_uint16))]


class BsrStats(C.Structure):
    _fields_ = [("num_blocks", C.c_int32), ("stored_elements", C.c_int64), ("original_nnz", C.c_int32),
                ("fill_in_ratio", C.c_double), ("block_density", C.c_double)]


class CsrTuning(C.Structure):
    _fields_ = [("chunk", C.c_int32), ("col_pass", C.c_int32), ("b_policy", C.c_int32), ("k_phases", C.c_int32),
                ("schedule", C.c_int32), ("phase_mode", C.c_int32), ("reserved", C.c_int32 * 2)]


class HybridPlan(C.Structure):
    _fields_ = [("backend", C.c_int32), ("fill_in_ratio", C.c_double), ("block_density", C.c_double),
                ("threshold", C.c_float), ("n_aligned", C.c_int32), ("reason", C.c_char_p)]


_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load lib/libspmm_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {HERE}` (or __graft_entry__.build())")
    L = C.CDLL(str(LIB_PATH))
    vp, i32, i64, f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_float
    sig = {
        "spmm_status_string": (C.c_char_p, [C.c_int]),
        "spmm_version": (C.c_int, []),
        "spmm_csr_host_alloc": (C.c_int, [i32, i32, i32, C.POINTER(CsrHost)]),
        "spmm_csr_host_free": (None, [C.POINTER(CsrHost)]),
        "spmm_csr_from_coo_host": (C.c_int, [i32, i32, i32, vp, vp, vp, C.POINTER(CsrHost)]),
        "spmm_generate_uniform_csr": (C.c_int, [i32, i32, f32, i32, C.POINTER(CsrHost)]),
        "spmm_generate_uniform_csr_fast": (C.c_int, [i32, i32, f32, C.c_int64, i32, C.POINTER(CsrHost)]),
        "spmm_generate_dense": (C.c_int, [i32, i32, i32, vp]),
        "spmm_csr_row_slice_host": (C.c_int, [C.POINTER(CsrView), i32, i32, C.POINTER(CsrHost)]),
        "spmm_csr_read_binary": (C.c_int, [C.c_char_p, C.POINTER(CsrHost)]),
        "spmm_csr_write_binary": (C.c_int, [C.POINTER(CsrView), C.c_char_p]),
        "spmm_csr_validate_host": (C.c_int, [C.POINTER(CsrView), C.POINTER(i32)]),
        "spmm_csr_to_bsr16_host": (C.c_int, [C.POINTER(CsrView), i32, C.POINTER(BsrHost)]),
        "spmm_bsr_host_free": (None, [C.POINTER(BsrHost)]),
        "spmm_bsr_compute_stats": (C.c_int, [C.POINTER(BsrView), C.POINTER(BsrStats)]),
        "spmm_nnz_balanced_bounds": (C.c_int, [vp, i32, i64, i32, vp]),
        "spmm_csr_f32": (C.c_int, [C.POINTER(CsrView), vp, vp, i32, i32, vp]),
        "spmm_csr_f32_workspace_size": (C.c_int, [C.POINTER(CsrView), i32, i32, C.POINTER(CsrTuning),
                                                   C.POINTER(C.c_size_t)]),
        "spmm_csr_f32_ws": (C.c_int, [C.POINTER(CsrView), vp, vp, i32, i32, C.POINTER(CsrTuning), vp, C.c_size_t,
                                      vp]),
        "spmm_csr_f32_chunk": (C.c_int, [C.POINTER(CsrView), i32, i32, C.POINTER(CsrTuning), C.POINTER(i32)]),
        "spmm_csr_f32_host": (C.c_int, [C.POINTER(CsrView), vp, vp, i32, i32, vp]),
        "spmm_convert_f32": (C.c_int, [vp, vp, i64, i32, vp]),
        "spmm_bsr16": (C.c_int, [C.POINTER(BsrView), vp, vp, i32, vp]),
        "spmm_bsr16_algo": (C.c_int, [C.POINTER(BsrView), vp, vp, i32, i32, vp]),
        "spmm_bsr16_plan_create": (C.c_int, [C.POINTER(BsrView), i32, vp, C.POINTER(vp)]),
        "spmm_bsr16_plan_execute": (C.c_int, [vp, vp, vp, vp]),
        "spmm_bsr16_plan_info": (C.c_int, [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(C.c_size_t)]),
        "spmm_bsr16_plan_destroy": (None, [vp]),
        "spmm_bsr16_plan_a_stride": (C.c_int, [vp, C.POINTER(i32)]),
        "spmm_device_error": (C.c_int, [i32, C.POINTER(i32), C.POINTER(i64), i32]),
        "spmm_hybrid_default_threshold": (f32, []),
        "spmm_hybrid_choose": (C.c_int, [C.POINTER(CsrView), i32, f32, C.POINTER(HybridPlan)]),
        "spmm_backend_name": (C.c_char_p, [i32]),
        "spmm_hybrid_run": (C.c_int, [C.POINTER(HybridPlan), C.POINTER(CsrView), vp, vp, i32, i32, i32,
                                      C.POINTER(f32)]),
        "spmm_gpu_count": (C.c_int, []),
        "spmm_multigpu_run": (C.c_int, [C.POINTER(CsrView), vp, vp, i32, i32, i32, i32, C.POINTER(f32),
                                        C.POINTER(i32), vp, vp, C.POINTER(f32)]),
        "spmm_unified_run": (C.c_int, [C.POINTER(CsrView), vp, vp, i32, i32, i32, C.POINTER(f32)]),
        "spmm_unified_run_ex": (C.c_int, [C.POINTER(CsrView), vp, vp, i32, C.c_size_t, i32, i32, C.POINTER(f32),
                                          C.POINTER(i32)]),
        "spmm_csr_f32_noalloc": (C.c_int, [C.POINTER(CsrView), vp, vp, i32, i32, vp]),
        "spmm_csr_to_bsr16_device_count": (C.c_int, [C.POINTER(CsrView), vp, C.POINTER(i32), vp]),
        "spmm_csr_to_bsr16_device_fill": (C.c_int, [C.POINTER(CsrView), vp, vp, vp, i32, vp]),
        "spmm_csr_plan_create": (C.c_int, [C.POINTER(CsrView), i32, C.POINTER(CsrTuning), vp, C.POINTER(vp)]),
        "spmm_csr_plan_execute": (C.c_int, [vp, vp, vp, vp]),
        "spmm_csr_plan_info": (C.c_int, [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(C.c_size_t)]),
        "spmm_csr_plan_k_phases": (C.c_int, [vp, C.POINTER(i32)]),
        "spmm_csr_plan_launches": (C.c_int, [vp, C.POINTER(i32)]),
        "spmm_csr_plan_destroy": (None, [vp]),
        "spmm_comm_unique_id": (C.c_int, [vp]),
        "spmm_comm_init": (C.c_int, [vp, i32, i32, i32, C.POINTER(vp)]),
        "spmm_comm_wrap": (C.c_int, [vp, i32, C.POINTER(vp)]),
        "spmm_comm_info": (C.c_int, [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32)]),
        "spmm_comm_destroy": (None, [vp]),
        "spmm_rank_plan_create": (C.c_int, [vp, C.POINTER(CsrView), i32, vp, C.POINTER(vp)]),
        "spmm_rank_plan_info": (C.c_int, [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32), C.POINTER(i32),
                                          C.POINTER(i32), C.POINTER(i32), C.POINTER(i32)]),
        "spmm_rank_run": (C.c_int, [vp, C.POINTER(CsrView), vp, vp, vp]),
        "spmm_rank_submit": (C.c_int, [vp, C.POINTER(CsrView), vp, vp, vp]),
        "spmm_rank_wait": (C.c_int, [vp, vp]),
        "spmm_rank_execute": (C.c_int, [vp, vp]),
        "spmm_rank_gather_b": (C.c_int, [vp, vp]),
        "spmm_rank_plan_buffers": (C.c_int, [vp, C.POINTER(vp), C.POINTER(vp)]),
        "spmm_rank_plan_destroy": (None, [vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def status_string(status: int) -> str:
    try:
        return lib().spmm_status_string(status).decode()
    except Exception:  # noqa: BLE001 - used while formatting another error
        return "?"


def check(status: int, what: str) -> None:
    if status != OK:
        raise SpmmError(status, what)


# ------------------------------------------------------------------ pointers


def ptr(x) -> int:
    """Raw address of a torch tensor or numpy array (0 for None)."""
    if x is None:
        return 0
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr())
    return int(x.ctypes.data)


def stream_ptr(stream) -> int:
    if stream is None:
        return 0
    if hasattr(stream, "cuda_stream"):
        return int(stream.cuda_stream)
    return int(stream)


# ------------------------------------------------------------------ host CSR


@dataclass
class HostCSR:
    rows: int
    cols: int
    row_ptr: np.ndarray
    col_idx: np.ndarray
    values: np.ndarray

    @property
    def nnz(self) -> int:
        return int(self.col_idx.size)

    def view(self) -> CsrView:
        return CsrView(self.rows, self.cols, self.nnz, ptr(self.row_ptr), ptr(self.col_idx), ptr(self.values))


def _adopt(h: CsrHost) -> HostCSR:
    L = lib()
    rp = np.ctypeslib.as_array(h.row_ptr, shape=(h.rows + 1,)).copy()
    ci = np.ctypeslib.as_array(h.col_idx, shape=(h.nnz,)).copy() if h.nnz else np.zeros(0, np.int32)
    v = np.ctypeslib.as_array(h.values, shape=(h.nnz,)).copy() if h.nnz else np.zeros(0, np.float32)
    out = HostCSR(h.rows, h.cols, rp, ci, v)
    L.spmm_csr_host_free(C.byref(h))
    return out


def generate_uniform_csr(rows: int, cols: int, density: float, seed: int) -> HostCSR:
    h = CsrHost()
    check(lib().spmm_generate_uniform_csr(rows, cols, density, seed, C.byref(h)), "spmm_generate_uniform_csr")
    return _adopt(h)


def generate_uniform_csr_fast(rows: int, cols: int, density: float, seed: int, threads: int = 0) -> HostCSR:
    """Geometric-gap uniform CSR (not the reference's mt19937 stream; same expected nnz)."""
    h = CsrHost()
    check(lib().spmm_generate_uniform_csr_fast(rows, cols, density, seed, threads, C.byref(h)),
          "spmm_generate_uniform_csr_fast")
    return _adopt(h)


def generate_dense(rows: int, cols: int, seed: int) -> np.ndarray:
    out = np.empty((rows, cols), dtype=np.float32)
    check(lib().spmm_generate_dense(rows, cols, seed, ptr(out)), "spmm_generate_dense")
    return out


def csr_from_coo(rows: int, cols: int, r, c, v) -> HostCSR:
    r = np.ascontiguousarray(r, np.int32)
    c = np.ascontiguousarray(c, np.int32)
    v = np.ascontiguousarray(v, np.float32)
    h = CsrHost()
    check(lib().spmm_csr_from_coo_host(rows, cols, int(v.size), ptr(r), ptr(c), ptr(v), C.byref(h)),
          "spmm_csr_from_coo_host")
    return _adopt(h)


def row_slice(A: HostCSR, b: int, e: int) -> HostCSR:
    h = CsrHost()
    v = A.view()
    check(lib().spmm_csr_row_slice_host(C.byref(v), b, e, C.byref(h)), "spmm_csr_row_slice_host")
    return _adopt(h)


def read_binary(path: str | os.PathLike) -> HostCSR:
    h = CsrHost()
    check(lib().spmm_csr_read_binary(os.fsencode(path), C.byref(h)), "spmm_csr_read_binary")
    return _adopt(h)


def write_binary(A: HostCSR, path: str | os.PathLike) -> None:
    v = A.view()
    check(lib().spmm_csr_write_binary(C.byref(v), os.fsencode(path)), "spmm_csr_write_binary")


def validate(A: HostCSR) -> int:
    """-1 when A is well formed, else the first bad row (raises on bad arguments)."""
    bad = C.c_int32(-1)
    v = A.view()
    rc = lib().spmm_csr_validate_host(C.byref(v), C.byref(bad))
    if rc == OK:
        return -1
    if bad.value >= 0:
        return bad.value
    raise SpmmError(rc, "spmm_csr_validate_host")


@dataclass
class HostBSR:
    rows: int
    cols: int
    block_rows: int
    block_cols: int
    row_ptr: np.ndarray
    col_idx: np.ndarray
    values: np.ndarray  # uint16 bits
    nnz: int
    dtype: int

    @property
    def num_blocks(self) -> int:
        return int(self.col_idx.size)

    def view(self) -> BsrView:
        return BsrView(self.rows, self.cols, self.block_rows, self.block_cols, self.num_blocks, self.nnz,
                       ptr(self.row_ptr), ptr(self.col_idx), ptr(self.values), self.dtype)


def csr_to_bsr16(A: HostCSR, dtype: int = DTYPE_F16) -> HostBSR:
    b = BsrHost()
    v = A.view()
    check(lib().spmm_csr_to_bsr16_host(C.byref(v), dtype, C.byref(b)), "spmm_csr_to_bsr16_host")
    nb = b.num_blocks
    out = HostBSR(b.rows, b.cols, b.block_rows, b.block_cols,
                  np.ctypeslib.as_array(b.row_ptr, shape=(b.block_rows + 1,)).copy(),
                  np.ctypeslib.as_array(b.col_idx, shape=(nb,)).copy() if nb else np.zeros(0, np.int32),
                  np.ctypeslib.as_array(b.values, shape=(nb * 256,)).copy() if nb else np.zeros(0, np.uint16),
                  b.nnz, b.dtype)
    lib().spmm_bsr_host_free(C.byref(b))
    return out


def bsr_stats(B: HostBSR) -> dict:
    s = BsrStats()
    v = B.view()
    check(lib().spmm_bsr_compute_stats(C.byref(v), C.byref(s)), "spmm_bsr_compute_stats")
    return {"num_blocks": s.num_blocks, "stored_elements": s.stored_elements, "original_nnz": s.original_nnz,
            "fill_in_ratio": s.fill_in_ratio, "block_density": s.block_density}


def nnz_balanced_bounds(row_ptr: np.ndarray, rows: int, nnz: int, G: int) -> np.ndarray:
    row_ptr = np.ascontiguousarray(row_ptr, np.int32)
    out = np.zeros(G + 1, dtype=np.int32)
    check(lib().spmm_nnz_balanced_bounds(ptr(row_ptr), rows, nnz, G, ptr(out)), "spmm_nnz_balanced_bounds")
    return out


def hybrid_choose(A: HostCSR, N: int, threshold: float = 0.0) -> dict:
    p = HybridPlan()
    v = A.view()
    check(lib().spmm_hybrid_choose(C.byref(v), N, threshold, C.byref(p)), "spmm_hybrid_choose")
    return {"backend": p.backend, "backend_name": lib().spmm_backend_name(p.backend).decode(),
            "fill_in_ratio": p.fill_in_ratio, "block_density": p.block_density, "threshold": p.threshold,
            "n_aligned": bool(p.n_aligned), "reason": p.reason.decode(), "_plan": p}


# ------------------------------------------------------------------ device compute


def device_view(rows: int, cols: int, row_ptr, col_idx, values) -> CsrView:
    """CsrView over device tensors (int32 row_ptr/col_idx, float32 values)."""
    nnz = int(col_idx.numel()) if hasattr(col_idx, "numel") else int(col_idx.size)
    return CsrView(rows, cols, nnz, ptr(row_ptr), ptr(col_idx), ptr(values))


def csr_f32(A: CsrView, B, Cout, N: int, algo: int = CSR_AUTO, stream=None) -> None:
    check(lib().spmm_csr_f32(C.byref(A), ptr(B), ptr(Cout), N, algo, stream_ptr(stream)), "spmm_csr_f32")


def csr_f32_ws(A: CsrView, B, Cout, N: int, algo: int, tuning: CsrTuning | None, ws, ws_bytes: int,
               stream=None) -> None:
    t = C.byref(tuning) if tuning is not None else None
    check(lib().spmm_csr_f32_ws(C.byref(A), ptr(B), ptr(Cout), N, algo, t, ptr(ws), ws_bytes, stream_ptr(stream)),
          "spmm_csr_f32_ws")


def csr_workspace_size(A: CsrView, N: int, algo: int = CSR_AUTO, tuning: CsrTuning | None = None) -> int:
    n = C.c_size_t()
    t = C.byref(tuning) if tuning is not None else None
    check(lib().spmm_csr_f32_workspace_size(C.byref(A), N, algo, t, C.byref(n)), "spmm_csr_f32_workspace_size")
    return int(n.value)


def csr_chunk(A: CsrView, N: int, algo: int = CSR_AUTO, tuning: CsrTuning | None = None) -> int:
    c = C.c_int32()
    t = C.byref(tuning) if tuning is not None else None
    check(lib().spmm_csr_f32_chunk(C.byref(A), N, algo, t, C.byref(c)), "spmm_csr_f32_chunk")
    return int(c.value)


def csr_f32_host(A: HostCSR, B: np.ndarray, Cout: np.ndarray, N: int, algo: int = CSR_AUTO, stream=None) -> None:
    v = A.view()
    check(lib().spmm_csr_f32_host(C.byref(v), ptr(B), ptr(Cout), N, algo, stream_ptr(stream)), "spmm_csr_f32_host")


def convert_f32(src, dst, n: int, dtype: int = DTYPE_F16, stream=None) -> None:
    check(lib().spmm_convert_f32(ptr(src), ptr(dst), n, dtype, stream_ptr(stream)), "spmm_convert_f32")


def bsr16(A: BsrView, B16, Cout, N: int, algo: int = 0, stream=None) -> None:
    check(lib().spmm_bsr16_algo(C.byref(A), ptr(B16), ptr(Cout), N, algo, stream_ptr(stream)), "spmm_bsr16")


class BsrPlan:
    """spmm_bsr16_plan_* wrapper: precompute the per-CTA schedule once, execute many times."""

    def __init__(self, A: BsrView, N: int, stream=None):
        self._A = A
        self.N = N
        h = C.c_void_p()
        check(lib().spmm_bsr16_plan_create(C.byref(A), N, stream_ptr(stream), C.byref(h)), "spmm_bsr16_plan_create")
        self._h = h
        g, ms, nb = C.c_int32(), C.c_int32(), C.c_size_t()
        check(lib().spmm_bsr16_plan_info(h, C.byref(g), C.byref(ms), C.byref(nb)), "spmm_bsr16_plan_info")
        self.group, self.max_steps, self.schedule_bytes = int(g.value), int(ms.value), int(nb.value)
        st = C.c_int32()
        check(lib().spmm_bsr16_plan_a_stride(h, C.byref(st)), "spmm_bsr16_plan_a_stride")
        self.a_stride = int(st.value)  # block stride of the grouped A copies (0: none)

    def execute(self, B16, Cout, stream=None) -> None:
        check(lib().spmm_bsr16_plan_execute(self._h, ptr(B16), ptr(Cout), stream_ptr(stream)), "spmm_bsr16_plan_execute")

    def close(self) -> None:
        if self._h:
            lib().spmm_bsr16_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class CsrPlan:
    """spmm_csr_plan_* wrapper: inspect A once, execute many times (no allocation per call)."""

    def __init__(self, A: CsrView, N: int, tuning: CsrTuning | None = None, stream=None):
        self._A = A  # keep the view alive: the plan refers to the same device arrays
        self.N = N
        h = C.c_void_p()
        t = C.byref(tuning) if tuning is not None else None
        check(lib().spmm_csr_plan_create(C.byref(A), N, t, stream_ptr(stream), C.byref(h)), "spmm_csr_plan_create")
        self._h = h
        algo, mx, ws = C.c_int32(), C.c_int32(), C.c_size_t()
        check(lib().spmm_csr_plan_info(h, C.byref(algo), C.byref(mx), C.byref(ws)), "spmm_csr_plan_info")
        self.algo, self.max_row, self.ws_bytes = int(algo.value), int(mx.value), int(ws.value)
        ph = C.c_int32()
        check(lib().spmm_csr_plan_k_phases(h, C.byref(ph)), "spmm_csr_plan_k_phases")
        self.k_phases = int(ph.value)  # column phases
        check(lib().spmm_csr_plan_launches(h, C.byref(ph)), "spmm_csr_plan_launches")
        self.launches = int(ph.value)  # kernel launches per execute

    def execute(self, B, Cout, stream=None) -> None:
        check(lib().spmm_csr_plan_execute(self._h, ptr(B), ptr(Cout), stream_ptr(stream)), "spmm_csr_plan_execute")

    def close(self) -> None:
        if self._h:
            lib().spmm_csr_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def csr_to_bsr16_device(A: CsrView, dtype: int = DTYPE_F16, stream=None):
    """CSR (device view) -> BSR-16 on the GPU. Returns (BsrView, [row_ptr, col_idx, values]
    torch tensors that own the memory)."""
    import torch

    br = (A.rows + 15) // 16
    rp = torch.empty(br + 1, dtype=torch.int32, device="cuda")
    nb = C.c_int32()
    check(lib().spmm_csr_to_bsr16_device_count(C.byref(A), ptr(rp), C.byref(nb), stream_ptr(stream)),
          "spmm_csr_to_bsr16_device_count")
    n = int(nb.value)
    ci = torch.empty(max(n, 1), dtype=torch.int32, device="cuda")
    vals = torch.empty(max(n * 256, 2), dtype=torch.int16, device="cuda")
    check(lib().spmm_csr_to_bsr16_device_fill(C.byref(A), ptr(rp), ptr(ci), ptr(vals), dtype, stream_ptr(stream)),
          "spmm_csr_to_bsr16_device_fill")
    view = BsrView(A.rows, A.cols, br, (A.cols + 15) // 16, n, A.nnz, ptr(rp), ptr(ci), ptr(vals), dtype)
    return view, [rp, ci, vals]


def device_error(device: int = 0, clear: bool = True) -> tuple[int, int]:
    code, detail = C.c_int32(), C.c_int64()
    check(lib().spmm_device_error(device, C.byref(code), C.byref(detail), int(clear)), "spmm_device_error")
    return int(code.value), int(detail.value)


def gpu_count() -> int:
    return int(lib().spmm_gpu_count())


def hybrid_run(plan: dict, A: HostCSR, B: np.ndarray, Cout: np.ndarray, N: int, warmup: int, iters: int) -> float:
    ms = C.c_float()
    v = A.view()
    check(lib().spmm_hybrid_run(C.byref(plan["_plan"]), C.byref(v), ptr(B), ptr(Cout), N, warmup, iters,
                                C.byref(ms)), "spmm_hybrid_run")
    return float(ms.value)


def multigpu_run(A: HostCSR, B: np.ndarray, Cout: np.ndarray, N: int, gpus: int, warmup: int, iters: int) -> dict:
    ms, used, bc = C.c_float(), C.c_int32(), C.c_float()
    rows = np.zeros(max(gpus, 1), np.int32)
    nnz = np.zeros(max(gpus, 1), np.int32)
    v = A.view()
    check(lib().spmm_multigpu_run(C.byref(v), ptr(B), ptr(Cout), N, gpus, warmup, iters, C.byref(ms), C.byref(used),
                                  ptr(rows), ptr(nnz), C.byref(bc)), "spmm_multigpu_run")
    g = int(used.value)
    return {"time_ms": float(ms.value), "num_gpus": g, "rows": rows[:g].tolist(), "nnz": nnz[:g].tolist(),
            "bcast_ms": float(bc.value)}


def unified_run(A: HostCSR, B: np.ndarray, Cout: np.ndarray, N: int, warmup: int, iters: int) -> float:
    ms = C.c_float()
    v = A.view()
    check(lib().spmm_unified_run(C.byref(v), ptr(B), ptr(Cout), N, warmup, iters, C.byref(ms)), "spmm_unified_run")
    return float(ms.value)


def unified_run_ex(A: HostCSR, B: np.ndarray, Cout: np.ndarray, N: int, device_budget: int, warmup: int,
                   iters: int) -> tuple[float, int]:
    """spmm_unified_run_ex: (median ms per pass, column phases used)."""
    ms, ph = C.c_float(), C.c_int32()
    v = A.view()
    check(lib().spmm_unified_run_ex(C.byref(v), ptr(B), ptr(Cout), N, device_budget, warmup, iters, C.byref(ms),
                                    C.byref(ph)), "spmm_unified_run_ex")
    return float(ms.value), int(ph.value)


# ------------------------------------------------------------------ multi-GPU, one process per GPU

COMM_ID_BYTES = 128


def comm_unique_id() -> bytes:
    """A fresh communicator id (spmm_comm_unique_id): make it on one rank, send the bytes to all."""
    buf = (C.c_uint8 * COMM_ID_BYTES)()
    check(lib().spmm_comm_unique_id(buf), "spmm_comm_unique_id")
    return bytes(buf)


class RankComm:
    """spmm_comm_*: this process's member of an NCCL communicator over `world` ranks (one GPU each;
    the current device is this rank's)."""

    def __init__(self, comm_id: bytes, world: int, rank: int, timeout_ms: int = 0):
        if len(comm_id) != COMM_ID_BYTES:
            raise ValueError("communicator id must be 128 bytes")
        buf = (C.c_uint8 * COMM_ID_BYTES).from_buffer_copy(comm_id)
        h = C.c_void_p()
        check(lib().spmm_comm_init(buf, world, rank, timeout_ms, C.byref(h)), "spmm_comm_init")
        self._h = h
        w, r, d = C.c_int32(), C.c_int32(), C.c_int32()
        lib().spmm_comm_info(h, C.byref(w), C.byref(r), C.byref(d))
        self.world, self.rank, self.device = int(w.value), int(r.value), int(d.value)

    @property
    def handle(self):
        return self._h

    def close(self) -> None:
        if self._h:
            lib().spmm_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class RankPlan:
    """spmm_rank_plan_*: this rank's share of C = A @ B under the reference's nnz-balanced row split.

    A is the whole host CSR (the same on every rank); comm None is a world of one. run() is the
    end-to-end multiply from host buffers (collective), execute() the kernels alone on the
    device-resident operands the last run() left."""

    def __init__(self, comm: RankComm | None, A: HostCSR, N: int, stream=None):
        self._comm = comm
        self._A = A
        self.N = N
        v = A.view()
        h = C.c_void_p()
        check(lib().spmm_rank_plan_create(comm.handle if comm else None, C.byref(v), N, stream_ptr(stream),
                                          C.byref(h)), "spmm_rank_plan_create")
        self._h = h
        vals = [C.c_int32() for _ in range(7)]
        check(lib().spmm_rank_plan_info(h, *[C.byref(x) for x in vals]), "spmm_rank_plan_info")
        (self.row_begin, self.row_end, self.nnz, self.b_row_begin, self.b_row_end, self.algo,
         self.launches) = (int(x.value) for x in vals)
        dB, dC = C.c_void_p(), C.c_void_p()
        check(lib().spmm_rank_plan_buffers(h, C.byref(dB), C.byref(dC)), "spmm_rank_plan_buffers")
        self.d_B, self.d_C = int(dB.value or 0), int(dC.value or 0)

    @property
    def rows(self) -> int:
        return self.row_end - self.row_begin

    def run(self, A: HostCSR, B: np.ndarray, C_rows: np.ndarray, stream=None) -> None:
        v = A.view()
        check(lib().spmm_rank_run(self._h, C.byref(v), ptr(B), ptr(C_rows), stream_ptr(stream)), "spmm_rank_run")

    def submit(self, A: HostCSR, B: np.ndarray, C_rows: np.ndarray, stream=None) -> None:
        """run() without the wait; the arrays must stay alive and unchanged until wait()."""
        v = A.view()
        check(lib().spmm_rank_submit(self._h, C.byref(v), ptr(B), ptr(C_rows), stream_ptr(stream)),
              "spmm_rank_submit")

    def wait(self, stream=None) -> None:
        check(lib().spmm_rank_wait(self._h, stream_ptr(stream)), "spmm_rank_wait")

    def execute(self, stream=None) -> None:
        check(lib().spmm_rank_execute(self._h, stream_ptr(stream)), "spmm_rank_execute")

    def gather_b(self, stream=None) -> None:
        check(lib().spmm_rank_gather_b(self._h, stream_ptr(stream)), "spmm_rank_gather_b")

    def close(self) -> None:
        if self._h:
            lib().spmm_rank_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass
