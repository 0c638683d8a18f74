"""Host side of the product on the CPU (no GPU): the C ABI loads and exports every symbol
include/spmm_c.h declares; generators, COO->CSR, slicing, binary IO, BSR conversion, stats,
bounds and the hybrid decision equal the oracle (and so the reference) bit for bit; device
entry points fail loudly without a GPU instead of falling back."""
from __future__ import annotations

import ctypes
import json
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import _cases as K
import spmm_b200 as S
import spmm_patterns as SP
from oracle import oracle as O

REPO = Path(__file__).resolve().parent.parent
GOLDEN = json.loads((REPO / "tests" / "golden" / "golden.json").read_text())


def declared_functions() -> list[str]:
    text = (REPO / "include" / "spmm_c.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(spmm_[a-z0-9_]+)\s*\(", text)))


def test_c_abi_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 30
    L = S.lib()
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/spmm_c.h but not exported"
    assert sorted(S.EXPORTS) == names


def test_probe_library_loads_and_exports():
    import ctypes

    so = S.LIB_PATH.parent / "libspmm_probe.so"
    L = ctypes.CDLL(str(so))
    for n in ("spmm_probe_ctas", "spmm_probe_gather", "spmm_probe_gather_rows"):
        assert hasattr(L, n)


def test_cxx_api_library_exports_reference_symbols():
    out = subprocess.run(["nm", "-DC", "--defined-only", str(S.CXX_LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    for sym in ["spmm::csr_alloc_host(int, int, int)", "spmm::csr_free_host(spmm::CSR&)",
                "spmm::generate_uniform_random_csr(int, int, float, int)",
                "spmm::csr_row_slice_host(spmm::CSR const&, int, int)", "spmm::csr_to_device(spmm::CSR const&)",
                "spmm::bsr_from_csr_host(spmm::CSR const&)", "spmm::bsr_compute_stats(spmm::BSR_host const&)",
                "spmm::spmm_baseline(spmm::CSR const&, float const*, float*, int)",
                "spmm::spmm_tiled_v3(spmm::CSR const&, float const*, float*, int)",
                "spmm::spmm_wmma(spmm::BSR const&, __half const*, float*, int)",
                "spmm::float_to_half(float const*, __half*, int)",
                "spmm::hybrid_choose(spmm::CSR const&, int, float)", "spmm::backend_name(spmm::Backend)",
                "spmm::gpu_count()", "spmm::spmm_multigpu(spmm::CSR const&, float const*, float*, int, int, int, int)",
                "spmm::spmm_unified(spmm::CSR const&, float const*, float*, int, int, int)"]:
        assert sym in out, sym


@pytest.mark.parametrize("rows,cols,d,seed", [(1024, 1024, 0.05, 42), (4096, 4096, 0.01, 42), (333, 777, 0.2, 5),
                                              (64, 64, 1.0, 1), (10, 20, 0.0, 3), (1, 100000, 0.01, 9),
                                              (2000, 1, 0.5, 11)])
def test_generator_bit_identical(rows, cols, d, seed):
    a = S.generate_uniform_csr(rows, cols, d, seed)
    o = O.gen_uniform_csr(rows, cols, d, seed)
    assert np.array_equal(a.row_ptr, o.row_ptr) and np.array_equal(a.col_idx, o.col_idx)
    assert np.array_equal(a.values.view(np.uint32), o.values.view(np.uint32))


def test_generator_known_answer_16384():
    assert S.generate_uniform_csr(16384, 16384, 0.01, 42).nnz == GOLDEN["sweep_nnz"]["16384/0.01"]


def test_generator_rejects_bad_density():
    for d in (-0.1, 1.5, float("nan")):
        with pytest.raises(S.SpmmError) as e:
            S.generate_uniform_csr(10, 10, d, 1)
        assert e.value.status == -1


@pytest.mark.parametrize("rows,cols,d", [(4096, 4096, 0.01), (2000, 300, 0.3), (50, 100000, 0.001), (64, 64, 1.0),
                                         (10, 20, 0.0), (3, 0, 0.5), (0, 10, 0.5)])
def test_fast_generator_structure_and_thread_independence(rows, cols, d):
    a = S.generate_uniform_csr_fast(rows, cols, d, 1234, threads=1)
    b = S.generate_uniform_csr_fast(rows, cols, d, 1234, threads=7)
    assert np.array_equal(a.row_ptr, b.row_ptr) and np.array_equal(a.col_idx, b.col_idx)
    assert np.array_equal(a.values.view(np.uint32), b.values.view(np.uint32))
    assert a.row_ptr[0] == 0 and np.all(np.diff(a.row_ptr) >= 0) and a.row_ptr[-1] == a.nnz
    if a.nnz:
        assert a.col_idx.min() >= 0 and a.col_idx.max() < cols
        assert np.all(a.values >= -1.0) and np.all(a.values < 1.0)
        rows_of = np.repeat(np.arange(rows), np.diff(a.row_ptr))
        same_row = rows_of[1:] == rows_of[:-1]
        assert np.all(np.diff(a.col_idx)[same_row] > 0), "columns strictly increase inside a row"
    mean = rows * cols * d
    sd = np.sqrt(rows * cols * d * (1 - d))
    assert abs(a.nnz - mean) <= 6 * sd + 1e-9
    if d == 1.0:
        assert a.nnz == rows * cols


def test_fast_generator_is_uniform_and_seeded():
    a = S.generate_uniform_csr_fast(8192, 8192, 0.005, 99)
    # Column and row occupancy: chi-square over 64 equal buckets, far from the 1e-6 tail.
    for idx, n in ((a.col_idx, 8192), (np.repeat(np.arange(8192), np.diff(a.row_ptr)), 8192)):
        counts = np.bincount(idx * 64 // n, minlength=64)
        exp = a.nnz / 64
        chi2 = float(((counts - exp) ** 2 / exp).sum())
        assert chi2 < 140, chi2  # 63 d.o.f.: P(chi2 > 140) < 1e-7
    # Row lengths follow Binomial(cols, d): mean and variance.
    lens = np.diff(a.row_ptr)
    assert abs(lens.mean() - 8192 * 0.005) < 0.3
    assert abs(lens.var() / (8192 * 0.005 * 0.995) - 1) < 0.1
    # Values U[-1,1): mean ~0, variance ~1/3.
    assert abs(a.values.mean()) < 0.01 and abs(a.values.var() - 1 / 3) < 0.01
    c = S.generate_uniform_csr_fast(8192, 8192, 0.005, 100)
    assert c.nnz != a.nnz or not np.array_equal(c.col_idx, a.col_idx)


def test_fast_generator_config5_size_quickly():
    import time
    t = time.perf_counter()
    a = S.generate_uniform_csr_fast(131072, 131072, 0.001, 42)
    dt = time.perf_counter() - t
    assert abs(a.nnz - 17179869) < 6 * np.sqrt(17179869)
    assert dt < 30, dt


def test_fast_generator_rejects_bad_density():
    for d in (-0.1, 1.5, float("nan")):
        with pytest.raises(S.SpmmError) as e:
            S.generate_uniform_csr_fast(10, 10, d, 1)
        assert e.value.status == -1


def test_dense_bit_identical():
    for r, c, s in [(4096, 64, 43), (123, 45, 9), (1, 1, 0)]:
        assert np.array_equal(S.generate_dense(r, c, s).view(np.uint32), O.gen_dense(r, c, s).view(np.uint32))


def test_coo_to_csr_with_duplicates():
    rng = np.random.default_rng(3)
    r = rng.integers(0, 50, 3000).astype(np.int32)
    c = rng.integers(0, 40, 3000).astype(np.int32)
    v = rng.uniform(-1, 1, 3000).astype(np.float32)
    a, o = S.csr_from_coo(50, 40, r, c, v), O.csr_from_coo(50, 40, r, c, v)
    assert np.array_equal(a.row_ptr, o.row_ptr) and np.array_equal(a.col_idx, o.col_idx)
    assert np.array_equal(a.values.view(np.uint32), o.values.view(np.uint32))
    with pytest.raises(S.SpmmError):
        S.csr_from_coo(5, 5, np.array([7], np.int32), np.array([0], np.int32), np.array([1.0], np.float32))


def test_row_slice_and_binary_round_trip(tmp_path):
    A = S.generate_uniform_csr(500, 300, 0.03, 4)
    for b, e in [(0, 500), (0, 0), (17, 230), (499, 500)]:
        s, o = S.row_slice(A, b, e), O.row_slice(K.to_oracle(A), b, e)
        assert np.array_equal(s.row_ptr, o.row_ptr) and np.array_equal(s.col_idx, o.col_idx)
        assert np.array_equal(s.values, o.values)
    with pytest.raises(S.SpmmError):
        S.row_slice(A, 10, 5)
    f = tmp_path / "a.bin"
    S.write_binary(A, f)
    raw = f.read_bytes()
    hdr = np.frombuffer(raw[:12], "<i4")
    assert hdr.tolist() == [500, 300, A.nnz] and len(raw) == 12 + 4 * 501 + 8 * A.nnz
    B = S.read_binary(f)
    assert np.array_equal(B.row_ptr, A.row_ptr) and np.array_equal(B.values, A.values)
    f.write_bytes(raw[:-4])  # short body
    with pytest.raises(S.SpmmError) as e:
        S.read_binary(f)
    assert e.value.status == -9
    with pytest.raises(S.SpmmError):
        S.read_binary(tmp_path / "missing.bin")


def test_validate():
    A = S.generate_uniform_csr(100, 50, 0.1, 1)
    assert S.validate(A) == -1
    bad = S.HostCSR(A.rows, A.cols, A.row_ptr.copy(), A.col_idx.copy(), A.values)
    bad.col_idx[A.row_ptr[40]] = 50
    assert S.validate(bad) == 40
    bad2 = S.HostCSR(A.rows, A.cols, A.row_ptr.copy(), A.col_idx, A.values)
    bad2.row_ptr[20], bad2.row_ptr[21] = bad2.row_ptr[21] + 1, bad2.row_ptr[20]
    assert S.validate(bad2) in (19, 20)


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4"])
def test_bsr_conversion_bit_identical(name):
    A = SP.config(name)[0] if name != "c1" else S.generate_uniform_csr(4096, 4096, 0.01, 42)
    b = S.csr_to_bsr16(A)
    o = O.bsr_from_csr(K.to_oracle(A))
    assert np.array_equal(b.row_ptr, o.row_ptr) and np.array_equal(b.col_idx, o.col_idx)
    assert np.array_equal(b.values, o.values)
    st, ost = S.bsr_stats(b), O.bsr_stats(o)
    assert st == ost
    want = {"c1": 60630, "c2": 3572, "c3": 4096}
    if name in want:
        assert st["num_blocks"] == want[name]


def test_bsr_rounding_edges_and_bf16():
    edge = np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, -70000.0, 1e-8, 2.98023e-8, 2.98024e-8, 5.96e-8,
                     6.1035e-5, 6.1e-5, 1.0 + 2**-11, 1.0 + 3 * 2**-11, 0.333333, np.inf, -np.inf, 1e-45, 3.0e38,
                     -1.17549435e-38], np.float32)
    n = edge.size
    A = S.HostCSR(1, n, np.array([0, n], np.int32), np.arange(n, dtype=np.int32), edge)
    at = (np.arange(n) // 16) * 256 + np.arange(n) % 16  # element (0, c % 16) of block c // 16
    b = S.csr_to_bsr16(A, S.DTYPE_F16)
    assert np.array_equal(b.values[at], O.to_half_bits(edge))
    bb = S.csr_to_bsr16(A, S.DTYPE_BF16)
    assert np.array_equal(bb.values[at], O.to_half_bits(edge, bf16=True))


def test_bounds_bit_identical():
    cases = [S.generate_uniform_csr(4096, 4096, 0.01, 42), K.random_csr(100, 10, np.zeros(100, np.int64), 1),
             K.random_csr(50, 1000, [0] * 20 + [900] + [0] * 29, 2), K.random_csr(7, 100, [3, 0, 9, 9, 0, 1, 50], 3)]
    for A in cases:
        for G in (1, 2, 3, 4, 8, 9, 64):
            assert np.array_equal(S.nnz_balanced_bounds(A.row_ptr, A.rows, A.nnz, G),
                                  O.nnz_balanced_bounds(K.to_oracle(A), G))
    for key, want in GOLDEN["bounds"].items():
        A = cases[0]
        G = int(key.rsplit("G", 1)[1])
        assert S.nnz_balanced_bounds(A.row_ptr, A.rows, A.nnz, G).tolist() == want


def test_product_patterns_match_reference_digests():
    import hashlib

    def digest(*arrays):
        h = hashlib.sha256()
        for a in arrays:
            h.update(np.ascontiguousarray(a).tobytes())
        return h.hexdigest()

    makers = {"banded": SP.banded_arrays, "block-diagonal": SP.block_diagonal_arrays,
              "power-law": SP.power_law_arrays, "uniform": SP.uniform_mask_arrays}
    for name, g in GOLDEN["patterns"].items():
        kw = g["kw"]
        args = {"banded": (kw.get("bandwidth"),), "block-diagonal": (kw.get("block"),),
                "power-law": (kw.get("mean_deg"), kw.get("alpha")), "uniform": (kw.get("density"),)}[g["pattern"]]
        rp, ci, v = makers[g["pattern"]](g["rows"], g["cols"], *args, g["seed"])
        assert digest(rp.astype("<i4"), ci.astype("<i4"), v.astype("<f4")) == g["sha256"], name


def test_hybrid_decisions():
    # Reference rule: TC iff N % 16 == 0 and fill-in <= threshold (default 2.0).
    A1 = S.generate_uniform_csr(4096, 4096, 0.01, 42)
    p = S.hybrid_choose(A1, 64)
    assert p["backend_name"] == "csr" and abs(p["fill_in_ratio"] - 92.5616) < 1e-3
    A2 = SP.config("c2")[0]
    p = S.hybrid_choose(A2, 128)
    assert p["backend_name"] == "wmma" and abs(p["fill_in_ratio"] - 1.348) < 1e-3
    assert S.hybrid_choose(A2, 100)["reason"] == "N not a multiple of 16 -> CUDA-core CSR"
    assert S.hybrid_choose(A2, 128, 1.2)["backend_name"] == "csr"
    A3 = SP.config("c3")[0]
    assert S.hybrid_choose(A3, 256)["backend_name"] == "wmma"


def test_device_entry_points_fail_loudly_without_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    A = S.generate_uniform_csr(10, 10, 0.5, 1)
    B = np.zeros((10, 4), np.float32)
    C = np.zeros((10, 4), np.float32)
    with pytest.raises(S.SpmmError) as e:
        S.csr_f32_host(A, B, C, 4)
    assert e.value.status == -6  # SPMM_ERR_UNSUPPORTED, never a silent CPU fallback
    assert S.gpu_count() == 0
    # The per-rank multi-GPU path refuses as well, with or without a communicator.
    with pytest.raises(S.SpmmError) as e:
        S.RankPlan(None, A, 4)
    assert e.value.status == -6
    with pytest.raises(S.SpmmError) as e:
        S.RankComm(bytes(S.COMM_ID_BYTES), 2, 0, timeout_ms=1000)
    assert e.value.status == -6


def test_status_strings():
    L = S.lib()
    for code in [0, -1, -2, -3, -4, -5, -6, -7, -8, -9, -10]:
        assert L.spmm_status_string(code).decode() not in ("", "unknown status")
    assert L.spmm_version() >= 100


def test_c_abi_argument_validation():
    L = S.lib()
    v = S.CsrView(-1, 5, 0, 0, 0, 0)
    assert L.spmm_nnz_balanced_bounds(None, 5, 0, 0, None) == -1
    out = (ctypes.c_int32 * 3)()
    assert L.spmm_nnz_balanced_bounds(None, 0, 0, 2, out) == 0 and list(out) == [0, 0, 0]
    assert L.spmm_csr_validate_host(ctypes.byref(v), None) == -1
