"""GPU CSR -> BSR-16 conversion (spmm_csr_to_bsr16_device_*) against the host conversion,
which the CPU tests pin to the reference's bsr_from_csr_host bit for bit: row_ptr, col_idx
and every 16-bit value must be identical."""
from __future__ import annotations

import numpy as np
import pytest

import _cases as K
import spmm_b200 as S
import spmm_patterns as SP

pytestmark = pytest.mark.gpu


def device_bsr(torch, A: S.HostCSR, dtype: int):
    dev = torch.device("cuda")
    rp, ci, v = (torch.from_numpy(x).to(dev) for x in (A.row_ptr, A.col_idx, A.values))
    view = S.device_view(A.rows, A.cols, rp, ci, v)
    bview, (brp, bci, bva) = S.csr_to_bsr16_device(view, dtype, torch.cuda.current_stream())
    torch.cuda.synchronize()
    n = bview.num_blocks
    return (brp.cpu().numpy(), bci.cpu().numpy()[:n], bva.cpu().numpy().view(np.uint16)[: n * 256], n)


def assert_same(torch, A: S.HostCSR, dtype=S.DTYPE_F16):
    h = S.csr_to_bsr16(A, dtype)
    rp, ci, vals, n = device_bsr(torch, A, dtype)
    assert n == h.num_blocks
    assert np.array_equal(rp, h.row_ptr)
    assert np.array_equal(ci, h.col_idx)
    assert np.array_equal(vals, h.values)


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4"])
@pytest.mark.parametrize("dtype", [S.DTYPE_F16, S.DTYPE_BF16])
def test_configs(cuda, name, dtype):
    A = S.generate_uniform_csr(4096, 4096, 0.01, 42) if name == "c1" else SP.config(name)[0]
    assert_same(cuda, A, dtype)


def test_ragged_and_empty(cuda):
    for M, Kc in [(1, 1), (17, 33), (1000, 999), (300, 70000)]:
        lens = np.random.default_rng(M).integers(0, min(Kc, 50), size=M)
        lens[::5] = 0
        assert_same(cuda, K.random_csr(M, Kc, lens, seed=M))
    assert_same(cuda, K.random_csr(40, 40, np.zeros(40, np.int64), seed=1))


def test_duplicates_last_wins_and_rounding_edges(cuda):
    # Sorted rows with repeated coordinates (the reference keeps duplicates; the last wins)
    # and values at FP16 rounding boundaries.
    rows = np.array([0, 0, 0, 1, 1, 5, 5, 5, 17, 17], np.int32)
    cols = np.array([3, 3, 20, 0, 0, 5, 6, 6, 31, 40], np.int32)
    vals = np.array([1.0, 2.0, 65519.99, 1e-8, 2.98024e-8, 65520.0, -0.0, 1.0 + 2**-11, 6.1e-5, np.inf],
                    np.float32)
    A = S.csr_from_coo(18, 41, rows, cols, vals)
    for dt in (S.DTYPE_F16, S.DTYPE_BF16):
        assert_same(cuda, A, dt)


def test_unsorted_rows_are_refused(cuda):
    torch = cuda
    A = K.random_csr(32, 64, np.full(32, 5), seed=2)
    ci = A.col_idx.copy()
    ci[A.row_ptr[7]], ci[A.row_ptr[7] + 1] = ci[A.row_ptr[7] + 1], ci[A.row_ptr[7]]
    B = S.HostCSR(A.rows, A.cols, A.row_ptr, ci, A.values)
    with pytest.raises(S.SpmmError) as e:
        device_bsr(torch, B, S.DTYPE_F16)
    assert e.value.status == -6
    bad = S.HostCSR(A.rows, A.cols, A.row_ptr, A.col_idx.copy(), A.values)
    bad.col_idx[3] = 64
    with pytest.raises(S.SpmmError) as e:
        device_bsr(torch, bad, S.DTYPE_F16)
    assert e.value.status == -8
