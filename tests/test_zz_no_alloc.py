"""spmm_csr_f32_noalloc -- the CSR SpMM for callers that cannot allocate device memory.

Some callers cannot let a library call cudaMalloc (a host whose allocator or memory budget
owns all device memory, a loop that cannot afford cudaMalloc's implicit synchronisation);
this entry point uses a fixed 16 MiB scratch array compiled into the library instead of an
allocated workspace. The test calls it through the C ABI and checks it against the existing
entry point, spmm_csr_f32, with the bar the other CSR tests use (bit equality), on two calls
in a row; then checks that an oversized request is refused with SPMM_ERR_TOO_LARGE.

This file is named so that pytest collects it last; it must also pass alone in a fresh
process (python -m pytest tests/test_zz_no_alloc.py -m gpu).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import _cases as K
import spmm_b200 as S

pytestmark = pytest.mark.gpu


def _noalloc(view, B, Cout, N, algo, stream):
    return S.lib().spmm_csr_f32_noalloc(ctypes.byref(view), S.ptr(B), S.ptr(Cout), N, algo, S.stream_ptr(stream))


def test_noalloc_matches_allocating_entry_point_twice(cuda):
    torch = cuda
    # Power-law rows (up to 14850 nonzeros) so the scratch's long-row slots are exercised.
    A, Bh = K.config("c4")
    N = Bh.shape[1]
    dev = torch.device("cuda")
    rp, ci, v = (torch.from_numpy(x).to(dev) for x in (A.row_ptr, A.col_idx, A.values))
    B = torch.from_numpy(Bh).to(dev)
    view = S.device_view(A.rows, A.cols, rp, ci, v)
    stream = torch.cuda.current_stream()

    need = S.csr_workspace_size(view, N, S.CSR_AUTO)
    assert 0 < need <= 16 << 20

    want = torch.empty((A.rows, N), dtype=torch.float32, device=dev)
    S.csr_f32(view, B, want, N, S.CSR_AUTO, stream)
    torch.cuda.synchronize()

    for call in range(2):
        got = torch.full((A.rows, N), float("nan"), dtype=torch.float32, device=dev)
        rc = _noalloc(view, B, got, N, S.CSR_AUTO, stream)
        assert rc == 0, f"call {call}: {S.status_string(rc)}"
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int32), want.view(torch.int32)), f"call {call} differs"

    # The warp-per-row variant needs no scratch and must agree as well.
    want_rw = torch.empty_like(want)
    S.csr_f32(view, B, want_rw, N, S.CSR_ROWWARP, stream)
    got_rw = torch.empty_like(want)
    assert _noalloc(view, B, got_rw, N, S.CSR_ROWWARP, stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(got_rw.view(torch.int32), want_rw.view(torch.int32))


def test_noalloc_refuses_requests_beyond_its_scratch(cuda):
    torch = cuda
    # 4M rows and 64M nonzeros at N = 512 need far more than 16 MiB of workspace; the call
    # is refused on the host before anything is launched, so the pointers are never read.
    dummy = torch.empty(16, dtype=torch.float32, device="cuda")
    view = S.CsrView(4 << 20, 4 << 20, 64 << 20, S.ptr(dummy), S.ptr(dummy), S.ptr(dummy))
    rc = _noalloc(view, dummy, dummy, 512, S.CSR_AUTO, torch.cuda.current_stream())
    assert rc == -10  # SPMM_ERR_TOO_LARGE
    assert _noalloc(view, dummy, dummy, -1, S.CSR_AUTO, None) == -1
    # A null B (or C) is an invalid argument, reported before the size check and before
    # anything is queued on the stream.
    assert _noalloc(view, None, dummy, 512, S.CSR_AUTO, None) == -1
    assert _noalloc(view, dummy, None, 512, S.CSR_AUTO, None) == -1
