"""GPU parity of the BSR-16 tensor-core path (tcgen05) and the FP32 -> FP16/BF16 conversion.

Tolerances (BASELINE: "FP16/BF16 BSR output within 1e-2 relative to an FP32 result"):
  * against the FP64 oracle on the same 16-bit-rounded inputs (the arithmetic the tensor
    cores are asked to do): max |err| / max |ref| <= 1e-5 and compare()'s filtered max
    relative error <= 1e-3 -- products are exact, only the FP32 accumulation rounds;
  * against the FP32 CSR result on the unrounded inputs: rel_l2 <= 1e-2.
"""
from __future__ import annotations

import numpy as np
import pytest

import _cases as K
import spmm_b200 as S
from oracle import oracle as O
from oracle import patterns as P

pytestmark = pytest.mark.gpu


def run_bsr(torch, Hb: S.HostBSR, B16: np.ndarray, N: int, algo: int = 0, c_off: int = 0):
    dev = torch.device("cuda")
    brp = torch.from_numpy(Hb.row_ptr).to(dev)
    bci = torch.from_numpy(Hb.col_idx).to(dev)
    bva = torch.from_numpy(Hb.values.view(np.int16)).to(dev)
    Bt = torch.from_numpy(np.ascontiguousarray(B16).view(np.int16)).to(dev)
    Cbuf = torch.full((Hb.rows * N + c_off + 4,), float("nan"), dtype=torch.float32, device=dev)
    view = Hb.view()
    view.row_ptr, view.col_idx, view.values = S.ptr(brp), S.ptr(bci), S.ptr(bva)
    S.bsr16(view, Bt, Cbuf[c_off:], N, algo, torch.cuda.current_stream())
    torch.cuda.synchronize()
    code, detail = S.device_error(0)
    assert code == 0, f"device error {code} ({detail})"
    return Cbuf[c_off:c_off + Hb.rows * N].view(Hb.rows, N).cpu().numpy()


def check_bsr(got: np.ndarray, Hb: S.HostBSR, B16: np.ndarray, dtype: int):
    ob = O.BSR(Hb.rows, Hb.cols, Hb.block_rows, Hb.block_cols, Hb.row_ptr, Hb.col_idx, Hb.values, Hb.nnz)
    ref = O.spmm_bsr_f64(ob, B16, dtype)
    scale = max(float(np.abs(ref).max()), 1e-30)
    assert float(np.abs(got - ref).max()) / scale <= 1e-5
    _, max_rel, _ = O.compare(got, ref.astype(np.float32))
    assert max_rel <= 1e-3
    return ref


@pytest.mark.parametrize("dtype", [S.DTYPE_F16, S.DTYPE_BF16])
def test_config3_block_diagonal(cuda, dtype):
    A, Bf = K.config("c3")
    Hb = S.csr_to_bsr16(A, dtype)
    st = S.bsr_stats(Hb)
    assert st["num_blocks"] == 4096 and st["fill_in_ratio"] == 1.0
    B16 = O.to_half_bits(Bf, bf16=dtype == S.DTYPE_BF16)
    got = run_bsr(cuda, Hb, B16, 256, algo=1)
    check_bsr(got, Hb, B16, dtype)
    # Against the FP32 CSR product of the unrounded inputs.
    c32 = O.spmm_csr_f32(K.to_oracle(A), Bf)
    assert np.linalg.norm(got - c32) / np.linalg.norm(c32) <= 1e-2


@pytest.mark.parametrize("algo", [1, 2])
def test_config2_banded(cuda, algo):
    A, Bf = K.config("c2")
    Hb = S.csr_to_bsr16(A)
    assert Hb.num_blocks == 3572
    B16 = O.to_half_bits(Bf)
    check_bsr(run_bsr(cuda, Hb, B16, 128, algo=algo), Hb, B16, S.DTYPE_F16)


@pytest.mark.parametrize("M,Kc,N", [(16, 16, 8), (33, 47, 24), (100, 70, 136), (1000, 999, 128), (257, 4096, 256),
                                    (2048, 512, 40)])
@pytest.mark.parametrize("algo", [1, 2])
def test_ragged_shapes(cuda, M, Kc, N, algo):
    A = K.random_csr(M, Kc, np.random.default_rng(M).integers(0, min(Kc, 40), size=M), seed=M + Kc)
    Hb = S.csr_to_bsr16(A)
    B16 = O.to_half_bits(K.dense(Kc, N, 3))
    check_bsr(run_bsr(cuda, Hb, B16, N, algo=algo), Hb, B16, S.DTYPE_F16)


@pytest.mark.parametrize("M,Kc,N", [(32768, 512, 128), (20000, 333, 136)])
def test_eight_block_rows_per_cta(cuda, M, Kc, N):
    # Enough block-rows that the launcher groups eight per CTA (>= one CTA per SM at G=8),
    # with skewed rows so the producer merges lists of very different lengths.
    lens = np.random.default_rng(M).integers(0, 12, size=M)
    lens[::97] = np.minimum(Kc, 300)
    A = K.random_csr(M, Kc, lens, seed=5)
    Hb = S.csr_to_bsr16(A)
    assert (Hb.block_rows + 7) // 8 * ((N + 127) // 128) >= 148
    B16 = O.to_half_bits(K.dense(Kc, N, 6))
    check_bsr(run_bsr(cuda, Hb, B16, N, algo=1), Hb, B16, S.DTYPE_F16)


def test_empty_block_rows_and_uniform_fill(cuda):
    # Uniform sparsity (high fill-in) with whole empty block-rows in between.
    lens = np.random.default_rng(1).integers(0, 30, size=512)
    lens[64:160] = 0
    A = K.random_csr(512, 2048, lens, seed=4)
    Hb = S.csr_to_bsr16(A)
    B16 = O.to_half_bits(K.dense(2048, 128, 5))
    for algo in (1, 2):
        check_bsr(run_bsr(cuda, Hb, B16, 128, algo=algo), Hb, B16, S.DTYPE_F16)


def test_unaligned_n_falls_back(cuda):
    A = K.random_csr(64, 64, np.full(64, 8), seed=1)
    Hb = S.csr_to_bsr16(A)
    B16 = O.to_half_bits(K.dense(64, 20, 2))
    with pytest.raises(S.SpmmError) as e:
        run_bsr(cuda, Hb, B16, 20, algo=1)  # tensor-core path demands N % 8 == 0
    assert e.value.status == -2
    check_bsr(run_bsr(cuda, Hb, B16, 20, algo=0), Hb, B16, S.DTYPE_F16)


@pytest.mark.parametrize("bf16", [False, True])
def test_convert_round_to_nearest_even(cuda, bf16):
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.uniform(-1, 1, 100003).astype(np.float32),
                        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e-8, 5.96e-8, 2.98e-8, 6.1e-5, 1e30, -1e30,
                                  np.inf, -np.inf, 1.0 + 2**-11, 1.0 + 3 * 2**-11, 3.0e38], np.float32)])
    torch = cuda
    src = torch.from_numpy(x).cuda()
    for off in (0, 1):  # vector and scalar kernels
        dst = torch.empty(x.size - off, dtype=torch.int16, device="cuda")
        S.convert_f32(src[off:], dst, x.size - off, S.DTYPE_BF16 if bf16 else S.DTYPE_F16,
                      torch.cuda.current_stream())
        torch.cuda.synchronize()
        got = dst.cpu().numpy().view(np.uint16)
        want = O.to_half_bits(x[off:], bf16=bf16)
        assert np.array_equal(got, want)


def _plan_run(torch, Hb: S.HostBSR, B16: np.ndarray, N: int):
    dev = torch.device("cuda")
    brp = torch.from_numpy(Hb.row_ptr).to(dev)
    bci = torch.from_numpy(Hb.col_idx).to(dev)
    bva = torch.from_numpy(Hb.values.view(np.int16)).to(dev)
    Bt = torch.from_numpy(np.ascontiguousarray(B16).view(np.int16)).to(dev)
    view = Hb.view()
    view.row_ptr, view.col_idx, view.values = S.ptr(brp), S.ptr(bci), S.ptr(bva)
    plan = S.BsrPlan(view, N, stream=torch.cuda.current_stream())
    outs = []
    for _ in range(2):  # the schedule is reused across executions
        Cd = torch.full((Hb.rows, N), float("nan"), device=dev)
        plan.execute(Bt, Cd, torch.cuda.current_stream())
        torch.cuda.synchronize()
        outs.append(Cd.cpu().numpy())
    code, detail = S.device_error(0)
    assert code == 0, f"device error {code} ({detail})"
    info = (plan.group, plan.max_steps, plan.schedule_bytes, plan.a_stride)
    plan.close()
    return outs, info


def _block_diagonal_with_extras(n: int, blk: int, extra_rows, seed: int) -> S.HostCSR:
    """Dense blk x blk diagonal blocks; each row in extra_rows also gets one nonzero three blocks
    to the right (another BSR block in its block-row)."""
    rng = np.random.default_rng(seed)
    row_ptr, cols = [0], []
    for i in range(n):
        d = i // blk
        c = list(range(d * blk, min((d + 1) * blk, n)))
        if i in extra_rows:
            c = sorted(set(c) | {(d * blk + 3 * blk + 5) % n})
        cols.extend(c)
        row_ptr.append(len(cols))
    vals = rng.uniform(-1, 1, size=len(cols)).astype(np.float32)
    return S.HostCSR(n, n, np.array(row_ptr, np.int32), np.array(cols, np.int32), vals)


@pytest.mark.parametrize("case", ["c3", "c3_bf16", "banded", "ragged_g8", "empty_groups", "n_tail", "diag_mixed"])
def test_plan_schedule_matches_per_call(cuda, case):
    # The precomputed per-CTA schedule gives the per-call kernel's result bit for bit, with
    # the grouped A copies where a step's blocks are evenly spaced and single-block copies
    # where they are not (diag_mixed: extra blocks shift and unbalance some block-rows, and
    # the last group of the grouped view is partial).
    dtype = S.DTYPE_BF16 if case == "c3_bf16" else S.DTYPE_F16
    if case.startswith("c3"):
        A, Bf = K.config("c3")
        N = 256
    elif case == "diag_mixed":
        A = _block_diagonal_with_extras(2048, 128, {5, 700, 1500}, seed=8)
        Bf, N = K.dense(2048, 256, 3), 256
    elif case == "banded":
        A, Bf = K.config("c2")
        N = 128
    elif case == "ragged_g8":
        lens = np.random.default_rng(2).integers(0, 12, size=32768)
        lens[::97] = 300
        A = K.random_csr(32768, 512, lens, seed=5)
        Bf, N = K.dense(512, 128, 6), 128
    elif case == "empty_groups":
        lens = np.random.default_rng(3).integers(0, 30, size=4096)
        lens[512:1536] = 0
        A = K.random_csr(4096, 2048, lens, seed=4)
        Bf, N = K.dense(2048, 192, 5), 192
    else:
        A = K.random_csr(1000, 999, np.random.default_rng(1).integers(0, 40, size=1000), seed=9)
        Bf, N = K.dense(999, 136, 2), 136
    Hb = S.csr_to_bsr16(A, dtype)
    B16 = O.to_half_bits(Bf, bf16=dtype == S.DTYPE_BF16)
    (c0, c1), (group, steps, nbytes, a_stride) = _plan_run(cuda, Hb, B16, N)
    assert group in (4, 8) and steps > 0 and nbytes > 0
    if case.startswith("c3") or case == "diag_mixed":
        assert a_stride == 8  # 8 blocks per block-row: a step's 4 blocks are 8 apart
        assert Hb.num_blocks == (1024 if case == "diag_mixed" else 4096) + (3 if case == "diag_mixed" else 0)
    want = run_bsr(cuda, Hb, B16, N, algo=1)
    assert np.array_equal(c0.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(c1.view(np.uint32), want.view(np.uint32))
    check_bsr(c0, Hb, B16, dtype)


def test_plan_falls_back_off_the_tensor_core_path(cuda):
    A = K.random_csr(64, 64, np.full(64, 8), seed=1)
    Hb = S.csr_to_bsr16(A)
    B16 = O.to_half_bits(K.dense(64, 20, 2))
    (c0, _), (group, _, nbytes, _) = _plan_run(cuda, Hb, B16, 20)  # N % 8 != 0: CUDA-core kernel
    assert group == 0 and nbytes == 0
    check_bsr(c0, Hb, B16, S.DTYPE_F16)
