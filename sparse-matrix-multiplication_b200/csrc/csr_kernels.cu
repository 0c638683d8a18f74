// FP32 CSR x dense SpMM on the B200 CUDA cores.
//
// Replaces the reference's CSR kernel family (src/kernels/spmm_baseline.cu ...
// spmm_tiled_v4.cu): same product, same per-element arithmetic (a sequential FP32 FMA chain
// over the row's nonzeros), new work distribution and memory access.
//
// The product is a gather: every nonzero (k, v) of row i reads the whole B row k (N floats)
// and adds v * B[k, :] into C[i, :]. On B200 that gather is served by L2 (B is re-read once
// per nonzero), so the kernels are built to keep many wide, coalesced B-row loads in flight:
//   * a warp owns a run of columns of one C row; each lane owns VEC consecutive columns per
//     R strides of 32*VEC, so one nonzero costs R vector loads per lane, all coalesced;
//   * the row's (col, val) pairs are fetched 32 at a time, one pair per lane, with the next
//     group prefetched while the current one is consumed; pairs reach the other lanes by
//     warp shuffle;
//   * U nonzeros' B-row loads are issued before their FMAs, in nonzero order, so the FMA
//     chain per element stays sequential (bit-identical to the reference's order).
//
// Two work distributions:
//   ROWWARP  one warp per row, grid-stride over rows.
//   MERGE    the merge-path item space (one item per row start plus one per nonzero,
//            item(r, p) = r + p) is cut into chunks of S items, one warp per chunk. A row
//            belongs to the chunk holding its first item. Rows with more than S nonzeros
//            ("long" rows) are cut at every multiple of S; each piece is summed from zero by
//            its chunk's warp, written to a workspace slot, and the last piece to arrive
//            (a per-row arrival counter) adds the pieces left to right and writes C. The
//            counter is reset by that last arrival, so the workspace is all-zero between
//            calls. No float atomics: results are deterministic.
//
// Every index read from A is range-checked; a bad index is recorded in the device error
// record and replaced by a harmless one, so malformed input cannot fault the GPU.

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"

namespace spmm_b200 {
namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kThreads = kWarpsPerCta * 32;
constexpr unsigned kFull = 0xffffffffu;

struct CsrArgs {
    int M, K, N;
    int nnz;
    const int* __restrict__ row_ptr;
    const int* __restrict__ col_idx;
    const float* __restrict__ values;
    const float* __restrict__ B;
    float* __restrict__ C;
    int S;               // merge-path chunk (items per warp) == long-row threshold
    long long items;     // M + nnz
    int num_chunks;
    int* counters;       // num_chunks, all-zero between calls
    float* partials;     // num_chunks * 2 * N
    DeviceErrorRecord* err;
};

template <int VEC> struct Vec;
template <> struct Vec<1> {
    using T = float;
    __device__ static T load(const float* p) { return __ldg(p); }
    __device__ static T loadcg(const float* p) { return __ldcg(p); }
    __device__ static void store_cs(float* p, T v) { __stcs(p, v); }
    __device__ static void store_cg(float* p, T v) { __stcg(p, v); }
    __device__ static float get(const T& v, int) { return v; }
    __device__ static void set(T& v, int, float x) { v = x; }
};
template <> struct Vec<2> {
    using T = float2;
    __device__ static T load(const float* p) { return __ldg(reinterpret_cast<const float2*>(p)); }
    __device__ static T loadcg(const float* p) { return __ldcg(reinterpret_cast<const float2*>(p)); }
    __device__ static void store_cs(float* p, T v) { __stcs(reinterpret_cast<float2*>(p), v); }
    __device__ static void store_cg(float* p, T v) { __stcg(reinterpret_cast<float2*>(p), v); }
    __device__ static float get(const T& v, int e) { return e == 0 ? v.x : v.y; }
    __device__ static void set(T& v, int e, float x) { if (e == 0) v.x = x; else v.y = x; }
};
template <> struct Vec<4> {
    using T = float4;
    __device__ static T load(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
    __device__ static T loadcg(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
    __device__ static void store_cs(float* p, T v) { __stcs(reinterpret_cast<float4*>(p), v); }
    __device__ static void store_cg(float* p, T v) { __stcg(reinterpret_cast<float4*>(p), v); }
    __device__ static float get(const T& v, int e) { return e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w; }
    __device__ static void set(T& v, int e, float x) {
        if (e == 0) v.x = x; else if (e == 1) v.y = x; else if (e == 2) v.z = x; else v.w = x;
    }
};

// Columns of lane `lane` in stride r of a pass starting at col0.
template <int VEC>
__device__ __forceinline__ int lane_col(int col0, int r, int lane) {
    return col0 + (r * 32 + lane) * VEC;
}

__device__ __forceinline__ int clampi(int x, int lo, int hi) { return x < lo ? lo : (x > hi ? hi : x); }

// Sum of v_p * B[col_p, cols] over p in [p0, p1) into acc (caller zeroes acc), as one
// sequential FMA chain per column.
template <int VEC, int R, int U>
__device__ __forceinline__ void accumulate(const CsrArgs& a, int p0, int p1, int col0, int lane,
                                           float (&acc)[R][VEC]) {
    using V = Vec<VEC>;
    bool ok[R];
#pragma unroll
    for (int r = 0; r < R; ++r) ok[r] = lane_col<VEC>(col0, r, lane) < a.N;

    const float* __restrict__ Bp = a.B + col0 + lane * VEC;
    int base = p0;
    int kk = 0;
    float vv = 0.f;
    if (base < p1 && lane < p1 - base) {
        kk = __ldcs(a.col_idx + base + lane);
        vv = __ldcs(a.values + base + lane);
    }
    while (base < p1) {
        const int cnt = min(32, p1 - base);
        // Prefetch the next group of (col, val) pairs.
        const int nbase = base + 32;
        int nk = 0;
        float nv = 0.f;
        if (nbase < p1 && lane < p1 - nbase) {
            nk = __ldcs(a.col_idx + nbase + lane);
            nv = __ldcs(a.values + nbase + lane);
        }
        if (lane < cnt && static_cast<unsigned>(kk) >= static_cast<unsigned>(a.K)) {
            record_device_error(a.err, SPMM_ERR_BAD_INDEX, static_cast<long long>(base + lane));
            kk = 0;
            vv = 0.f;
        }
        int q = 0;
        for (; q + U <= cnt; q += U) {
            typename V::T b[U][R];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int k = __shfl_sync(kFull, kk, q + u);
                const float* brow = Bp + static_cast<size_t>(k) * a.N;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if (ok[r]) b[u][r] = V::load(brow + r * 32 * VEC);
                    else b[u][r] = typename V::T{};
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const float v = __shfl_sync(kFull, vv, q + u);
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int e = 0; e < VEC; ++e) acc[r][e] = fmaf(v, V::get(b[u][r], e), acc[r][e]);
            }
        }
        for (; q < cnt; ++q) {
            const int k = __shfl_sync(kFull, kk, q);
            const float v = __shfl_sync(kFull, vv, q);
            const float* brow = Bp + static_cast<size_t>(k) * a.N;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (ok[r]) {
                    const typename V::T b = V::load(brow + r * 32 * VEC);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) acc[r][e] = fmaf(v, V::get(b, e), acc[r][e]);
                }
            }
        }
        base = nbase;
        kk = nk;
        vv = nv;
    }
}

template <int VEC, int R>
__device__ __forceinline__ void store_row(const CsrArgs& a, float* dst, int col0, int lane, const float (&acc)[R][VEC]) {
    using V = Vec<VEC>;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int c = lane_col<VEC>(col0, r, lane);
        if (c < a.N) {
            typename V::T t;
#pragma unroll
            for (int e = 0; e < VEC; ++e) V::set(t, e, acc[r][e]);
            V::store_cs(dst + c, t);
        }
    }
}

// Full row i: C[i, :] = A[i, :] * B.
template <int VEC, int R, int U>
__device__ __forceinline__ void full_row(const CsrArgs& a, int i, int rs, int re, int lane) {
    constexpr int W = 32 * VEC * R;
    float* crow = a.C + static_cast<size_t>(i) * a.N;
    for (int col0 = 0; col0 < a.N; col0 += W) {
        float acc[R][VEC];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[r][e] = 0.f;
        accumulate<VEC, R, U>(a, rs, re, col0, lane, acc);
        store_row<VEC, R>(a, crow, col0, lane, acc);
    }
}

// Row bounds clamped into [0, nnz] with re >= rs (malformed row_ptr is recorded).
__device__ __forceinline__ void row_bounds(const CsrArgs& a, int i, int& rs, int& re) {
    const int x = __ldg(a.row_ptr + i);
    const int y = __ldg(a.row_ptr + i + 1);
    rs = clampi(x, 0, a.nnz);
    re = clampi(y, rs, a.nnz);
    if ((x != rs || y != re) && (threadIdx.x & 31) == 0)
        record_device_error(a.err, SPMM_ERR_BAD_INDEX, -1 - static_cast<long long>(i));
}

template <int VEC, int R, int U>
__global__ void __launch_bounds__(kThreads) csr_rowwarp_kernel(CsrArgs a) {
    const int lane = threadIdx.x & 31;
    const int warp = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * kWarpsPerCta;
    for (int i = warp; i < a.M; i += nwarps) {
        int rs, re;
        row_bounds(a, i, rs, re);
        full_row<VEC, R, U>(a, i, rs, re, lane);
    }
}

// First row r in [0, M) with r + row_ptr[r] >= d (M if none), searched by the whole warp:
// 32 probes per round shrink the interval 33-fold.
__device__ __forceinline__ int warp_lower_bound(const CsrArgs& a, long long d, int lane) {
    int lo = 0, hi = a.M;  // answer in [lo, hi]
    while (hi > lo) {
        const int n = hi - lo;
        if (n <= 32) {
            const int r = lo + lane;
            const bool lt = lane < n && static_cast<long long>(r) + __ldg(a.row_ptr + r) < d;
            return lo + __popc(__ballot_sync(kFull, lt));
        }
        const int p = lo + static_cast<int>((static_cast<long long>(n) * (lane + 1)) / 33);
        const bool lt = static_cast<long long>(p) + __ldg(a.row_ptr + p) < d;
        const int k = __popc(__ballot_sync(kFull, lt));
        const int nlo = k > 0 ? __shfl_sync(kFull, p, max(k - 1, 0)) + 1 : lo;
        const int nhi = k < 32 ? __shfl_sync(kFull, p, min(k, 31)) : hi;
        lo = nlo;
        hi = max(nhi, nlo);
    }
    return lo;
}

// One piece [p0, p1) of long row i (rs..re); `slot` is this chunk's workspace slot.
template <int VEC, int R, int U>
__device__ __forceinline__ void long_piece(const CsrArgs& a, int i, int rs, int re, int p0, int p1, int slot, int lane) {
    using V = Vec<VEC>;
    constexpr int W = 32 * VEC * R;
    float* mine = a.partials + static_cast<size_t>(slot) * a.N;
    for (int col0 = 0; col0 < a.N; col0 += W) {
        float acc[R][VEC];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[r][e] = 0.f;
        accumulate<VEC, R, U>(a, p0, p1, col0, lane, acc);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int c = lane_col<VEC>(col0, r, lane);
            if (c < a.N) {
                typename V::T t;
#pragma unroll
                for (int e = 0; e < VEC; ++e) V::set(t, e, acc[r][e]);
                V::store_cg(mine + c, t);
            }
        }
    }
    // Publish the piece, then count arrivals on the row's first chunk.
    __threadfence();
    __syncwarp();
    const long long first_item = static_cast<long long>(i) + rs;
    const long long last_item = static_cast<long long>(i) + re - 1;
    const int ca = static_cast<int>(first_item / a.S);
    const int cb = static_cast<int>(last_item / a.S);
    const int pieces = cb - ca + 1;
    int prev = 0;
    if (lane == 0) prev = atomicAdd(a.counters + ca, 1);
    prev = __shfl_sync(kFull, prev, 0);
    if (prev != pieces - 1) return;
    // Last arrival: add the pieces in chunk order and write the row.
    __threadfence();
    float* crow = a.C + static_cast<size_t>(i) * a.N;
    for (int col0 = 0; col0 < a.N; col0 += W) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int c = lane_col<VEC>(col0, r, lane);
            if (c < a.N) {
                typename V::T s = V::loadcg(a.partials + static_cast<size_t>(2 * ca + 1) * a.N + c);
                for (int cc = ca + 1; cc <= cb; ++cc) {
                    const typename V::T t = V::loadcg(a.partials + static_cast<size_t>(2 * cc) * a.N + c);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) V::set(s, e, V::get(s, e) + V::get(t, e));
                }
                V::store_cs(crow + c, s);
            }
        }
    }
    if (lane == 0) a.counters[ca] = 0;
}

template <int VEC, int R, int U>
__global__ void __launch_bounds__(kThreads) csr_merge_kernel(CsrArgs a) {
    const int lane = threadIdx.x & 31;
    const int c = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    if (c >= a.num_chunks) return;
    const long long d0 = static_cast<long long>(c) * a.S;
    const long long d1 = min(d0 + a.S, a.items);
    const int r0 = warp_lower_bound(a, d0, lane);
    const int r1 = warp_lower_bound(a, d1, lane);

    // A long row that started in an earlier chunk and reaches into this one.
    if (r0 > 0) {
        const int q = r0 - 1;
        int qs, qe;
        row_bounds(a, q, qs, qe);
        if (qe - qs > a.S) {
            const int p0 = static_cast<int>(max(static_cast<long long>(qs), d0 - q));
            const int p1 = static_cast<int>(min(static_cast<long long>(qe), d1 - q));
            if (p0 < p1) long_piece<VEC, R, U>(a, q, qs, qe, p0, p1, 2 * c, lane);
        }
    }
    // Rows whose first item lies in this chunk.
    for (int i = r0; i < r1; ++i) {
        int rs, re;
        row_bounds(a, i, rs, re);
        if (re - rs <= a.S) {
            full_row<VEC, R, U>(a, i, rs, re, lane);
        } else {
            const int p1 = static_cast<int>(min(static_cast<long long>(re), d1 - i));
            long_piece<VEC, R, U>(a, i, rs, re, rs, max(p1, rs), 2 * c + 1, lane);
        }
    }
}

// ---------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------

struct Geometry {
    int vec = 1;
    int r = 1;
};

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

Geometry pick_geometry(const float* B, const float* C, int N, int col_pass) {
    Geometry g;
    const bool a16 = aligned(B, 16) && aligned(C, 16);
    const bool a8 = aligned(B, 8) && aligned(C, 8);
    if (N % 4 == 0 && a16 && (N >= 128 || col_pass >= 128)) g.vec = 4;
    else if (N % 2 == 0 && a8 && (N >= 64 || col_pass >= 64)) g.vec = 2;
    else g.vec = 1;
    const int want = col_pass > 0 ? col_pass : N;
    const int per = 32 * g.vec;
    int r = (want + per - 1) / per;
    const int rmax = g.vec == 1 ? 4 : 2;
    if (r > rmax) r = rmax;
    if (r == 3) r = 4;
    if (g.vec != 1 && r > 2) r = 2;
    if (r < 1) r = 1;
    g.r = r;
    return g;
}

int default_chunk(long long items, int sm_count) {
    // Aim at ~32 chunks per SM in one wave, in multiples of 32 items, within [64, 2048].
    const long long target = items / (static_cast<long long>(std::max(sm_count, 1)) * 32);
    long long s = ((target + 31) / 32) * 32;
    s = std::max<long long>(64, std::min<long long>(2048, s));
    return static_cast<int>(s);
}

int resolve_chunk(const spmm_csr_view* A, const spmm_csr_tuning* tune, int sm_count) {
    const long long items = static_cast<long long>(A->rows) + A->nnz;
    if (tune && tune->chunk > 0) return tune->chunk;
    return default_chunk(items, sm_count);
}

int check_view(const spmm_csr_view* A, const float* B, const float* C, int N) {
    if (!A || A->rows < 0 || A->cols < 0 || A->nnz < 0 || N < 0) return SPMM_ERR_INVALID_ARG;
    if (A->rows > 0 && !A->row_ptr) return SPMM_ERR_INVALID_ARG;
    if (A->nnz > 0 && (!A->col_idx || !A->values || A->cols == 0)) return SPMM_ERR_INVALID_ARG;
    if (A->rows > 0 && N > 0 && !C) return SPMM_ERR_INVALID_ARG;
    if (A->nnz > 0 && N > 0 && !B) return SPMM_ERR_INVALID_ARG;
    if (!aligned(B, 4) || !aligned(C, 4)) return SPMM_ERR_MISALIGNED;
    return SPMM_OK;
}

int check_tune(const spmm_csr_tuning* tune) {
    if (!tune) return SPMM_OK;
    if (tune->chunk != 0 && (tune->chunk < 64 || tune->chunk > 8192 || tune->chunk % 32)) return SPMM_ERR_INVALID_ARG;
    if (tune->col_pass != 0 && tune->col_pass != 32 && tune->col_pass != 64 && tune->col_pass != 128 &&
        tune->col_pass != 256)
        return SPMM_ERR_INVALID_ARG;
    return SPMM_OK;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

size_t merge_workspace_bytes(long long num_chunks, int N) {
    if (num_chunks <= 0) return 0;
    return align_up(static_cast<size_t>(num_chunks) * sizeof(int), 256) +
           static_cast<size_t>(num_chunks) * 2 * static_cast<size_t>(N) * sizeof(float);
}

template <int VEC, int R>
void launch_vr(int algo, const CsrArgs& a, int grid, cudaStream_t s) {
    constexpr int U = (R == 1) ? 8 : (R == 2 ? 4 : 2);
    if (algo == SPMM_CSR_ROWWARP) csr_rowwarp_kernel<VEC, R, U><<<grid, kThreads, 0, s>>>(a);
    else csr_merge_kernel<VEC, R, U><<<grid, kThreads, 0, s>>>(a);
}

void launch(const Geometry& g, int algo, const CsrArgs& a, int grid, cudaStream_t s) {
    switch (g.vec * 10 + g.r) {
        case 11: launch_vr<1, 1>(algo, a, grid, s); break;
        case 12: launch_vr<1, 2>(algo, a, grid, s); break;
        case 14: launch_vr<1, 4>(algo, a, grid, s); break;
        case 21: launch_vr<2, 1>(algo, a, grid, s); break;
        case 22: launch_vr<2, 2>(algo, a, grid, s); break;
        case 41: launch_vr<4, 1>(algo, a, grid, s); break;
        default: launch_vr<4, 2>(algo, a, grid, s); break;
    }
}

}  // namespace

// Shared by the C entry points below and by the no-workspace variants in other files.
int csr_f32_launch(const spmm_csr_view* A, const float* B, float* C, int32_t N, int32_t algo,
                   const spmm_csr_tuning* tune, void* ws, size_t ws_bytes, cudaStream_t stream,
                   DeviceState* st) {
    SPMM_TRY(check_view(A, B, C, N));
    SPMM_TRY(check_tune(tune));
    if (algo == SPMM_CSR_AUTO) algo = SPMM_CSR_MERGE;
    if (algo != SPMM_CSR_MERGE && algo != SPMM_CSR_ROWWARP) return SPMM_ERR_INVALID_ARG;
    if (A->rows == 0 || N == 0) return SPMM_OK;

    CsrArgs a{};
    a.M = A->rows;
    a.K = A->cols;
    a.N = N;
    a.nnz = A->nnz;
    a.row_ptr = A->row_ptr;
    a.col_idx = A->col_idx;
    a.values = A->values;
    a.B = B;
    a.C = C;
    a.err = st->err;
    const Geometry g = pick_geometry(B, C, N, tune ? tune->col_pass : 0);

    int grid = 0;
    if (algo == SPMM_CSR_ROWWARP) {
        const long long warps = std::min<long long>(A->rows, static_cast<long long>(st->sm_count) * 64);
        grid = static_cast<int>((warps + kWarpsPerCta - 1) / kWarpsPerCta);
    } else {
        a.S = resolve_chunk(A, tune, st->sm_count);
        a.items = static_cast<long long>(A->rows) + A->nnz;
        const long long chunks = (a.items + a.S - 1) / a.S;
        if (chunks > (1ll << 30)) return SPMM_ERR_TOO_LARGE;
        a.num_chunks = static_cast<int>(chunks);
        const size_t need = merge_workspace_bytes(chunks, N);
        if (need > ws_bytes || (need > 0 && !ws)) return SPMM_ERR_INVALID_ARG;
        a.counters = static_cast<int*>(ws);
        a.partials = reinterpret_cast<float*>(static_cast<char*>(ws) + align_up(static_cast<size_t>(chunks) * sizeof(int), 256));
        grid = static_cast<int>((chunks + kWarpsPerCta - 1) / kWarpsPerCta);
    }
    launch(g, algo, a, grid, stream);
    SPMM_CUDA_TRY(cudaGetLastError());
    return SPMM_OK;
}

int csr_f32_workspace_bytes(const spmm_csr_view* A, int32_t N, int32_t algo, const spmm_csr_tuning* tune,
                            int sm_count, size_t* bytes) {
    if (!A || !bytes || N < 0 || A->rows < 0 || A->nnz < 0) return SPMM_ERR_INVALID_ARG;
    SPMM_TRY(check_tune(tune));
    *bytes = 0;
    if (algo == SPMM_CSR_AUTO) algo = SPMM_CSR_MERGE;
    if (algo == SPMM_CSR_ROWWARP || A->rows == 0 || N == 0) return SPMM_OK;
    if (algo != SPMM_CSR_MERGE) return SPMM_ERR_INVALID_ARG;
    const int S = resolve_chunk(A, tune, sm_count);
    const long long items = static_cast<long long>(A->rows) + A->nnz;
    *bytes = merge_workspace_bytes((items + S - 1) / S, N);
    return SPMM_OK;
}

int csr_f32_chunk(const spmm_csr_view* A, const spmm_csr_tuning* tune, int sm_count) {
    return resolve_chunk(A, tune, sm_count);
}

}  // namespace spmm_b200

using namespace spmm_b200;

extern "C" {

int spmm_csr_f32_workspace_size(const spmm_csr_view* A, int32_t N, int32_t algo, const spmm_csr_tuning* tune,
                                size_t* bytes) {
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    return csr_f32_workspace_bytes(A, N, algo, tune, st->sm_count, bytes);
}

int spmm_csr_f32_chunk(const spmm_csr_view* A, int32_t N, int32_t algo, const spmm_csr_tuning* tune,
                       int32_t* chunk) {
    (void)N;
    (void)algo;
    if (!A || !chunk) return SPMM_ERR_INVALID_ARG;
    SPMM_TRY(check_tune(tune));
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    *chunk = csr_f32_chunk(A, tune, st->sm_count);
    return SPMM_OK;
}

int spmm_csr_f32_ws(const spmm_csr_view* A, const float* B, float* C, int32_t N, int32_t algo,
                    const spmm_csr_tuning* tune, void* ws, size_t ws_bytes, void* stream) {
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    return csr_f32_launch(A, B, C, N, algo, tune, ws, ws_bytes, as_stream(stream), st);
}

int spmm_csr_f32(const spmm_csr_view* A, const float* B, float* C, int32_t N, int32_t algo, void* stream) {
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    SPMM_TRY(check_view(A, B, C, N));
    size_t need = 0;
    SPMM_TRY(csr_f32_workspace_bytes(A, N, algo, nullptr, st->sm_count, &need));
    std::lock_guard<std::mutex> lock(st->mu);
    SPMM_TRY(ensure_device_buffer(&st->csr_ws, &st->csr_ws_bytes, need, true, as_stream(stream)));
    return csr_f32_launch(A, B, C, N, algo, nullptr, st->csr_ws, st->csr_ws_bytes, as_stream(stream), st);
}

}  // extern "C"
