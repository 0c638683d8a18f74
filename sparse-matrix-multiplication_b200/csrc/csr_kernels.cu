// FP32 CSR x dense SpMM on the B200 CUDA cores.
//
// Replaces the reference's CSR kernel family (src/kernels/spmm_baseline.cu ...
// spmm_tiled_v4.cu): same product, same per-element arithmetic (a sequential FP32 FMA chain
// over the row's nonzeros), new work distribution and memory access.
//
// The product is a gather: every nonzero (k, v) of row i reads B row k and adds v * B[k, :]
// into C[i, :]. B is re-read once per nonzero, so the kernels are built around the L2:
//   * column slabs: the grid's y dimension walks N in slabs of W <= 256 columns; CTAs are
//     issued slab by slab, so a narrower slab (tuning) keeps its B columns L2-resident at the
//     price of re-reading A. The streamed A arrays and C stores carry evict-first hints; B
//     loads are plain non-coherent loads by default (L2 evict-last variants are tunable);
//   * inside a slab a warp owns one C row: each lane holds VEC consecutive columns per stride,
//     R strides of 32*VEC columns (W = 32*VEC*R), so one nonzero costs R coalesced
//     VEC-wide loads per lane;
//   * the row's (col, val) pairs are fetched 32 at a time, one pair per lane, the next group
//     prefetched while the current one is consumed, and broadcast by warp shuffle;
//   * U nonzeros' B loads are issued before their FMAs, in nonzero order, so the FMA chain
//     per element stays sequential (bit-identical to the reference's order).
//
// Two work distributions:
//   ROWWARP  one warp per row, grid-stride over rows.
//   MERGE    the merge-path item space (one item per row start plus one per nonzero,
//            item(r, p) = r + p) is cut into chunks of S items, one warp per chunk. A row
//            belongs to the chunk holding its first item. Rows with more than S nonzeros
//            ("long" rows) are cut at every multiple of S; each piece is summed from zero by
//            its chunk's warp, written to a workspace slot, and the last piece to arrive
//            (a per-row, per-slab arrival counter) adds the pieces left to right and writes
//            C. That last arrival resets the counter, so the workspace is all-zero between
//            calls. No float atomics: results are deterministic.
//
// Every index read from A is range-checked; a bad index is recorded in the device error
// record and replaced by a harmless one, so malformed input cannot fault the GPU.

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"

// Resident CTAs per SM the register allocation is sized for (256 threads per CTA; 4 caps a
// thread at 64 registers). The default chunk size assumes exactly this residency.
#ifndef SPMM_CSR_MIN_CTAS
#define SPMM_CSR_MIN_CTAS 4
#endif
// Nonzeros whose B loads are issued before their FMAs, for one and two 32-lane strides per
// nonzero (compile-time tuning).
#ifndef SPMM_CSR_UNROLL_R1
#define SPMM_CSR_UNROLL_R1 8
#endif
#ifndef SPMM_CSR_UNROLL_R2
#define SPMM_CSR_UNROLL_R2 4
#endif

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
    int* counters;       // num_chunks per slab, all-zero between calls
    float* partials;     // num_chunks * 2 * N
    int b_policy;        // B loads: 0 plain, 1 L2 evict-last, 2 evict-last + no L1 allocation
    // Column phases (ROWWARP): launch `phase` of `phases` runs positions [split[phase-1][i],
    // split[phase][i]) of row i (split[-1] = row start, split[phases-1] = row end). With
    // phase_loop set, one launch runs every phase: each warp takes its rows through phase 0,
    // then the same rows through phase 1, and so on.
    int phase, phases;
    int phase_loop;
    int* ksplit;         // (phases - 1) x M split positions
    int* sched_counters; // dynamic merge schedule: [next chunk, warps done] per slab, zero between calls
    DeviceErrorRecord* err;
};

__device__ __forceinline__ uint64_t evict_last_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

template <int VEC> struct Vec;
template <> struct Vec<1> {
    using T = float;
    __device__ static T load(const float* p, uint64_t pol, int mode) {
        float v;
        if (mode == 0) return __ldg(p);
        if (mode == 2)
            asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(v) : "l"(p), "l"(pol));
        else
            asm volatile("ld.global.nc.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(v) : "l"(p), "l"(pol));
        return v;
    }
    __device__ static T loadcg(const float* p) { return __ldcg(p); }
    __device__ static void store_cs(float* p, T v) { __stcs(p, v); }
    __device__ static void store_cg(float* p, T v) { __stcg(p, v); }
    __device__ static float get(const T& v, int) { return v; }
    __device__ static void set(T& v, int, float x) { v = x; }
};
template <> struct Vec<2> {
    using T = float2;
    __device__ static T load(const float* p, uint64_t pol, int mode) {
        float2 v;
        if (mode == 0) return __ldg(reinterpret_cast<const float2*>(p));
        if (mode == 2)
            asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.f32 {%0, %1}, [%2], %3;"
                         : "=f"(v.x), "=f"(v.y)
                         : "l"(p), "l"(pol));
        else
            asm volatile("ld.global.nc.L2::cache_hint.v2.f32 {%0, %1}, [%2], %3;"
                         : "=f"(v.x), "=f"(v.y)
                         : "l"(p), "l"(pol));
        return v;
    }
    __device__ static T loadcg(const float* p) { return __ldcg(reinterpret_cast<const float2*>(p)); }
    __device__ static void store_cs(float* p, T v) { __stcs(reinterpret_cast<float2*>(p), v); }
    __device__ static void store_cg(float* p, T v) { __stcg(reinterpret_cast<float2*>(p), v); }
    __device__ static float get(const T& v, int e) { return e == 0 ? v.x : v.y; }
    __device__ static void set(T& v, int e, float x) { if (e == 0) v.x = x; else v.y = x; }
};
template <> struct Vec<4> {
    using T = float4;
    __device__ static T load(const float* p, uint64_t pol, int mode) {
        float4 v;
        if (mode == 0) return __ldg(reinterpret_cast<const float4*>(p));
        if (mode == 2)
            asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                         : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                         : "l"(p), "l"(pol));
        else
            asm volatile("ld.global.nc.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                         : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                         : "l"(p), "l"(pol));
        return v;
    }
    __device__ static T loadcg(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
    __device__ static void store_cs(float* p, T v) { __stcs(reinterpret_cast<float4*>(p), v); }
    __device__ static void store_cg(float* p, T v) { __stcg(reinterpret_cast<float4*>(p), v); }
    __device__ static float get(const T& v, int e) { return e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w; }
    __device__ static void set(T& v, int e, float x) {
        if (e == 0) v.x = x; else if (e == 1) v.y = x; else if (e == 2) v.z = x; else v.w = x;
    }
};

// First column of lane `lane` in stride r of the slab starting at col0.
template <int VEC>
__device__ __forceinline__ int lane_col(int col0, int r, int lane) {
    return col0 + (r * 32 + lane) * VEC;
}

__device__ __forceinline__ int clampi(int x, int lo, int hi) { return x < lo ? lo : (x > hi ? hi : x); }

// Per-warp staging ring for A's (col, val) pairs: two groups of 32, filled with cp.async
// (global -> shared, no registers held while in flight) one group ahead of use, read back
// as one broadcast 8-byte shared load per nonzero.
struct PairRing {
    int2 g[2][32];
};

__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int Pending>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(Pending) : "memory");
}

// Copy the pairs [base, min(base + 32, p1)) of A into ring slot `slot` (one commit group).
__device__ __forceinline__ void stage_pairs(const CsrArgs& a, PairRing* ring, int slot, int base, int p1, int lane) {
    const int p = base + lane;
    if (p < p1) {
        cp_async4(&ring->g[slot][lane].x, a.col_idx + p);
        cp_async4(&ring->g[slot][lane].y, a.values + p);
    }
    cp_async_commit();
}

// Sum of v_p * B[col_p, slab columns] over p in [p0, p1) into acc (caller zeroes acc), as
// one sequential FMA chain per column.
template <int VEC, int R, int U, bool HINT>
__device__ __forceinline__ void accumulate(const CsrArgs& a, PairRing* ring, int p0, int p1, int col0, int lane,
                                           uint64_t pol, float (&acc)[R][VEC]) {
    using V = Vec<VEC>;
    const int hint = a.b_policy;
    // B row loads: plain non-coherent loads unless the caller asked for an L2 policy (a
    // separate instantiation, so the default kernels carry no policy register or branch).
    auto load_b = [&](const float* p) {
        if constexpr (HINT) return V::load(p, pol, hint);
        else return V::load(p, 0, 0);
    };
    bool ok[R];
#pragma unroll
    for (int r = 0; r < R; ++r) ok[r] = lane_col<VEC>(col0, r, lane) < a.N;

    const float* __restrict__ Bp = a.B + col0 + lane * VEC;
    if (p0 >= p1) return;
    stage_pairs(a, ring, 0, p0, p1, lane);
    int slot = 0;
    for (int base = p0; base < p1; base += 32) {
        stage_pairs(a, ring, slot ^ 1, base + 32, p1, lane);  // next group (empty past p1)
        cp_async_wait<1>();
        __syncwarp();
        const int cnt = min(32, p1 - base);
        if (lane < cnt && static_cast<unsigned>(ring->g[slot][lane].x) >= static_cast<unsigned>(a.K)) {
            record_device_error(a.err, SPMM_ERR_BAD_INDEX, static_cast<long long>(base + lane));
            ring->g[slot][lane] = make_int2(0, 0);
        }
        __syncwarp();
        const int2* grp = ring->g[slot];
        int q = 0;
        for (; q + U <= cnt; q += U) {
            // Two strides per nonzero (R = 2): keep the U values from the 8-byte pair loads;
            // one stride: re-read each value at its FMA (fewer live registers; measured
            // faster on configs 1, 2 and 4, slower on config 5).
            constexpr bool kKeepV = R >= 2;
            typename V::T b[U][R];
            float v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int2 pr = grp[q + u];
                if constexpr (kKeepV) v[u] = __int_as_float(pr.y);
                const float* brow = Bp + static_cast<size_t>(pr.x) * a.N;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if (ok[r]) b[u][r] = load_b(brow + r * 32 * VEC);
                    else b[u][r] = typename V::T{};
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const float vu = kKeepV ? v[u] : __int_as_float(grp[q + u].y);
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int e = 0; e < VEC; ++e) acc[r][e] = fmaf(vu, V::get(b[u][r], e), acc[r][e]);
            }
        }
        for (; q < cnt; ++q) {
            const int2 pr = grp[q];
            const float v = __int_as_float(pr.y);
            const float* brow = Bp + static_cast<size_t>(pr.x) * a.N;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (ok[r]) {
                    const typename V::T b = load_b(brow + r * 32 * VEC);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) acc[r][e] = fmaf(v, V::get(b, e), acc[r][e]);
                }
            }
        }
        __syncwarp();  // every lane is done with this slot before it is refilled
        slot ^= 1;
    }
    cp_async_wait<0>();
}

template <int VEC, int R>
__device__ __forceinline__ void store_slab(const CsrArgs& a, float* dst, int col0, int lane,
                                           const float (&acc)[R][VEC], bool streaming) {
    using V = Vec<VEC>;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int c = lane_col<VEC>(col0, r, lane);
        if (c < a.N) {
            typename V::T t;
#pragma unroll
            for (int e = 0; e < VEC; ++e) V::set(t, e, acc[r][e]);
            if (streaming) V::store_cs(dst + c, t);
            else V::store_cg(dst + c, t);
        }
    }
}

template <int VEC, int R>
__device__ __forceinline__ void load_slab(const CsrArgs& a, const float* src, int col0, int lane,
                                          float (&acc)[R][VEC]) {
    using V = Vec<VEC>;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int c = lane_col<VEC>(col0, r, lane);
        typename V::T t{};
        if (c < a.N) t = V::loadcg(src + c);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[r][e] = V::get(t, e);
    }
}

template <int VEC, int R>
__device__ __forceinline__ void zero(float (&acc)[R][VEC]) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[r][e] = 0.f;
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

template <int VEC, int R, int U, bool PHASED, bool HINT>
__global__ void __launch_bounds__(kThreads, SPMM_CSR_MIN_CTAS) csr_rowwarp_kernel(CsrArgs a) {
    // A programmatic dependent of the previous kernel in the stream: its launch overlaps that
    // kernel's tail; nothing global is touched before the wait.
    grid_dependency_wait();
    allow_dependent_launch();
    constexpr int W = 32 * VEC * R;
    __shared__ PairRing rings[kWarpsPerCta];
    PairRing* ring = &rings[threadIdx.x >> 5];
    const int lane = threadIdx.x & 31;
    const int warp = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * kWarpsPerCta;
    const int col0 = blockIdx.y * W;
    const uint64_t pol = HINT ? evict_last_policy() : 0;
    if constexpr (PHASED) {
        // Phase ph of row i: its positions [split[ph-1][i], split[ph][i]); the chain continues
        // from the value phase ph-1 stored in C (phase 0 starts from +0 and writes every row).
        // In one launch (phase_loop) a row's phases run on the same warp, lane for lane, in
        // order: each lane reads back (ld.global.cg) only the C elements it stored itself.
        const int ph0 = a.phase_loop ? 0 : a.phase;
        const int ph1 = a.phase_loop ? a.phases : a.phase + 1;
        for (int ph = ph0; ph < ph1; ++ph) {
            const bool last = ph == a.phases - 1;
            for (int i = warp; i < a.M; i += nwarps) {
                int rs, re;
                row_bounds(a, i, rs, re);
                float acc[R][VEC];
                float* crow = a.C + static_cast<size_t>(i) * a.N;
                int lo = rs, hi = re;
                if (ph > 0) lo = clampi(__ldcg(a.ksplit + static_cast<size_t>(ph - 1) * a.M + i), rs, re);
                if (!last) hi = clampi(__ldcg(a.ksplit + static_cast<size_t>(ph) * a.M + i), lo, re);
                if (ph > 0 && lo == hi) continue;
                if (ph > 0) load_slab<VEC, R>(a, crow, col0, lane, acc);
                else zero(acc);
                accumulate<VEC, R, U, HINT>(a, ring, lo, hi, col0, lane, pol, acc);
                // A partial that this launch reads back stays cached; the rest streams.
                store_slab<VEC, R>(a, crow, col0, lane, acc, last || !a.phase_loop);
            }
        }
    } else {
        for (int i = warp; i < a.M; i += nwarps) {
            int rs, re;
            row_bounds(a, i, rs, re);
            float acc[R][VEC];
            zero(acc);
            accumulate<VEC, R, U, HINT>(a, ring, rs, re, col0, lane, pol, acc);
            store_slab<VEC, R>(a, a.C + static_cast<size_t>(i) * a.N, col0, lane, acc, true);
        }
    }
}

// Split positions for column phases: split[b][i] = row start + number of row-i nonzeros with
// column < K * (b + 1) / phases. Any monotone cut of a row's positions gives the same FMA
// chain, so the results do not depend on these values; sorted rows make each phase touch
// only its range of B rows.
__global__ void __launch_bounds__(kThreads) csr_ksplit_kernel(CsrArgs a) {
    const int lane = threadIdx.x & 31;
    const int warp = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * kWarpsPerCta;
    const int nb = a.phases - 1;  // <= 32: lane b keeps boundary b's count
    for (int i = warp; i < a.M; i += nwarps) {
        int rs, re;
        row_bounds(a, i, rs, re);
        int mine = 0;  // lane b < nb counts columns below boundary b
        for (int base = rs; base < re; base += 32) {
            const int p = base + lane;
            const int k = p < re ? __ldcs(a.col_idx + p) : 0x7fffffff;
#pragma unroll 1
            for (int b = 0; b < nb; ++b) {
                const long long kb = static_cast<long long>(a.K) * (b + 1) / a.phases;
                const int n = __popc(__ballot_sync(kFull, p < re && static_cast<long long>(k) < kb));
                if (lane == b) mine += n;
            }
        }
        if (lane < nb) a.ksplit[static_cast<size_t>(lane) * a.M + i] = rs + mine;
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

// First row r >= r0 with r + row_ptr[r] >= d (M if none): a chunk spans few rows, so scan
// forward 32 rows per coalesced probe; after 4 probes fall back to the search.
__device__ __forceinline__ int warp_forward_bound(const CsrArgs& a, int r0, long long d, int lane) {
    int r = r0;
    for (int step = 0; step < 4 && r < a.M; ++step, r += 32) {
        const int cand = r + lane;
        const bool lt = cand < a.M && static_cast<long long>(cand) + __ldg(a.row_ptr + cand) < d;
        const unsigned m = __ballot_sync(kFull, lt);
        if (m != kFull) return r + __popc(m);
    }
    if (r >= a.M) return a.M;
    return warp_lower_bound(a, d, lane);
}

// One piece [p0, p1) of long row i (rs..re) for this CTA's slab; `slot` is this chunk's
// workspace slot.
template <int VEC, int R, int U, bool HINT>
__device__ __forceinline__ void long_piece(const CsrArgs& a, PairRing* ring, int i, int rs, int re, int p0, int p1,
                                           int slot, int col0, int lane, uint64_t pol) {
    using V = Vec<VEC>;
    float acc[R][VEC];
    zero(acc);
    accumulate<VEC, R, U, HINT>(a, ring, p0, p1, col0, lane, pol, acc);
    store_slab<VEC, R>(a, a.partials + static_cast<size_t>(slot) * a.N, col0, lane, acc, false);
    // Publish the piece, then count arrivals on the row's first chunk (per slab).
    __threadfence();
    __syncwarp();
    const long long first_item = static_cast<long long>(i) + rs;
    const long long last_item = static_cast<long long>(i) + re - 1;
    const int ca = static_cast<int>(first_item / a.S);
    const int cb = static_cast<int>(last_item / a.S);
    const int pieces = cb - ca + 1;
    int* counter = a.counters + static_cast<size_t>(blockIdx.y) * a.num_chunks + ca;
    int prev = 0;
    if (lane == 0) prev = atomicAdd(counter, 1);
    prev = __shfl_sync(kFull, prev, 0);
    if (prev != pieces - 1) return;
    // Last arrival: add the pieces in chunk order and write the row's slab; clear every slot
    // it read and the counter, so the whole workspace is zero again after the launch.
    __threadfence();
    float* crow = a.C + static_cast<size_t>(i) * a.N;
    const typename V::T zero_v{};
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int c = lane_col<VEC>(col0, r, lane);
        if (c < a.N) {
            float* first = a.partials + static_cast<size_t>(2 * ca + 1) * a.N + c;
            typename V::T s = V::loadcg(first);
            V::store_cg(first, zero_v);
            for (int cc = ca + 1; cc <= cb; ++cc) {
                float* slot_p = a.partials + static_cast<size_t>(2 * cc) * a.N + c;
                const typename V::T t = V::loadcg(slot_p);
                V::store_cg(slot_p, zero_v);
#pragma unroll
                for (int e = 0; e < VEC; ++e) V::set(s, e, V::get(s, e) + V::get(t, e));
            }
            V::store_cs(crow + c, s);
        }
    }
    if (lane == 0) *counter = 0;
}

// One merge-path chunk c (items [c S, (c + 1) S)) for this warp.
template <int VEC, int R, int U, bool HINT>
__device__ __forceinline__ void merge_chunk(const CsrArgs& a, PairRing* ring, int c, int col0, int lane, uint64_t pol) {
    const long long d0 = static_cast<long long>(c) * a.S;
    const long long d1 = min(d0 + a.S, a.items);
    const int r0 = warp_lower_bound(a, d0, lane);
    const int r1 = warp_forward_bound(a, r0, d1, lane);

    // A long row that started in an earlier chunk and reaches into this one.
    if (r0 > 0) {
        const int q = r0 - 1;
        int qs, qe;
        row_bounds(a, q, qs, qe);
        if (qe - qs > a.S) {
            const int p0 = static_cast<int>(max(static_cast<long long>(qs), d0 - q));
            const int p1 = static_cast<int>(min(static_cast<long long>(qe), d1 - q));
            if (p0 < p1) long_piece<VEC, R, U, HINT>(a, ring, q, qs, qe, p0, p1, 2 * c, col0, lane, pol);
        }
    }
    // Rows whose first item lies in this chunk.
    for (int i = r0; i < r1; ++i) {
        int rs, re;
        row_bounds(a, i, rs, re);
        if (re - rs <= a.S) {
            float acc[R][VEC];
            zero(acc);
            accumulate<VEC, R, U, HINT>(a, ring, rs, re, col0, lane, pol, acc);
            store_slab<VEC, R>(a, a.C + static_cast<size_t>(i) * a.N, col0, lane, acc, true);
        } else {
            const int p1 = static_cast<int>(min(static_cast<long long>(re), d1 - i));
            long_piece<VEC, R, U, HINT>(a, ring, i, rs, re, rs, max(p1, rs), 2 * c + 1, col0, lane, pol);
        }
    }
}

// DYN = false: warp w of the grid takes chunk w. DYN = true: a persistent grid whose warps
// take chunks from a per-slab work counter until none is left (chunks of unequal cost no
// longer leave SMs idle at the end); the last warp to leave resets the counters. Which warp
// runs a chunk does not change any result.
template <int VEC, int R, int U, bool HINT, bool DYN>
__global__ void __launch_bounds__(kThreads, SPMM_CSR_MIN_CTAS) csr_merge_kernel(CsrArgs a) {
    grid_dependency_wait();  // a programmatic dependent launch, as csr_rowwarp_kernel
    allow_dependent_launch();
    constexpr int W = 32 * VEC * R;
    __shared__ PairRing rings[kWarpsPerCta];
    PairRing* ring = &rings[threadIdx.x >> 5];
    const int lane = threadIdx.x & 31;
    const int col0 = blockIdx.y * W;
    const uint64_t pol = HINT ? evict_last_policy() : 0;
    if constexpr (!DYN) {
        const int c = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
        if (c < a.num_chunks) merge_chunk<VEC, R, U, HINT>(a, ring, c, col0, lane, pol);
    } else {
        int* work = a.sched_counters + 2 * blockIdx.y;
        for (;;) {
            int c = 0;
            if (lane == 0) c = atomicAdd(work, 1);
            c = __shfl_sync(kFull, c, 0);
            if (c >= a.num_chunks) break;
            merge_chunk<VEC, R, U, HINT>(a, ring, c, col0, lane, pol);
        }
        if (lane == 0) {
            const int warps = gridDim.x * kWarpsPerCta;
            if (atomicAdd(work + 1, 1) == warps - 1) {
                work[0] = 0;
                work[1] = 0;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------

struct Geometry {
    int vec = 1;
    int r = 1;
    int width() const { return 32 * vec * r; }
};

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

constexpr int kMaxPhases = 8;

// Slab width: the narrowest of 32/64/128/256 columns that covers N, at most 256. Narrower
// slabs that keep a slab's B columns L2-resident (col_pass) re-read A once per slab; on B200
// at config 5 (B = 134 MB) one 256-wide slab with evict-last B loads measured faster than two
// 128-wide ones (1.02 vs 1.13 ms), so N is not split further by default.
int slab_width(int N, int col_pass) {
    if (col_pass > 0) return col_pass;
    int w = 32;
    while (w < N && w < 256) w *= 2;
    return w;
}

// Realise a slab width with the widest vector the operands allow.
Geometry pick_geometry(const float* B, const float* C, int N, int w) {
    Geometry g;
    const bool v4 = N % 4 == 0 && aligned(B, 16) && aligned(C, 16);
    const bool v2 = N % 2 == 0 && aligned(B, 8) && aligned(C, 8);
    if (w >= 256) {
        if (v4) { g.vec = 4; g.r = 2; }
        else if (v2) { g.vec = 2; g.r = 4; }
        else { g.vec = 1; g.r = 8; }
    } else if (w >= 128) {
        if (v4) { g.vec = 4; g.r = 1; }
        else if (v2) { g.vec = 2; g.r = 2; }
        else { g.vec = 1; g.r = 4; }
    } else if (w >= 64) {
        if (v2) { g.vec = 2; g.r = 1; }
        else { g.vec = 1; g.r = 2; }
    } else {
        g.vec = 1;
        g.r = 1;
    }
    return g;
}

// One chunk per resident warp: the grid is a single wave (SMs x SPMM_CSR_MIN_CTAS CTAs of 8
// warps), every warp gets the same number of merge-path items, no tail wave. Multiple of 32,
// at least 64.
int default_chunk(long long items, int sm_count) {
    const long long warps = static_cast<long long>(std::max(sm_count, 1)) * SPMM_CSR_MIN_CTAS * kWarpsPerCta;
    long long s = (items + warps - 1) / warps;
    s = ((s + 31) / 32) * 32;
    s = std::max<long long>(64, std::min<long long>(1ll << 30, s));
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
    if (tune->b_policy < 0 || tune->b_policy > 2) return SPMM_ERR_INVALID_ARG;
    if (tune->k_phases < 0 || tune->k_phases > kMaxPhases) return SPMM_ERR_INVALID_ARG;
    if (tune->schedule < 0 || tune->schedule > 2) return SPMM_ERR_INVALID_ARG;
    if (tune->phase_mode < 0 || tune->phase_mode > 2) return SPMM_ERR_INVALID_ARG;
    return SPMM_OK;
}

// Column phases in one launch (tune->phase_mode 2) or one launch per phase (0, 1).
bool phase_in_one_launch(const spmm_csr_tuning* tune) { return tune && tune->phase_mode == 2; }

int resolve_phases(int algo, const spmm_csr_tuning* tune) {
    return (algo == SPMM_CSR_ROWWARP && tune && tune->k_phases > 1) ? tune->k_phases : 1;
}

size_t ksplit_bytes(int phases, int M) {
    return phases > 1 ? align_up(static_cast<size_t>(phases - 1) * static_cast<size_t>(M) * sizeof(int), 256) : 0;
}

// Counters for every slab the narrowest slab width (32 columns) could need, so the size does
// not depend on the operands' alignment.
size_t counter_bytes(long long num_chunks, int N) {
    // Arrival counters (num_chunks per possible 32-column slab), then the dynamic schedule's
    // two counters per slab.
    const size_t slabs = static_cast<size_t>((N + 31) / 32);
    return align_up((static_cast<size_t>(num_chunks) + 2) * slabs * sizeof(int), 256);
}

size_t merge_workspace_bytes(long long num_chunks, int N) {
    if (num_chunks <= 0) return 0;
    return counter_bytes(num_chunks, N) + static_cast<size_t>(num_chunks) * 2 * static_cast<size_t>(N) * sizeof(float);
}

// A CSR kernel launched as a programmatic dependent of the previous kernel in the stream (the
// kernel waits for it before touching global memory). Errors surface through cudaGetLastError.
void launch_pdl(void (*kernel)(CsrArgs), dim3 grid, cudaStream_t s, const CsrArgs& a) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    (void)cudaLaunchKernelEx(&cfg, kernel, a);
}

template <int VEC, int R>
void launch_vr(int algo, const CsrArgs& a, dim3 grid, cudaStream_t s) {
    // Vector loads per lane in flight: U nonzeros x R strides (eight by default).
    constexpr int U = R == 1 ? SPMM_CSR_UNROLL_R1 : (R == 2 ? SPMM_CSR_UNROLL_R2 : ((8 / R) > 0 ? (8 / R) : 1));
    const bool hint = a.b_policy != 0;
    if (algo == SPMM_CSR_ROWWARP) {
        if (a.phases > 1) {
            if (hint) launch_pdl(csr_rowwarp_kernel<VEC, R, U, true, true>, grid, s, a);
            else launch_pdl(csr_rowwarp_kernel<VEC, R, U, true, false>, grid, s, a);
        } else {
            if (hint) launch_pdl(csr_rowwarp_kernel<VEC, R, U, false, true>, grid, s, a);
            else launch_pdl(csr_rowwarp_kernel<VEC, R, U, false, false>, grid, s, a);
        }
    } else {
        const bool dyn = a.sched_counters != nullptr;
        if (hint) {
            if (dyn) launch_pdl(csr_merge_kernel<VEC, R, U, true, true>, grid, s, a);
            else launch_pdl(csr_merge_kernel<VEC, R, U, true, false>, grid, s, a);
        } else {
            if (dyn) launch_pdl(csr_merge_kernel<VEC, R, U, false, true>, grid, s, a);
            else launch_pdl(csr_merge_kernel<VEC, R, U, false, false>, grid, s, a);
        }
    }
}

void launch(const Geometry& g, int algo, const CsrArgs& a, dim3 grid, cudaStream_t s) {
    switch (g.vec * 10 + g.r) {
        case 11: launch_vr<1, 1>(algo, a, grid, s); break;
        case 12: launch_vr<1, 2>(algo, a, grid, s); break;
        case 14: launch_vr<1, 4>(algo, a, grid, s); break;
        case 18: launch_vr<1, 8>(algo, a, grid, s); break;
        case 21: launch_vr<2, 1>(algo, a, grid, s); break;
        case 22: launch_vr<2, 2>(algo, a, grid, s); break;
        case 24: launch_vr<2, 4>(algo, a, grid, s); break;
        case 41: launch_vr<4, 1>(algo, a, grid, s); break;
        default: launch_vr<4, 2>(algo, a, grid, s); break;
    }
}

}  // namespace

int csr_f32_check_args(const spmm_csr_view* A, const float* B, const float* C, int32_t N) {
    return check_view(A, B, C, N);
}

// Shared by the C entry points below and by the allocation-free variant in noalloc.cu.
int csr_f32_launch(const spmm_csr_view* A, const float* B, float* C, int32_t N, int32_t algo,
                   const spmm_csr_tuning* tune, void* ws, size_t ws_bytes, cudaStream_t stream,
                   DeviceState* st, bool ksplit_ready) {
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
    a.b_policy = tune ? tune->b_policy : 0;
    const int w = slab_width(N, tune ? tune->col_pass : 0);
    const Geometry g = pick_geometry(B, C, N, w);
    const int slabs = (N + g.width() - 1) / g.width();
    if (slabs > 65535) return SPMM_ERR_TOO_LARGE;

    dim3 grid(1, slabs, 1);
    if (algo == SPMM_CSR_ROWWARP) {
        const long long warps = std::min<long long>(A->rows, static_cast<long long>(st->sm_count) * 64);
        grid.x = static_cast<unsigned>((warps + kWarpsPerCta - 1) / kWarpsPerCta);
        a.phases = resolve_phases(algo, tune);
        if (a.phases > 1) {
            // Column phases: split positions (computed here unless the caller holds them),
            // then one launch per phase (or one launch for all of them, on one wave of
            // resident warps), then the workspace is cleared again.
            const size_t need = ksplit_bytes(a.phases, A->rows);
            if (need > ws_bytes || !ws) return SPMM_ERR_INVALID_ARG;
            a.ksplit = static_cast<int*>(ws);
            if (!ksplit_ready) {
                csr_ksplit_kernel<<<grid.x, kThreads, 0, stream>>>(a);
                SPMM_CUDA_TRY(cudaGetLastError());
            }
            if (phase_in_one_launch(tune)) {
                const long long resident = static_cast<long long>(st->sm_count) * SPMM_CSR_MIN_CTAS * kWarpsPerCta;
                const long long warps1 = std::min<long long>(A->rows, resident);
                dim3 grid1(static_cast<unsigned>((warps1 + kWarpsPerCta - 1) / kWarpsPerCta), grid.y, 1);
                a.phase_loop = 1;
                a.phase = 0;
                launch(g, algo, a, grid1, stream);
                SPMM_CUDA_TRY(cudaGetLastError());
            } else {
                for (a.phase = 0; a.phase < a.phases; ++a.phase) {
                    launch(g, algo, a, grid, stream);
                    SPMM_CUDA_TRY(cudaGetLastError());
                }
            }
            if (!ksplit_ready) SPMM_CUDA_TRY(cudaMemsetAsync(ws, 0, need, stream));
            return SPMM_OK;
        }
    } else {
        a.S = resolve_chunk(A, tune, st->sm_count);
        a.items = static_cast<long long>(A->rows) + A->nnz;
        const long long chunks = (a.items + a.S - 1) / a.S;
        if (chunks > (1ll << 30)) return SPMM_ERR_TOO_LARGE;
        a.num_chunks = static_cast<int>(chunks);
        const size_t need = merge_workspace_bytes(chunks, N);
        if (need > ws_bytes || (need > 0 && !ws)) return SPMM_ERR_INVALID_ARG;
        a.counters = static_cast<int*>(ws);
        a.partials = reinterpret_cast<float*>(static_cast<char*>(ws) + counter_bytes(chunks, N));
        long long warps = chunks;
        if (tune && tune->schedule == 2) {
            // Persistent warps pulling chunks from a counter: one wave of resident warps.
            a.sched_counters = a.counters + static_cast<size_t>(chunks) * ((N + 31) / 32);
            warps = std::min<long long>(chunks, static_cast<long long>(st->sm_count) * SPMM_CSR_MIN_CTAS * kWarpsPerCta);
        }
        grid.x = static_cast<unsigned>((warps + kWarpsPerCta - 1) / kWarpsPerCta);
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
    if (A->rows == 0 || N == 0) return SPMM_OK;
    if (algo == SPMM_CSR_ROWWARP) {
        *bytes = ksplit_bytes(resolve_phases(algo, tune), A->rows);
        return SPMM_OK;
    }
    if (algo != SPMM_CSR_MERGE) return SPMM_ERR_INVALID_ARG;
    const int S = resolve_chunk(A, tune, sm_count);
    const long long items = static_cast<long long>(A->rows) + A->nnz;
    *bytes = merge_workspace_bytes((items + S - 1) / S, N);
    return SPMM_OK;
}

// Split positions for a plan that keeps them across executions (phases <= 33: one warp
// lane per boundary).
int csr_f32_ksplit(const spmm_csr_view* A, int phases, int* split, cudaStream_t stream, DeviceState* st) {
    if (phases <= 1 || A->rows == 0) return SPMM_OK;
    if (phases > 33) return SPMM_ERR_INVALID_ARG;
    CsrArgs a{};
    a.M = A->rows;
    a.K = A->cols;
    a.nnz = A->nnz;
    a.row_ptr = A->row_ptr;
    a.col_idx = A->col_idx;
    a.phases = phases;
    a.ksplit = split;
    a.err = st->err;
    const long long warps = std::min<long long>(A->rows, static_cast<long long>(st->sm_count) * 64);
    csr_ksplit_kernel<<<static_cast<unsigned>((warps + kWarpsPerCta - 1) / kWarpsPerCta), kThreads, 0, stream>>>(a);
    SPMM_CUDA_TRY(cudaGetLastError());
    return SPMM_OK;
}

// One column phase of the ROWWARP kernel (callers that interleave other work between
// phases, e.g. moving B's slices in and out of device memory); `split` holds the
// (phases - 1) x M positions from csr_f32_ksplit.
int csr_f32_phase_launch(const spmm_csr_view* A, const float* B, float* C, int32_t N, int phases, int phase,
                         int* split, cudaStream_t stream, DeviceState* st) {
    SPMM_TRY(check_view(A, B, C, N));
    if (phases < 1 || phase < 0 || phase >= phases || (phases > 1 && !split)) return SPMM_ERR_INVALID_ARG;
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
    a.phases = phases;
    a.phase = phase;
    a.ksplit = split;
    const Geometry g = pick_geometry(B, C, N, slab_width(N, 0));
    const int slabs = (N + g.width() - 1) / g.width();
    if (slabs > 65535) return SPMM_ERR_TOO_LARGE;
    const long long warps = std::min<long long>(A->rows, static_cast<long long>(st->sm_count) * 64);
    const dim3 grid(static_cast<unsigned>((warps + kWarpsPerCta - 1) / kWarpsPerCta), slabs, 1);
    launch(g, SPMM_CSR_ROWWARP, a, grid, stream);
    SPMM_CUDA_TRY(cudaGetLastError());
    return SPMM_OK;
}

// Bytes at the start of the merge-path workspace that must be zero when a launch starts.
size_t csr_f32_counter_bytes(const spmm_csr_view* A, int32_t N, const spmm_csr_tuning* tune, int sm_count) {
    const int S = resolve_chunk(A, tune, sm_count);
    const long long items = static_cast<long long>(A->rows) + A->nnz;
    return counter_bytes((items + S - 1) / S, N);
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
    return csr_f32_launch(A, B, C, N, algo, tune, ws, ws_bytes, as_stream(stream), st, false);
}

int spmm_csr_f32(const spmm_csr_view* A, const float* B, float* C, int32_t N, int32_t algo, void* stream) {
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    SPMM_TRY(check_view(A, B, C, N));
    size_t need = 0;
    SPMM_TRY(csr_f32_workspace_bytes(A, N, algo, nullptr, st->sm_count, &need));
    std::lock_guard<std::mutex> lock(st->mu);
    SPMM_TRY(ensure_device_buffer(&st->csr_ws, &st->csr_ws_bytes, need, true, as_stream(stream)));
    return csr_f32_launch(A, B, C, N, algo, nullptr, st->csr_ws, st->csr_ws_bytes, as_stream(stream), st, false);
}

}  // extern "C"
