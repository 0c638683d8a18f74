// BSR-16 x dense SpMM on the B200 tensor cores (tcgen05 MMA, TMEM accumulators, TMA).
//
// Replaces the reference's WMMA kernel (src/kernels/spmm_wmma.cu:49-142): same product,
// C[M x N] (FP32) = A (BSR, 16x16 FP16/BF16 blocks) * B (K x N, same 16-bit type), FP32
// accumulation.
//
// Mapping. A 16-row block-row is too short for an MMA's M (64/128), so the kernel computes
// the transposed tile: for block (br, bc)
//     C[br*16 : +16, n0 : n0+128]^T  +=  B[bc*16 : +16, n0 : n0+128]^T  *  A_blk^T
// i.e. one tcgen05.mma kind::f16 with M = 128 (a 128-column slice of C), N = 16 (the block's
// 16 rows), K = 16 (the block's 16 columns). Operand A of the MMA is the B tile, read
// MN-major from shared memory (128B swizzle); operand B is the BSR block itself, read K-major
// (32B swizzle) -- exactly its row-major storage. The accumulator lives in TMEM: lane m =
// column n0+m of C, columns 16j..16j+15 = the 16 rows of block-row j of the CTA.
//
// A CTA owns G consecutive block-rows and one 128-column slice of N. A producer warp merges
// the G sorted block-column lists; for every distinct block-column it TMA-loads the B tile
// once (2 boxes of 16 x 64) plus the blocks of the block-rows that contain it, and the MMA
// thread issues one MMA per such block into that block-row's TMEM columns -- or, when all G
// block-rows have the column, a single MMA with N = 16 G over the G consecutive block slots
// (their accumulator columns are consecutive too). So a B tile shared by several block-rows
// (e.g. dense diagonal blocks larger than 16) crosses L2 once per CTA. An 8-deep shared-memory
// ring with mbarriers decouples TMA and MMA (the producer fills it a batch at a time, the MMA
// thread takes every stage that has landed); four epilogue warps move TMEM -> registers ->
// coalesced FP32 stores.
//
// Every mbarrier wait is bounded (iteration count and %globaltimer); on expiry the kernel
// records SPMM_ERR_TIMEOUT, stops issuing work, drains what it issued, frees its TMEM and
// returns. No TMA multicast is used.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdint>
#include <mutex>
#include <new>
#include <vector>

#include "common.cuh"

// A BSR-16 plan: the view, the tile group size, the per-CTA schedule (device memory, NULL when
// the schedule would be too large or the tensor-core path does not apply) and A's tensor map.
struct spmm_bsr_plan {
    spmm_bsr_view A{};
    int32_t N = 0;
    int32_t group = 0;
    int32_t max_steps = 0;
    int32_t stride = 0;
    int* sched = nullptr;
    size_t sched_bytes = 0;
    int32_t device = 0;
    bool tc = false;
    CUtensorMap ta{};
    CUtensorMap ta4{};     // A's blocks in groups of a_stride (grouped copies), if a_stride > 0
    int32_t a_stride = 0;
    int32_t a_groups = 0;
    // B's tensor map for the last B16 pointer executed (re-encoded only when B16 changes: the
    // encode is host work between the caller's launch and the kernel's start).
    mutable std::mutex tb_mu;
    mutable CUtensorMap tb{};
    mutable const void* tb_for = nullptr;
};

namespace spmm_b200 {
namespace {

constexpr int kStages = 8;
constexpr int kColCache = 4096;       // block-column indices cached in shared memory per CTA
constexpr int kTcThreads = 192;       // warp 0 TMA, warp 1 MMA + TMEM, warps 2..5 epilogue
constexpr unsigned kFullMask = 0xffffffffu;
constexpr int kDone = -1;
constexpr uint32_t kFullArrivals = 1;  // the lane that claims the stage (arrive + expect_tx)
constexpr unsigned long long kWaitNs = 500ull * 1000 * 1000;  // 0.5 s per wait

struct BsrArgs {
    int M, K, N;
    int block_rows, block_cols, num_blocks;
    const int* __restrict__ row_ptr;
    const int* __restrict__ col_idx;
    const uint16_t* __restrict__ values;
    const uint16_t* __restrict__ B;
    float* __restrict__ C;
    int dtype;
    DeviceErrorRecord* err;
    // Precomputed per-CTA schedule (plans): group g's record at sched + g * sched_stride:
    // [steps, rows_mask, then per step: block column, row mask, G block indices].
    const int* __restrict__ sched;
    int sched_stride;
    // Grouped A loads (plans): when a stage's G blocks sit at p, p + S, ..., p + (G-1) S in the
    // value array (S = a_stride > 0; the same S for every block-row step of a block-diagonal
    // or evenly filled band), one 4-D copy of A's blocks viewed as [a_groups][S][16][16]
    // fetches all G of them. 0: one copy per block.
    int a_stride;
    int a_groups;
};

template <int G>
struct Layout {
    static constexpr int kBTile = 4096;                    // 16 x 128 x 2 B, two SW128 boxes
    static constexpr int kASlot = 512;                     // 16 x 16 x 2 B, SW32
    static constexpr int kStage = kBTile + G * kASlot;     // multiple of 1024
    static constexpr int kCols = kStages * kStage;         // int[kColCache]
    static constexpr int kMeta = kCols + kColCache * 4;
    // meta: full[kStages], empty[kStages], acc (u64); mask[kStages] (int); row_ptr[G+1];
    //       tmem base; abort flag
    static constexpr int kFull = kMeta;
    static constexpr int kEmpty = kFull + 8 * kStages;
    static constexpr int kAcc = kEmpty + 8 * kStages;
    static constexpr int kMask = kAcc + 8;
    static constexpr int kRp = kMask + 4 * kStages;
    static constexpr int kTmem = kRp + 4 * (G + 1);
    static constexpr int kAbort = kTmem + 4;
    // Producer schedule of one batch of kStages steps: block column, row mask, and the block
    // index of each of the G block-rows (where its mask bit is set).
    static constexpr int kSchedBc = kAbort + 4;
    static constexpr int kSchedMask = kSchedBc + 4 * kStages;
    static constexpr int kSchedBlk = kSchedMask + 4 * kStages;
    static constexpr int kBytes = kSchedBlk + 4 * kStages * G;
    static constexpr int kDynamic = kBytes + 1024;         // room to align the base to 1 KB
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test of a phase.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait, slow path: polls with the abort flag and the clock checked every 64 polls
// (the clock is read only once a wait has lasted that long: a %globaltimer read costs
// hundreds of nanoseconds, which at one read per wait dominated the producer's step time).
__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    unsigned long long t0 = 0;
    for (uint32_t it = 0; it < (1u << 26); ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63) == 63) {
            if (*abort_flag) return false;
            const unsigned long long t = global_ns();
            if (t0 == 0) t0 = t;
            else if (t - t0 > kWaitNs) return false;
        }
    }
    return false;
}

// Bounded wait: true when the phase completed; false on timeout or when another role of the
// CTA has already given up (abort flag). One poll inline, the rest out of line.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, abort_flag);
}

__device__ __forceinline__ void mbar_arrive_count(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z,
                                            int w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05 "version 1" format): start address, leading and
// stride byte offsets (16-byte units), swizzle mode in bits 61..63.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint64_t swizzle) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr & 0x3ffffu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32;
    d |= 1ull << 46;
    d |= swizzle << 61;
    return d;
}

constexpr uint64_t kSwizzle128 = 2;
constexpr uint64_t kSwizzle32 = 6;

// Instruction descriptor for kind::f16: D = F32, A and B the same 16-bit type, A MN-major,
// B K-major, M = 128, N = n (16 .. 256, a multiple of 16).
__device__ __forceinline__ uint32_t instr_desc(int dtype, uint32_t n) {
    const uint32_t fmt = dtype == SPMM_DTYPE_BF16 ? 1u : 0u;
    return (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 15) | (0u << 16) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

template <int G, bool SCHED>
__global__ void __launch_bounds__(kTcThreads, 1)
    bsr_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ CUtensorMap tmap_a,
                       const __grid_constant__ CUtensorMap tmap_a4, BsrArgs a) {
    using L = Layout<G>;
    extern __shared__ uint8_t smem_raw[];
    // 1 KB alignment (SW128 atoms) in the shared address space.
    const uint32_t raw = smem_addr(smem_raw);
    uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const uint32_t sbase = smem_addr(base);

    int* cols = reinterpret_cast<int*>(base + L::kCols);
    int* masks = reinterpret_cast<int*>(base + L::kMask);
    int* rp = reinterpret_cast<int*>(base + L::kRp);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + L::kTmem);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(base + L::kAbort);
    const uint32_t full0 = sbase + L::kFull, empty0 = sbase + L::kEmpty, acc_bar = sbase + L::kAcc;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int br0 = blockIdx.x * G;
    const int n0 = blockIdx.y * 128;

    // Launched as a programmatic dependent of the previous kernel in the stream: no global memory
    // is read or written before grid_dependency_wait(). A planned CTA's setup (barriers, TMEM)
    // touches only shared memory and TMEM, so it overlaps the previous kernel's tail; the per-call
    // kernel reads row pointers first, so it waits at once.
    if constexpr (!SCHED) grid_dependency_wait();
    if (threadIdx.x == 0) allow_dependent_launch();

    // Block-row extents and the group's block-column list (prefix up to kColCache); with a
    // precomputed schedule neither is needed.
    const int* my_sched = SCHED ? a.sched + static_cast<size_t>(blockIdx.x) * a.sched_stride : nullptr;
    if (!SCHED && threadIdx.x <= G) {
        const int br = min(br0 + static_cast<int>(threadIdx.x), a.block_rows);
        int v = __ldg(a.row_ptr + br);
        v = max(0, min(v, a.num_blocks));
        rp[threadIdx.x] = v;
    }
    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full0 + 8 * s, kFullArrivals);
            mbar_init(empty0 + 8 * s, 1);
        }
        mbar_init(acc_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(sbase + L::kTmem, G * 16 <= 32 ? 32 : (G * 16 <= 64 ? 64 : 128));
    __syncthreads();
    if constexpr (SCHED) grid_dependency_wait();
    // Monotone block-row extents.
    int lo = 0;
    if constexpr (!SCHED) {
        lo = rp[0];
        int hi = lo;
        for (int j = 1; j <= G; ++j) hi = max(hi, rp[j]);
        for (int i = threadIdx.x; i < min(hi - lo, kColCache); i += kTcThreads) cols[i] = __ldg(a.col_idx + lo + i);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer: merge G block-column lists, load tiles
        // Batches of up to kStages steps: first the merge decides each step's block column and
        // rows (a short serial loop on shared memory, no waits), then lane k of the warp
        // claims step k's ring slot and issues its loads, all lanes at once. One step at a
        // time (wait, arrive, TMA issue, next merge step) measured ~0.6 us per step on B200
        // and made the producer the critical path.
        int* sched_bc = reinterpret_cast<int*>(base + L::kSchedBc);
        int* sched_mask = reinterpret_cast<int*>(base + L::kSchedMask);
        int* sched_blk = reinterpret_cast<int*>(base + L::kSchedBlk);
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
            if (a.a_stride > 0)
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a4)) : "memory");
        }
        int cur = 0, end = 0;
        if (!SCHED && lane < G) {
            cur = rp[lane];
            end = max(cur, rp[lane + 1]);
        }
        const int total_steps = SCHED ? __ldg(my_sched) : 0;
        int step = 0;           // steps fully issued so far
        unsigned last_issued = 0;  // stages of the last batch whose loads were issued
        int last_nb = 0;
        bool ok = true, done = false;
        while (ok && !done) {
            int nb = 0;
            if constexpr (SCHED) {
                // The batch's entries, one per lane, straight from the schedule. They are loaded
                // before the step count is known (one dependent memory round trip fewer before the
                // first copy is issued): the schedule is padded by a batch of entries past its
                // last record, so these loads stay inside it; entries past the count are ignored.
                int e_bc = 0, e_mask = 0, e_blk[G];
                if (lane < kStages) {
                    const int* e = my_sched + 2 + (step + lane) * (2 + G);
                    e_bc = __ldg(e);
                    e_mask = __ldg(e + 1);
#pragma unroll
                    for (int j = 0; j < G; ++j) e_blk[j] = __ldg(e + 2 + j);
                }
                nb = min(kStages, total_steps - step);
                if (lane < nb) {
                    sched_bc[lane] = e_bc;
                    sched_mask[lane] = e_mask;
#pragma unroll
                    for (int j = 0; j < G; ++j) sched_blk[lane * G + j] = e_blk[j];
                }
                done = step + nb >= total_steps;
            }
            for (; !SCHED && nb < kStages; ++nb) {
                int my = INT_MAX;
                if (lane < G && cur < end) {
                    const int off = cur - lo;
                    my = off < kColCache ? cols[off] : __ldg(a.col_idx + cur);
                    if (my < 0 || my >= a.block_cols) {
                        record_device_error(a.err, SPMM_ERR_BAD_INDEX, cur);
                        my = max(0, min(my, a.block_cols - 1));
                    }
                }
                const int bc = __reduce_min_sync(kFullMask, my);
                if (bc == INT_MAX) {
                    done = true;
                    break;
                }
                const unsigned mask = __ballot_sync(kFullMask, lane < G && my == bc);
                if (lane == 0) {
                    sched_bc[nb] = bc;
                    sched_mask[nb] = static_cast<int>(mask);
                }
                if (lane < G) sched_blk[nb * G + lane] = cur;
                if ((mask >> lane) & 1u) ++cur;
            }
            __syncwarp();
            bool mine = true;
            if (lane < nb) {
                const int t = step + lane;
                const int sl = t % kStages;
                mine = mbar_wait(empty0 + 8 * sl, ((t / kStages) & 1u) ^ 1u, abort_flag);
                if (mine) {
                    const uint32_t stage = sbase + sl * L::kStage;
                    masks[sl] = sched_mask[lane];
                    const unsigned mask = static_cast<unsigned>(sched_mask[lane]);
                    mbar_arrive_expect_tx(full0 + 8 * sl, L::kBTile + __popc(mask) * L::kASlot);
                    // The B tile: one TMA copy per 64-column half (128-byte swizzle); each block
                    // one 16 x 16 box (32-byte swizzle, K-major as the MMA reads it).
                    tma_load_2d(stage, &tmap_b, full0 + 8 * sl, n0, sched_bc[lane] * 16);
                    tma_load_2d(stage + 2048, &tmap_b, full0 + 8 * sl, n0 + 64, sched_bc[lane] * 16);
                    // A's blocks: one grouped copy when they are S apart in the value array (and
                    // the group lies inside the grouped view), else one copy per block.
                    const int p0 = sched_blk[lane * G];
                    bool grouped = a.a_stride > 0 && mask == (1u << G) - 1u && p0 >= 0 &&
                                   p0 / a.a_stride + G - 1 < a.a_groups;
#pragma unroll
                    for (int j = 1; j < G; ++j) grouped = grouped && sched_blk[lane * G + j] == p0 + j * a.a_stride;
                    if (grouped) {
                        tma_load_4d(stage + L::kBTile, &tmap_a4, full0 + 8 * sl, 0, 0, p0 % a.a_stride,
                                    p0 / a.a_stride);
                    } else {
                        for (unsigned m = mask; m; m &= m - 1) {
                            const int j = __ffs(m) - 1;
                            tma_load_2d(stage + L::kBTile + j * L::kASlot, &tmap_a, full0 + 8 * sl, 0,
                                        sched_blk[lane * G + j] * 16);
                        }
                    }
                }
            }
            const unsigned issued = __ballot_sync(kFullMask, lane < nb && mine);
            __syncwarp();
            last_issued = issued;
            last_nb = nb;
            if (issued != (nb >= 32 ? kFullMask : ((1u << nb) - 1u))) {
                ok = false;
                break;
            }
            step += nb;
            last_issued = 0;
            last_nb = 0;
            __syncwarp();  // every lane is done with this batch's schedule
        }
        if (ok) {
            // End marker in the next slot.
            const int sl = step % kStages;
            if (lane == 0) {
                ok = mbar_wait(empty0 + 8 * sl, ((step / kStages) & 1u) ^ 1u, abort_flag);
                if (ok) {
                    masks[sl] = kDone;
                    mbar_arrive_count(full0 + 8 * sl, kFullArrivals);
                }
            }
            ok = __shfl_sync(kFullMask, ok ? 1 : 0, 0) != 0;
        }
        if (!ok && lane == 0) {
            *abort_flag = 1;
            record_device_error(a.err, SPMM_ERR_TIMEOUT, 1);
            // Let the copies issued for the last stages land before the CTA's shared memory
            // is released (each wait is bounded again).
            for (int t = max(0, step + last_nb - kStages); t < step + last_nb; ++t) {
                if (t >= step && !((last_issued >> (t - step)) & 1u)) continue;
                const unsigned long long t0 = global_ns();
                while (!mbar_try_wait(full0 + 8 * (t % kStages), (t / kStages) & 1u) && global_ns() - t0 < kWaitNs) {
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (one thread)
        if (lane == 0) {
            const uint32_t idesc = instr_desc(a.dtype, 16);
            // A stage holding the block column for all G block-rows is one MMA with N = 16 G:
            // the blocks sit in consecutive 512-byte slots, i.e. one K-major operand of 16 G
            // rows, and the accumulator columns of the G block-rows are consecutive too.
            const uint32_t idesc_all = instr_desc(a.dtype, 16 * G);
            constexpr unsigned kAll = (1u << G) - 1u;
            unsigned started = 0;
            bool ok = true, done = false;
            int step = 0;
            while (!done) {
                // Wait for the next stage, then also take every following stage that has
                // already landed.
                if (!mbar_wait(full0 + 8 * (step % kStages), (step / kStages) & 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                int n = 1;
                while (n < kStages && mbar_test_wait(full0 + 8 * ((step + n) % kStages), ((step + n) / kStages) & 1u)) ++n;
                tc_fence_after();
                for (int k = 0; k < n; ++k) {
                    const int s = (step + k) % kStages;
                    const int mask = masks[s];
                    if (mask == kDone) {
                        done = true;
                        break;
                    }
                    const uint32_t stage = sbase + s * L::kStage;
                    const uint64_t adesc = smem_desc(stage, 2048, 1024, kSwizzle128);
                    if (static_cast<unsigned>(mask) == kAll && (started == 0 || started == kAll)) {
                        const uint64_t bdesc = smem_desc(stage + L::kBTile, 16, 256, kSwizzle32);
                        umma_f16(tmem, adesc, bdesc, idesc_all, started == kAll ? 1u : 0u);
                        started = kAll;
                    } else {
                        for (int j = 0; j < G; ++j) {
                            if (!((mask >> j) & 1)) continue;
                            const uint64_t bdesc = smem_desc(stage + L::kBTile + j * L::kASlot, 16, 256, kSwizzle32);
                            umma_f16(tmem + 16 * j, adesc, bdesc, idesc, (started >> j) & 1u);
                            started |= 1u << j;
                        }
                    }
                    umma_commit(empty0 + 8 * s);
                }
                step += n;
            }
            umma_commit(acc_bar);  // arrives when every MMA issued above has completed
            if (!ok) {
                *abort_flag = 1;
                record_device_error(a.err, SPMM_ERR_TIMEOUT, 2);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: TMEM -> registers -> C
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int rows_mask = SCHED ? __ldg(my_sched + 1) : 0;
        const bool ok = __all_sync(kFullMask, mbar_wait(acc_bar, 0, abort_flag));
        tc_fence_after();
        const int col = n0 + q * 32 + lane;
        for (int j = 0; j < G; ++j) {
            const int br = br0 + j;
            if (br >= a.block_rows) break;
            uint32_t v[16];
            const bool has = SCHED ? ((rows_mask >> j) & 1) != 0 : rp[j + 1] > rp[j];
            if (ok && has) {
                tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + 16 * j, v);
            } else {
#pragma unroll
                for (int r = 0; r < 16; ++r) v[r] = 0u;
            }
            if (col < a.N) {
#pragma unroll
                for (int r = 0; r < 16; ++r) {
                    const int row = br * 16 + r;
                    if (row < a.M) __stcs(a.C + static_cast<size_t>(row) * a.N + col, __uint_as_float(v[r]));
                }
            }
        }
        if (!ok && lane == 0) record_device_error(a.err, SPMM_ERR_TIMEOUT, 3);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, G * 16 <= 32 ? 32 : (G * 16 <= 64 ? 64 : 128));
    }
}

// CUDA-core BSR kernel: one CTA per (block-row, 128-column slice), a thread per column,
// 16 row accumulators per thread, each block staged in shared memory as FP32.
template <bool BF16>
__global__ void __launch_bounds__(128) bsr_cudacore_kernel(BsrArgs a) {
    __shared__ float As[256];
    const int br = blockIdx.x;
    const int n = blockIdx.y * 128 + threadIdx.x;
    float acc[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) acc[r] = 0.f;
    const int b0 = max(0, min(__ldg(a.row_ptr + br), a.num_blocks));
    const int b1 = max(b0, min(__ldg(a.row_ptr + br + 1), a.num_blocks));
    for (int b = b0; b < b1; ++b) {
        __syncthreads();
        for (int i = threadIdx.x; i < 256; i += 128) {
            const uint16_t h = __ldg(a.values + static_cast<size_t>(b) * 256 + i);
            if constexpr (BF16) As[i] = __uint_as_float(static_cast<uint32_t>(h) << 16);
            else As[i] = __half2float(__ushort_as_half(h));
        }
        __syncthreads();
        int bc = __ldg(a.col_idx + b);
        if (bc < 0 || bc >= a.block_cols) {
            if (threadIdx.x == 0) record_device_error(a.err, SPMM_ERR_BAD_INDEX, b);
            continue;
        }
        if (n >= a.N) continue;
        for (int k = 0; k < 16; ++k) {
            const int kk = bc * 16 + k;
            if (kk >= a.K) break;
            const uint16_t h = __ldg(a.B + static_cast<size_t>(kk) * a.N + n);
            float bv;
            if constexpr (BF16) bv = __uint_as_float(static_cast<uint32_t>(h) << 16);
            else bv = __half2float(__ushort_as_half(h));
#pragma unroll
            for (int r = 0; r < 16; ++r) acc[r] = fmaf(As[r * 16 + k], bv, acc[r]);
        }
    }
    if (n < a.N) {
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const int row = br * 16 + r;
            if (row < a.M) a.C[static_cast<size_t>(row) * a.N + n] = acc[r];
        }
    }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        cudaGetLastError();
    });
    return fn;
}

int encode_2d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
              uint32_t box_outer, CUtensorMapSwizzle swz) {
    auto enc = tensor_map_encoder();
    if (!enc) return SPMM_ERR_UNSUPPORTED;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? SPMM_OK : SPMM_ERR_INVALID_ARG;
}

int encode_b_map(CUtensorMap* tb, const BsrArgs& a) {
    return encode_2d(tb, a.B, static_cast<uint64_t>(a.N), static_cast<uint64_t>(a.K), static_cast<uint64_t>(a.N) * 2, 64,
                     16, CU_TENSOR_MAP_SWIZZLE_128B);
}

int encode_a_map(CUtensorMap* ta, const BsrArgs& a) {
    return encode_2d(ta, a.values, 16, static_cast<uint64_t>(a.num_blocks) * 16, 32, 16, 16, CU_TENSOR_MAP_SWIZZLE_32B);
}

// A's blocks as [num_blocks / S][S][16][16] (blocks past the last whole group left out): a box of
// {16, 16, 1, G} at (0, 0, p % S, p / S) is blocks p, p + S, ..., p + (G-1) S, landing as G
// consecutive 512-byte SW32 slots, the layout of G single-block copies.
int encode_a_group_map(CUtensorMap* map, const BsrArgs& a, int S, int G) {
    auto enc = tensor_map_encoder();
    if (!enc) return SPMM_ERR_UNSUPPORTED;
    const cuuint64_t dims[4] = {16, 16, static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(a.num_blocks / S)};
    const cuuint64_t strides[3] = {32, 512, 512ull * static_cast<cuuint64_t>(S)};
    const cuuint32_t box[4] = {16, 16, 1, static_cast<cuuint32_t>(G)};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<uint16_t*>(a.values), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? SPMM_OK : SPMM_ERR_INVALID_ARG;
}

// The block stride S of the grouped A copies: the most common distance between the blocks of
// consecutive block-rows in the schedule's full steps (every row of the group present and the
// blocks evenly spaced), over the first `ints` entries of a schedule copied to the host. 0 when
// no full step is evenly spaced. Any S is safe: the kernel checks every stage against it.
int pick_a_stride(const std::vector<int>& sched, int stride, int groups, int G) {
    std::vector<std::pair<int, int>> counts;  // (S, steps)
    const unsigned all = (1u << G) - 1u;
    for (int g = 0; g < groups; ++g) {
        const size_t rec = static_cast<size_t>(g) * stride;
        if (rec + 2 > sched.size()) break;
        const int steps = sched[rec];
        for (int t = 0; t < steps; ++t) {
            const size_t e = rec + 2 + static_cast<size_t>(t) * (2 + G);
            if (e + 2 + G > sched.size()) break;
            if (static_cast<unsigned>(sched[e + 1]) != all) continue;
            const int d = sched[e + 3] - sched[e + 2];
            bool even = d > 0;
            for (int j = 2; j < G && even; ++j) even = sched[e + 2 + j] - sched[e + 2 + j - 1] == d;
            if (!even) continue;
            auto it = std::find_if(counts.begin(), counts.end(), [d](const std::pair<int, int>& c) { return c.first == d; });
            if (it == counts.end()) {
                if (counts.size() < 64) counts.emplace_back(d, 1);
            } else {
                ++it->second;
            }
        }
    }
    int best = 0, best_n = 0;
    for (const auto& c : counts)
        if (c.second > best_n) best = c.first, best_n = c.second;
    return best;
}

template <int G, bool SCHED>
int launch_tc_maps(const BsrArgs& a, const CUtensorMap& tb, const CUtensorMap& ta, const CUtensorMap& ta4,
                   cudaStream_t s) {
    using L = Layout<G>;
    // The shared-memory attribute belongs to the current device's context: set it once per
    // device (a bit per device id), not on every launch.
    static std::atomic<unsigned long long> attr_set{0};
    int dev = 0;
    SPMM_CUDA_TRY(cudaGetDevice(&dev));
    const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
    if (!bit || !(attr_set.load(std::memory_order_acquire) & bit)) {
        SPMM_CUDA_TRY(cudaFuncSetAttribute(bsr_tcgen05_kernel<G, SCHED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           L::kDynamic));
        attr_set.fetch_or(bit, std::memory_order_acq_rel);
    }
    // A programmatic dependent of the previous kernel in the stream (the kernel waits for it
    // before touching global memory).
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((a.block_rows + G - 1) / G, (a.N + 127) / 128);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = L::kDynamic;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SPMM_CUDA_TRY(cudaLaunchKernelEx(&cfg, bsr_tcgen05_kernel<G, SCHED>, tb, ta, ta4, a));
    return SPMM_OK;
}

template <int G>
int launch_tc(const BsrArgs& a, cudaStream_t s) {
    CUtensorMap tb, ta;
    SPMM_TRY(encode_b_map(&tb, a));
    SPMM_TRY(encode_a_map(&ta, a));
    return launch_tc_maps<G, false>(a, tb, ta, ta, s);  // a.a_stride == 0: no grouped copies
}

// Plans: the producer's merge of G block-column lists, done once for every CTA group and
// stored as a fixed-stride schedule (one warp per group). count != 0: only the step count
// (atomicMax into *max_steps); else the records.
template <int G>
__global__ void __launch_bounds__(256) bsr_schedule_kernel(BsrArgs a, int* sched, int stride, int* max_steps,
                                                          int count) {
    const int lane = threadIdx.x & 31;
    const int g = static_cast<int>((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
    const int groups = (a.block_rows + G - 1) / G;
    if (g >= groups) return;
    const int br0 = g * G;
    int cur = 0, end = 0;
    if (lane < G) {
        const int br = min(br0 + lane, a.block_rows);
        const int br1 = min(br0 + lane + 1, a.block_rows);
        cur = max(0, min(__ldg(a.row_ptr + br), a.num_blocks));
        end = max(cur, min(__ldg(a.row_ptr + br1), a.num_blocks));
    }
    const unsigned rows = __ballot_sync(kFullMask, lane < G && end > cur);
    int* rec = sched + static_cast<size_t>(g) * stride;
    int steps = 0;
    for (;;) {
        int my = INT_MAX;
        if (lane < G && cur < end) {
            my = __ldg(a.col_idx + cur);
            if (my < 0 || my >= a.block_cols) {
                if (count) record_device_error(a.err, SPMM_ERR_BAD_INDEX, cur);
                my = max(0, min(my, a.block_cols - 1));
            }
        }
        const int bc = __reduce_min_sync(kFullMask, my);
        if (bc == INT_MAX) break;
        const unsigned mask = __ballot_sync(kFullMask, lane < G && my == bc);
        if (!count) {
            int* e = rec + 2 + steps * (2 + G);
            if (lane == 0) {
                e[0] = bc;
                e[1] = static_cast<int>(mask);
            }
            if (lane < G) e[2 + lane] = ((mask >> lane) & 1u) ? cur : 0;
        }
        if ((mask >> lane) & 1u) ++cur;
        ++steps;
    }
    if (lane == 0) {
        if (count) {
            atomicMax(max_steps, steps);
        } else {
            rec[0] = steps;
            rec[1] = static_cast<int>(rows);
        }
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// algo: 0 auto, 1 tensor cores (error if the operands do not fit it), 2 CUDA cores.
int bsr16_launch(const spmm_bsr_view* A, const void* B16, float* C, int32_t N, int32_t algo, cudaStream_t s,
                 DeviceState* st) {
    if (!A || N < 0 || A->rows < 0 || A->cols < 0 || A->num_blocks < 0 || A->block_rows < 0) return SPMM_ERR_INVALID_ARG;
    if (A->dtype != SPMM_DTYPE_F16 && A->dtype != SPMM_DTYPE_BF16) return SPMM_ERR_INVALID_ARG;
    if (A->block_rows != (A->rows + 15) / 16 || A->block_cols != (A->cols + 15) / 16) return SPMM_ERR_INVALID_ARG;
    if (algo < 0 || algo > 2) return SPMM_ERR_INVALID_ARG;
    if (A->rows == 0 || N == 0) return SPMM_OK;
    if (!C || !A->row_ptr || (A->num_blocks > 0 && (!A->col_idx || !A->values || !B16))) return SPMM_ERR_INVALID_ARG;
    if (A->num_blocks > (1 << 26)) return SPMM_ERR_TOO_LARGE;
    BsrArgs a{};
    a.M = A->rows;
    a.K = A->cols;
    a.N = N;
    a.block_rows = A->block_rows;
    a.block_cols = A->block_cols;
    a.num_blocks = A->num_blocks;
    a.row_ptr = A->row_ptr;
    a.col_idx = A->col_idx;
    a.values = A->values;
    a.B = static_cast<const uint16_t*>(B16);
    a.C = C;
    a.dtype = A->dtype;
    a.err = st->err;
    const bool tc_ok = st->cc_major == 10 && N % 8 == 0 && A->num_blocks > 0 && A->cols > 0 && aligned16(B16) &&
                       aligned16(A->values);
    if (algo == 1 && !tc_ok) return SPMM_ERR_MISALIGNED;
    if (algo != 2 && tc_ok) {
        // Eight block-rows per CTA when that still fills the GPU, else four.
        const long long ctas8 = static_cast<long long>((a.block_rows + 7) / 8) * ((N + 127) / 128);
        if (ctas8 >= st->sm_count) return launch_tc<8>(a, s);
        return launch_tc<4>(a, s);
    }
    const dim3 grid(a.block_rows, (N + 127) / 128);
    if (a.dtype == SPMM_DTYPE_BF16) bsr_cudacore_kernel<true><<<grid, 128, 0, s>>>(a);
    else bsr_cudacore_kernel<false><<<grid, 128, 0, s>>>(a);
    SPMM_CUDA_TRY(cudaGetLastError());
    return SPMM_OK;
}

}  // namespace spmm_b200

using namespace spmm_b200;

extern "C" {

int spmm_bsr16_algo(const spmm_bsr_view* A, const void* B16, float* C, int32_t N, int32_t algo, void* stream) {
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    return bsr16_launch(A, B16, C, N, algo, as_stream(stream), st);
}

int spmm_bsr16(const spmm_bsr_view* A, const void* B16, float* C, int32_t N, void* stream) {
    return spmm_bsr16_algo(A, B16, C, N, 0, stream);
}

int spmm_bsr16_plan_create(const spmm_bsr_view* A, int32_t N, void* stream, spmm_bsr_plan** out) {
    if (!A || !out || N < 0 || A->rows < 0 || A->cols < 0 || A->num_blocks < 0 || A->block_rows < 0)
        return SPMM_ERR_INVALID_ARG;
    if (A->dtype != SPMM_DTYPE_F16 && A->dtype != SPMM_DTYPE_BF16) return SPMM_ERR_INVALID_ARG;
    if (A->block_rows != (A->rows + 15) / 16 || A->block_cols != (A->cols + 15) / 16) return SPMM_ERR_INVALID_ARG;
    if (A->rows > 0 && (!A->row_ptr || (A->num_blocks > 0 && (!A->col_idx || !A->values)))) return SPMM_ERR_INVALID_ARG;
    if (A->num_blocks > (1 << 26)) return SPMM_ERR_TOO_LARGE;
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    const cudaStream_t s = as_stream(stream);
    spmm_bsr_plan* p = new (std::nothrow) spmm_bsr_plan();
    if (!p) return SPMM_ERR_NO_MEMORY;
    p->A = *A;
    p->N = N;
    p->device = st->device;
    p->tc = st->cc_major == 10 && N % 8 == 0 && N > 0 && A->rows > 0 && A->num_blocks > 0 && A->cols > 0 &&
            aligned16(A->values);
    int rc = SPMM_OK;
    if (p->tc) {
        const long long ctas8 = static_cast<long long>((A->block_rows + 7) / 8) * ((N + 127) / 128);
        p->group = ctas8 >= st->sm_count ? 8 : 4;
        BsrArgs a{};
        a.block_rows = A->block_rows;
        a.block_cols = A->block_cols;
        a.num_blocks = A->num_blocks;
        a.row_ptr = A->row_ptr;
        a.col_idx = A->col_idx;
        a.values = A->values;
        a.err = st->err;
        rc = encode_a_map(&p->ta, a);
        const int groups = (A->block_rows + p->group - 1) / p->group;
        const unsigned blocks = static_cast<unsigned>((static_cast<long long>(groups) * 32 + 255) / 256);
        int* d_max = nullptr;
        if (rc == SPMM_OK && cudaMalloc(&d_max, sizeof(int)) != cudaSuccess) rc = SPMM_ERR_NO_MEMORY;
        if (rc == SPMM_OK && cudaMemsetAsync(d_max, 0, sizeof(int), s) != cudaSuccess) rc = SPMM_ERR_CUDA;
        if (rc == SPMM_OK) {
            if (p->group == 8) bsr_schedule_kernel<8><<<blocks, 256, 0, s>>>(a, nullptr, 0, d_max, 1);
            else bsr_schedule_kernel<4><<<blocks, 256, 0, s>>>(a, nullptr, 0, d_max, 1);
            if (cudaGetLastError() != cudaSuccess ||
                cudaMemcpyAsync(&p->max_steps, d_max, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
                cudaStreamSynchronize(s) != cudaSuccess)
                rc = SPMM_ERR_CUDA;
        }
        cudaFree(d_max);
        // A schedule of at most 256 MiB; beyond that the kernel merges on the fly.
        if (rc == SPMM_OK) {
            p->stride = 2 + p->max_steps * (2 + p->group);
            // Padded by one batch of entries: the kernel loads a batch before it knows how many
            // of its entries are real.
            const size_t bytes = sizeof(int) * (static_cast<size_t>(groups) * static_cast<size_t>(p->stride) +
                                                static_cast<size_t>(kStages) * (2 + p->group));
            if (bytes <= (256ull << 20)) {
                if (cudaMalloc(&p->sched, bytes) != cudaSuccess) {
                    rc = SPMM_ERR_NO_MEMORY;
                } else if (cudaMemsetAsync(p->sched, 0, bytes, s) != cudaSuccess) {
                    rc = SPMM_ERR_CUDA;
                } else {
                    p->sched_bytes = bytes;
                    if (p->group == 8) bsr_schedule_kernel<8><<<blocks, 256, 0, s>>>(a, p->sched, p->stride, nullptr, 0);
                    else bsr_schedule_kernel<4><<<blocks, 256, 0, s>>>(a, p->sched, p->stride, nullptr, 0);
                    if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess) rc = SPMM_ERR_CUDA;
                }
            }
        }
        // Grouped A copies: the block stride from (at most 1 MiB of) the schedule.
        if (rc == SPMM_OK && p->sched) {
            const size_t ints = std::min<size_t>(p->sched_bytes / sizeof(int), (1u << 20) / sizeof(int));
            std::vector<int> host(ints);
            if (cudaMemcpyAsync(host.data(), p->sched, ints * sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
                cudaStreamSynchronize(s) != cudaSuccess) {
                rc = SPMM_ERR_CUDA;
            } else {
                const int S = pick_a_stride(host, p->stride, groups, p->group);
                if (S > 0 && A->num_blocks / S >= p->group && encode_a_group_map(&p->ta4, a, S, p->group) == SPMM_OK) {
                    p->a_stride = S;
                    p->a_groups = A->num_blocks / S;
                }
            }
        }
    }
    if (rc != SPMM_OK) {
        cudaFree(p->sched);
        delete p;
        return rc;
    }
    *out = p;
    return SPMM_OK;
}

int spmm_bsr16_plan_execute(const spmm_bsr_plan* p, const void* B16, float* C, void* stream) {
    if (!p) return SPMM_ERR_INVALID_ARG;
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    if (st->device != p->device) return SPMM_ERR_INVALID_ARG;
    const cudaStream_t s = as_stream(stream);
    if (!p->tc || !p->sched || !aligned16(B16)) return bsr16_launch(&p->A, B16, C, p->N, 0, s, st);
    if (!C || !B16) return SPMM_ERR_INVALID_ARG;
    BsrArgs a{};
    a.M = p->A.rows;
    a.K = p->A.cols;
    a.N = p->N;
    a.block_rows = p->A.block_rows;
    a.block_cols = p->A.block_cols;
    a.num_blocks = p->A.num_blocks;
    a.row_ptr = p->A.row_ptr;
    a.col_idx = p->A.col_idx;
    a.values = p->A.values;
    a.B = static_cast<const uint16_t*>(B16);
    a.C = C;
    a.dtype = p->A.dtype;
    a.err = st->err;
    a.sched = p->sched;
    a.sched_stride = p->stride;
    a.a_stride = p->a_stride;
    a.a_groups = p->a_groups;
    CUtensorMap tb;
    {
        std::lock_guard<std::mutex> lock(p->tb_mu);
        if (p->tb_for != B16) {
            SPMM_TRY(encode_b_map(&p->tb, a));
            p->tb_for = B16;
        }
        tb = p->tb;
    }
    const CUtensorMap& ta4 = p->a_stride > 0 ? p->ta4 : p->ta;
    if (p->group == 8) return launch_tc_maps<8, true>(a, tb, p->ta, ta4, s);
    return launch_tc_maps<4, true>(a, tb, p->ta, ta4, s);
}

int spmm_bsr16_plan_info(const spmm_bsr_plan* p, int32_t* group, int32_t* max_steps, size_t* schedule_bytes) {
    if (!p) return SPMM_ERR_INVALID_ARG;
    if (group) *group = p->tc ? p->group : 0;
    if (max_steps) *max_steps = p->max_steps;
    if (schedule_bytes) *schedule_bytes = p->sched_bytes;
    return SPMM_OK;
}

int spmm_bsr16_plan_a_stride(const spmm_bsr_plan* p, int32_t* a_stride) {
    if (!p || !a_stride) return SPMM_ERR_INVALID_ARG;
    *a_stride = p->a_stride;
    return SPMM_OK;
}

void spmm_bsr16_plan_destroy(spmm_bsr_plan* p) {
    if (!p) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    cudaFree(p->sched);
    cudaSetDevice(prev);
    delete p;
}

}  // extern "C"
