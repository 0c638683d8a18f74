// CSR -> BSR-16 conversion on the GPU, bit-identical to the host conversion (and so to the
// reference's bsr_from_csr_host, src/bsr.cu:30-109): per block-row the sorted unique block
// columns, row_ptr by exclusive scan, every nonzero scattered into its block (a later
// duplicate of a coordinate wins), zero padding, FP32 -> FP16/BF16 round-to-nearest-even.
//
// One CTA per block-row keeps a bitmap of the block-row's block columns in shared memory
// (atomicOr per nonzero), so the unique sorted list is the bitmap's set bits and a block's
// index is a popcount prefix -- no sort. Two launches plus a scan:
//   count  : bitmap -> number of blocks of each block-row; also checks that columns are
//            sorted inside every row (duplicate handling relies on it);
//   scan   : exclusive scan of the counts -> BSR row_ptr, total = num_blocks;
//   fill   : bitmap again -> col_idx, zero the block-row's values, scatter the nonzeros.
// The bitmap holds up to kMaxBlockCols block columns (K <= 1,048,576); wider matrices and
// rows with unsorted columns are left to the host conversion (SPMM_ERR_UNSUPPORTED).

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <climits>

#include "common.cuh"

namespace spmm_b200 {
namespace {

constexpr int kConvThreads = 256;
constexpr int kMaxBlockCols = 65536;
constexpr int kWords = kMaxBlockCols / 32;

struct ConvArgs {
    int M, K, nnz, block_rows, block_cols;
    const int* __restrict__ row_ptr;
    const int* __restrict__ col_idx;
    const float* __restrict__ values;
    int* bsr_row_ptr;      // block_rows + 1
    int* bsr_col_idx;      // num_blocks
    uint16_t* bsr_values;  // num_blocks * 256
    int dtype;
    int* flags;            // [0] = first unsorted row + 1 (0: all sorted), [1] = bad index seen
    DeviceErrorRecord* err;
};

__device__ __forceinline__ int clampi(int x, int lo, int hi) { return x < lo ? lo : (x > hi ? hi : x); }

// Marks the block columns of block-row br in `bits`; returns the row_ptr of its 17 row
// boundaries in `rp` (clamped, monotone).
__device__ void build_bitmap(const ConvArgs& a, int br, uint32_t* bits, int* rp, bool check_sorted) {
    const int words = (a.block_cols + 31) / 32;
    for (int w = threadIdx.x; w < words; w += blockDim.x) bits[w] = 0u;
    if (threadIdx.x <= 16) {
        const int r = min(br * 16 + static_cast<int>(threadIdx.x), a.M);
        rp[threadIdx.x] = clampi(__ldg(a.row_ptr + r), 0, a.nnz);
    }
    __syncthreads();
    if (threadIdx.x == 0)
        for (int j = 1; j <= 16; ++j) rp[j] = max(rp[j], rp[j - 1]);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j = warp; j < 16; j += blockDim.x / 32) {
        const int p0 = rp[j], p1 = rp[j + 1];
        for (int p = p0 + lane; p < p1; p += 32) {
            const int c = __ldg(a.col_idx + p);
            if (c < 0 || c >= a.K) {
                atomicExch(a.flags + 1, 1);
                continue;
            }
            if (check_sorted && p + 1 < p1 && __ldg(a.col_idx + p + 1) < c) atomicCAS(a.flags, 0, br * 16 + j + 1);
            atomicOr(bits + (c >> 4) / 32, 1u << ((c >> 4) & 31));
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kConvThreads) bsr_count_kernel(ConvArgs a) {
    __shared__ uint32_t bits[kWords];
    __shared__ int rp[17];
    __shared__ int total;
    const int br = blockIdx.x;
    if (threadIdx.x == 0) total = 0;
    build_bitmap(a, br, bits, rp, true);
    const int words = (a.block_cols + 31) / 32;
    int mine = 0;
    for (int w = threadIdx.x; w < words; w += blockDim.x) mine += __popc(bits[w]);
    for (int o = 16; o > 0; o >>= 1) mine += __shfl_down_sync(0xffffffffu, mine, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(&total, mine);
    __syncthreads();
    if (threadIdx.x == 0) a.bsr_row_ptr[br + 1] = total;  // counts in [1..]; scanned next
}

// Inclusive scan of bsr_row_ptr[1..n] in place, bsr_row_ptr[0] = 0: one CTA, 1024 at a time.
__global__ void __launch_bounds__(1024) bsr_scan_kernel(int* data, int n) {
    __shared__ int warp_sums[32];
    __shared__ int carry;
    if (threadIdx.x == 0) {
        carry = 0;
        data[0] = 0;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int base = 0; base < n; base += 1024) {
        const int i = base + threadIdx.x;
        int v = i < n ? data[1 + i] : 0;
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += t;
        }
        if (lane == 31) warp_sums[warp] = v;
        __syncthreads();
        if (warp == 0) {
            int s = warp_sums[lane];
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += t;
            }
            warp_sums[lane] = s;
        }
        __syncthreads();
        const int add = carry + (warp > 0 ? warp_sums[warp - 1] : 0);
        if (i < n) data[1 + i] = v + add;
        __syncthreads();
        if (threadIdx.x == 1023) carry = v + add;
        __syncthreads();
    }
}

template <bool BF16>
__device__ __forceinline__ uint16_t to16(float x) {
    if constexpr (BF16) {
        const __nv_bfloat16 h = __float2bfloat16_rn(x);
        return *reinterpret_cast<const uint16_t*>(&h);
    } else {
        const __half h = __float2half_rn(x);
        return *reinterpret_cast<const uint16_t*>(&h);
    }
}

template <bool BF16>
__global__ void __launch_bounds__(kConvThreads) bsr_fill_kernel(ConvArgs a) {
    __shared__ uint32_t bits[kWords];
    __shared__ int wprefix[kWords];
    __shared__ int rp[17];
    const int br = blockIdx.x;
    build_bitmap(a, br, bits, rp, false);
    const int words = (a.block_cols + 31) / 32;
    // Exclusive popcount prefix over the words (one thread; the bitmap is at most 2048 words).
    if (threadIdx.x == 0) {
        int s = 0;
        for (int w = 0; w < words; ++w) {
            wprefix[w] = s;
            s += __popc(bits[w]);
        }
    }
    __syncthreads();
    const int base = a.bsr_row_ptr[br];
    const int nblk = a.bsr_row_ptr[br + 1] - base;
    // Block-column list (sorted by construction).
    for (int w = threadIdx.x; w < words; w += blockDim.x) {
        uint32_t m = bits[w];
        int k = wprefix[w];
        while (m) {
            const int b = __ffs(m) - 1;
            m &= m - 1;
            if (k < nblk) a.bsr_col_idx[base + k] = w * 32 + b;
            ++k;
        }
    }
    // Zero padding of the block-row's blocks, then the scatter.
    uint32_t* vals32 = reinterpret_cast<uint32_t*>(a.bsr_values + static_cast<size_t>(base) * 256);
    for (int i = threadIdx.x; i < nblk * 128; i += blockDim.x) vals32[i] = 0u;
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j = warp; j < 16; j += blockDim.x / 32) {
        const int p0 = rp[j], p1 = rp[j + 1];
        for (int p = p0 + lane; p < p1; p += 32) {
            const int c = __ldg(a.col_idx + p);
            if (c < 0 || c >= a.K) continue;
            // With sorted columns a repeated coordinate is adjacent; the last copy wins.
            if (p + 1 < p1 && __ldg(a.col_idx + p + 1) == c) continue;
            const int bc = c >> 4;
            const int w = bc / 32, b = bc & 31;
            const int k = wprefix[w] + __popc(bits[w] & ((1u << b) - 1u));
            if (k >= nblk) continue;
            a.bsr_values[(static_cast<size_t>(base) + k) * 256 + j * 16 + (c & 15)] = to16<BF16>(__ldg(a.values + p));
        }
    }
}

int check_conv(const spmm_csr_view* A) {
    if (!A || A->rows < 0 || A->cols < 0 || A->nnz < 0) return SPMM_ERR_INVALID_ARG;
    if (A->rows > 0 && !A->row_ptr) return SPMM_ERR_INVALID_ARG;
    if (A->nnz > 0 && (!A->col_idx || !A->values)) return SPMM_ERR_INVALID_ARG;
    if ((A->cols + 15) / 16 > kMaxBlockCols) return SPMM_ERR_UNSUPPORTED;
    return SPMM_OK;
}

ConvArgs make_args(const spmm_csr_view* A) {
    ConvArgs a{};
    a.M = A->rows;
    a.K = A->cols;
    a.nnz = A->nnz;
    a.block_rows = (A->rows + 15) / 16;
    a.block_cols = (A->cols + 15) / 16;
    a.row_ptr = A->row_ptr;
    a.col_idx = A->col_idx;
    a.values = A->values;
    return a;
}

}  // namespace
}  // namespace spmm_b200

using namespace spmm_b200;

extern "C" {

int spmm_csr_to_bsr16_device_count(const spmm_csr_view* dA, int32_t* d_bsr_row_ptr, int32_t* num_blocks,
                                   void* stream) {
    SPMM_TRY(check_conv(dA));
    if (!d_bsr_row_ptr || !num_blocks) return SPMM_ERR_INVALID_ARG;
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    const cudaStream_t s = as_stream(stream);
    ConvArgs a = make_args(dA);
    a.bsr_row_ptr = d_bsr_row_ptr;
    std::lock_guard<std::mutex> lock(st->mu);
    SPMM_TRY(ensure_device_buffer(&st->conv_flags, &st->conv_flags_bytes, 4 * sizeof(int), false, s));
    a.flags = static_cast<int*>(st->conv_flags);
    a.err = st->err;
    SPMM_CUDA_TRY(cudaMemsetAsync(a.flags, 0, 4 * sizeof(int), s));
    if (a.block_rows > 0) {
        bsr_count_kernel<<<a.block_rows, kConvThreads, 0, s>>>(a);
        SPMM_CUDA_TRY(cudaGetLastError());
    }
    bsr_scan_kernel<<<1, 1024, 0, s>>>(d_bsr_row_ptr, a.block_rows);
    SPMM_CUDA_TRY(cudaGetLastError());
    int host[4] = {0, 0, 0, 0};
    int total = 0;
    SPMM_CUDA_TRY(cudaMemcpyAsync(host, a.flags, sizeof(host), cudaMemcpyDeviceToHost, s));
    SPMM_CUDA_TRY(cudaMemcpyAsync(&total, d_bsr_row_ptr + a.block_rows, sizeof(int), cudaMemcpyDeviceToHost, s));
    SPMM_CUDA_TRY(cudaStreamSynchronize(s));
    if (host[1]) return SPMM_ERR_BAD_INDEX;
    if (host[0]) return SPMM_ERR_UNSUPPORTED;  // a row with unsorted columns: use the host path
    *num_blocks = total;
    return SPMM_OK;
}

int spmm_csr_to_bsr16_device_fill(const spmm_csr_view* dA, const int32_t* d_bsr_row_ptr, int32_t* d_col_idx,
                                  uint16_t* d_values, int32_t dtype, void* stream) {
    SPMM_TRY(check_conv(dA));
    if (!d_bsr_row_ptr || (dtype != SPMM_DTYPE_F16 && dtype != SPMM_DTYPE_BF16)) return SPMM_ERR_INVALID_ARG;
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    const cudaStream_t s = as_stream(stream);
    ConvArgs a = make_args(dA);
    if (a.block_rows == 0) return SPMM_OK;
    a.bsr_row_ptr = const_cast<int32_t*>(d_bsr_row_ptr);
    a.bsr_col_idx = d_col_idx;
    a.bsr_values = d_values;
    a.dtype = dtype;
    std::lock_guard<std::mutex> lock(st->mu);
    SPMM_TRY(ensure_device_buffer(&st->conv_flags, &st->conv_flags_bytes, 4 * sizeof(int), false, s));
    a.flags = static_cast<int*>(st->conv_flags);
    a.err = st->err;
    if (dtype == SPMM_DTYPE_BF16) bsr_fill_kernel<true><<<a.block_rows, kConvThreads, 0, s>>>(a);
    else bsr_fill_kernel<false><<<a.block_rows, kConvThreads, 0, s>>>(a);
    SPMM_CUDA_TRY(cudaGetLastError());
    return SPMM_OK;
}

}  // extern "C"
