// CSR SpMM plans: inspect a matrix once, then run it many times.
//
// spmm_csr_plan_create reads the device row_ptr once (one reduction kernel and a 4-byte
// read-back) for the longest row and picks the work distribution:
//   * ROWWARP when no row is much longer than a warp's fair share of the merge path --
//     longest row <= max(4 * (M + nnz) / resident warps, 256): one warp per row needs no
//     search and no fix-up and measured fastest on every such config on B200;
//   * MERGE otherwise (a skewed matrix: a warp per long row would be the straggler).
// The plan owns its workspace, so spmm_csr_plan_execute allocates nothing and only launches.

#include <cuda_runtime.h>

#include <algorithm>
#include <new>

#include "common.cuh"

struct spmm_csr_plan {
    spmm_csr_view A{};
    int32_t N = 0;
    int32_t algo = SPMM_CSR_MERGE;
    spmm_csr_tuning tune{};
    int32_t max_row = 0;
    int32_t device = 0;
    void* ws = nullptr;
    size_t ws_bytes = 0;
};

namespace spmm_b200 {


namespace {

constexpr int kResidentWarpsPerSm = 32;  // csr kernels: 4 CTAs x 8 warps

__global__ void max_row_kernel(const int* __restrict__ row_ptr, int M, int* out) {
    int best = 0;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < M; i += gridDim.x * blockDim.x)
        best = max(best, __ldg(row_ptr + i + 1) - __ldg(row_ptr + i));
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_down_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out, best);
}

// Column phases for ROWWARP. A random-row gather runs at the L2 rate (about 19-20 TB/s on
// B200) while B fits in about 80 % of the L2, and falls towards the HBM rate beyond it
// (14 TB/s at 128 MiB, 8 TB/s at 512 MiB). Phases bring B's footprint back into range at the
// price of re-reading and re-writing C per phase and one launch per phase, which only pays off
// on large launches. Measured on B200 (131072 rows x 131 nnz, N = 256), two regimes:
//   * B from 0.8x to 1.2x the L2 (config 5: 128 MiB, 1.06x): 400 back-to-back launches, where
//     one phase's 4 GB of DRAM traffic per launch let the SM clock sag to 1.5-1.75 GHz while
//     phased launches held 1.85-1.95 GHz: 3 phases -14 % of the time (1 GPU, 17.6 GB gathered),
//     -13 % at 8.8 GB (a rank of 2), -8 % at 4.4 GB (a rank of 4), a tie at 2.2 GB (a rank of 8);
//     2 and 4 phases -10 %, 6 phases -4 %. In short bursts at the full clock the phased and
//     unphased launches tie, so the phases cost nothing there.
//   * B above 1.2x the L2: 160 MiB of B 3 phases -4 %, 256 MiB 4 phases -13 %, 512 MiB 8 phases
//     -38 %, at >= 12 GB gathered; about one phase per half L2 of B.
int auto_phases(const spmm_csr_view* A, int32_t N, const DeviceState* st) {
    if (st->l2_bytes <= 0) return 1;
    const double b_bytes = 4.0 * A->cols * static_cast<double>(N);
    const double gather_bytes = 4.0 * A->nnz * static_cast<double>(N);
    const double l2 = st->l2_bytes;
    if (b_bytes > 0.8 * l2 && b_bytes <= 1.2 * l2) return gather_bytes >= 4e9 ? 3 : 1;
    if (b_bytes <= 1.2 * l2 || gather_bytes < 12e9) return 1;
    const int ph = static_cast<int>(b_bytes / (0.5 * l2) + 0.5);
    return std::min(std::max(ph, 1), 8);
}

}  // namespace
}  // namespace spmm_b200

using namespace spmm_b200;

extern "C" {

int spmm_csr_plan_create(const spmm_csr_view* A, int32_t N, const spmm_csr_tuning* tune, void* stream,
                         spmm_csr_plan** out) {
    if (!A || !out || N < 0 || A->rows < 0 || A->cols < 0 || A->nnz < 0) return SPMM_ERR_INVALID_ARG;
    if (A->rows > 0 && !A->row_ptr) return SPMM_ERR_INVALID_ARG;
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    const cudaStream_t s = as_stream(stream);
    spmm_csr_plan* p = new (std::nothrow) spmm_csr_plan();
    if (!p) return SPMM_ERR_NO_MEMORY;
    p->A = *A;
    p->N = N;
    p->device = st->device;
    if (tune) p->tune = *tune;
    int rc = SPMM_OK;
    if (A->rows > 0) {
        int* d = nullptr;
        if (cudaMalloc(&d, sizeof(int)) != cudaSuccess) rc = SPMM_ERR_NO_MEMORY;
        if (rc == SPMM_OK && cudaMemsetAsync(d, 0, sizeof(int), s) != cudaSuccess) rc = SPMM_ERR_CUDA;
        if (rc == SPMM_OK) {
            const int blocks = std::min((A->rows + 255) / 256, st->sm_count * 8);
            max_row_kernel<<<blocks, 256, 0, s>>>(A->row_ptr, A->rows, d);
            if (cudaGetLastError() != cudaSuccess ||
                cudaMemcpyAsync(&p->max_row, d, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
                cudaStreamSynchronize(s) != cudaSuccess)
                rc = SPMM_ERR_CUDA;
        }
        cudaFree(d);
    }
    if (rc == SPMM_OK) {
        const long long items = static_cast<long long>(A->rows) + A->nnz;
        const long long fair = items / (static_cast<long long>(st->sm_count) * kResidentWarpsPerSm);
        const long long limit = std::max<long long>(4 * fair, 256);
        p->algo = p->max_row <= limit ? SPMM_CSR_ROWWARP : SPMM_CSR_MERGE;
        if (p->algo == SPMM_CSR_ROWWARP) {
            if (p->tune.k_phases <= 0) p->tune.k_phases = auto_phases(A, N, st);
        } else {
            p->tune.k_phases = 0;
        }
        rc = csr_f32_workspace_bytes(A, N, p->algo, &p->tune, st->sm_count, &p->ws_bytes);
    }
    if (rc == SPMM_OK && p->ws_bytes) {
        if (cudaMalloc(&p->ws, p->ws_bytes) != cudaSuccess) rc = SPMM_ERR_NO_MEMORY;
        else if (cudaMemsetAsync(p->ws, 0, p->ws_bytes, s) != cudaSuccess) rc = SPMM_ERR_CUDA;
        else if (p->algo == SPMM_CSR_ROWWARP)
            rc = csr_f32_ksplit(&p->A, p->tune.k_phases, static_cast<int*>(p->ws), s, st);
        if (rc == SPMM_OK && cudaStreamSynchronize(s) != cudaSuccess) rc = SPMM_ERR_CUDA;
    }
    if (rc != SPMM_OK) {
        cudaFree(p->ws);
        delete p;
        return rc;
    }
    *out = p;
    return SPMM_OK;
}

int spmm_csr_plan_execute(const spmm_csr_plan* p, const float* B, float* C, void* stream) {
    if (!p) return SPMM_ERR_INVALID_ARG;
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    if (st->device != p->device) return SPMM_ERR_INVALID_ARG;
    return csr_f32_launch(&p->A, B, C, p->N, p->algo, &p->tune, p->ws, p->ws_bytes, as_stream(stream), st, true);
}

int spmm_csr_plan_k_phases(const spmm_csr_plan* p, int32_t* k_phases) {
    if (!p || !k_phases) return SPMM_ERR_INVALID_ARG;
    *k_phases = p->algo == SPMM_CSR_ROWWARP ? std::max(1, p->tune.k_phases) : 1;
    return SPMM_OK;
}

int spmm_csr_plan_launches(const spmm_csr_plan* p, int32_t* launches) {
    if (!p || !launches) return SPMM_ERR_INVALID_ARG;
    if (p->A.rows == 0 || p->N == 0) {
        *launches = 0;
        return SPMM_OK;
    }
    const bool phased = p->algo == SPMM_CSR_ROWWARP && p->tune.k_phases > 1;
    *launches = phased && p->tune.phase_mode != 2 ? p->tune.k_phases : 1;
    return SPMM_OK;
}

int spmm_csr_plan_info(const spmm_csr_plan* p, int32_t* algo, int32_t* max_row, size_t* ws_bytes) {
    if (!p) return SPMM_ERR_INVALID_ARG;
    if (algo) *algo = p->algo;
    if (max_row) *max_row = p->max_row;
    if (ws_bytes) *ws_bytes = p->ws_bytes;
    return SPMM_OK;
}

void spmm_csr_plan_destroy(spmm_csr_plan* p) {
    if (!p) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    cudaFree(p->ws);
    cudaSetDevice(prev);
    delete p;
}

}  // extern "C"
