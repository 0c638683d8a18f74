// Internal helpers shared by the CUDA translation units of libspmm_b200.so.
#pragma once

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <cstddef>
#include <cstdint>
#include <mutex>

#include "spmm_c.h"

namespace spmm_b200 {

// A named NVTX range over a host-side phase (copy issue, collective, launches), so that an
// nsys or ncu timeline of the host-buffer and multi-GPU paths splits into its phases. NVTX v3
// is header-only: without a profiler attached the push/pop calls return at once.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

// Return SPMM_ERR_CUDA from the enclosing function when a runtime call fails.
#define SPMM_CUDA_TRY(call)                                     \
    do {                                                        \
        cudaError_t e__ = (call);                               \
        if (e__ != cudaSuccess) {                               \
            spmm_b200::note_cuda_error(e__, #call, __FILE__, __LINE__); \
            return SPMM_ERR_CUDA;                               \
        }                                                       \
    } while (0)

#define SPMM_TRY(call)              \
    do {                            \
        int s__ = (call);           \
        if (s__ != SPMM_OK) return s__; \
    } while (0)

void note_cuda_error(cudaError_t e, const char* what, const char* file, int line);

// Device-side error record: word 0 = status code (first writer wins), word 1..2 = detail.
struct DeviceErrorRecord {
    int code;
    int pad;
    long long detail;
};

__device__ __forceinline__ void record_device_error(DeviceErrorRecord* rec, int code, long long detail) {
    if (rec && atomicCAS(&rec->code, 0, code) == 0) rec->detail = detail;
}

// Programmatic dependent launch (kernels launched with programmatic stream serialisation): wait
// until the previous grid in the stream has completed and its memory is visible -- no global
// memory may be read or written before this -- and let the next grid launch while this one runs.
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependent_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Per-device state owned by the library. Created lazily by the first call on a device;
// that first call allocates, so it must not be made inside a stream capture.
struct DeviceState {
    int device = -1;
    int sm_count = 0;
    int l2_bytes = 0;
    int cc_major = 0, cc_minor = 0;
    DeviceErrorRecord* err = nullptr;  // device memory, zeroed
    // CSR workspace (all-zero between calls).
    void* csr_ws = nullptr;
    size_t csr_ws_bytes = 0;
    // Cached device buffers of the host-buffer entry point.
    void* h_rp = nullptr; size_t h_rp_bytes = 0;
    void* h_ci = nullptr; size_t h_ci_bytes = 0;
    void* h_v = nullptr;  size_t h_v_bytes = 0;
    void* h_b = nullptr;  size_t h_b_bytes = 0;
    void* h_c = nullptr;  size_t h_c_bytes = 0;
    // Result flags of the device CSR -> BSR conversion.
    void* conv_flags = nullptr; size_t conv_flags_bytes = 0;
    // Copy-in, compute and copy-out streams and their events for the pipelined host-buffer
    // entry point (created on first use, non-blocking).
    cudaStream_t pipe_in = nullptr, pipe_k = nullptr, pipe_out = nullptr;
    cudaEvent_t pipe_ev[2 * 16 + 2] = {};
    std::mutex mu;
};

// State of the current device (nullptr + status on failure).
int current_device_state(DeviceState** out);
int device_state(int device, DeviceState** out);

// Grow `*buf` (device memory) to at least `bytes`; zero-fill when `zero` is set.
int ensure_device_buffer(void** buf, size_t* cur, size_t bytes, bool zero, cudaStream_t stream);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// FP32 CSR launcher shared by every entry point (csr_kernels.cu). `ksplit_ready`: the first
// (k_phases - 1) * M ints of `ws` already hold the column-phase split positions (plans).
int csr_f32_launch(const spmm_csr_view* A, const float* B, float* C, int32_t N, int32_t algo,
                   const spmm_csr_tuning* tune, void* ws, size_t ws_bytes, cudaStream_t stream, DeviceState* st,
                   bool ksplit_ready = false);
// The argument checks csr_f32_launch makes first (view, pointers, alignment), on their own.
int csr_f32_check_args(const spmm_csr_view* A, const float* B, const float* C, int32_t N);
int csr_f32_workspace_bytes(const spmm_csr_view* A, int32_t N, int32_t algo, const spmm_csr_tuning* tune,
                            int sm_count, size_t* bytes);
size_t csr_f32_counter_bytes(const spmm_csr_view* A, int32_t N, const spmm_csr_tuning* tune, int sm_count);
int csr_f32_chunk(const spmm_csr_view* A, const spmm_csr_tuning* tune, int sm_count);
int csr_f32_ksplit(const spmm_csr_view* A, int phases, int* split, cudaStream_t stream, DeviceState* st);
int csr_f32_phase_launch(const spmm_csr_view* A, const float* B, float* C, int32_t N, int phases, int phase,
                         int* split, cudaStream_t stream, DeviceState* st);

}  // namespace spmm_b200
