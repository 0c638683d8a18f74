// spmm_csr_f32_noalloc: the CSR SpMM for callers that must not allocate device memory.
//
// Some callers cannot let a library call cudaMalloc: hosts that give every byte of device
// memory to their own allocator or to a fixed budget (a caching allocator that must see all
// allocations, an embedding service sized to the card), and latency-critical loops where
// cudaMalloc's implicit device synchronisation is not acceptable. spmm_csr_f32 allocates its
// per-device workspace (and an error record) on first use; this entry point instead uses a
// fixed scratch array compiled into the library, so it allocates nothing at any call.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes (16 MiB). Every GPU
// that loads this library holds it until the process exits. Host code cannot use the
// array's name as a device address, so the first call on each device (with that device
// current) looks the address up with cudaGetSymbolAddress and caches it; make that first
// call before any stream capture. All calls on a device share the array: two calls whose
// kernels overlap on the GPU (different streams, no ordering between them) race and give
// wrong results. The arrival counters that must start at zero are cleared (cudaMemsetAsync
// on the caller's stream) before every launch; the rest is overwritten before it is read.
// The cached address belongs to the device's primary context: after cudaDeviceReset it no
// longer names mapped memory, so this entry point must not be called again in a process that
// has reset the device.

#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace spmm_b200 {


namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on `device` (which must be current).
int scratch_address(int device, void** out) {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return SPMM_ERR_CUDA;
        }
        g_scratch_addr[device] = p;
    }
    *out = g_scratch_addr[device];
    return SPMM_OK;
}

}  // namespace
}  // namespace spmm_b200

using namespace spmm_b200;

extern "C" int spmm_csr_f32_noalloc(const spmm_csr_view* A, const float* B, float* C, int32_t N, int32_t algo,
                                    void* stream) {
    // The same argument checks as spmm_csr_f32, before anything is queued on the stream.
    SPMM_TRY(csr_f32_check_args(A, B, C, N));
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        cudaGetLastError();
        return SPMM_ERR_UNSUPPORTED;
    }
    if (device < 0 || device >= kMaxDevices) return SPMM_ERR_UNSUPPORTED;
    // A stack-local device description: SM count only, no error record (an out-of-range
    // index is replaced by a safe one and is not reported on this path; validate inputs
    // with spmm_csr_validate_host).
    DeviceState local;
    local.device = device;
    SPMM_CUDA_TRY(cudaDeviceGetAttribute(&local.sm_count, cudaDevAttrMultiProcessorCount, device));
    size_t need = 0;
    SPMM_TRY(csr_f32_workspace_bytes(A, N, algo, nullptr, local.sm_count, &need));
    if (need > kNoAllocScratchBytes) return SPMM_ERR_TOO_LARGE;
    void* scratch = nullptr;
    SPMM_TRY(scratch_address(device, &scratch));
    if (need > 0) {
        // The merge-path workspace starts with the arrival counters (one per chunk and
        // column slab); only those must be zero when the kernel starts.
        const size_t counters = csr_f32_counter_bytes(A, N, nullptr, local.sm_count);
        SPMM_CUDA_TRY(cudaMemsetAsync(scratch, 0, counters < need ? counters : need, as_stream(stream)));
    }
    return csr_f32_launch(A, B, C, N, algo, nullptr, scratch, need, as_stream(stream), &local);
}
