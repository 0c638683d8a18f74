// Per-device state, status strings, device error record, FP32 -> FP16/BF16 conversion.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace spmm_b200 {

namespace {
std::mutex g_states_mu;
std::vector<std::unique_ptr<DeviceState>> g_states;

bool verbose() {
    static const bool v = [] {
        const char* e = std::getenv("SPMM_B200_VERBOSE");
        return e && e[0] && e[0] != '0';
    }();
    return v;
}
}  // namespace

void note_cuda_error(cudaError_t e, const char* what, const char* file, int line) {
    if (verbose()) std::fprintf(stderr, "spmm_b200: %s failed at %s:%d: %s\n", what, file, line, cudaGetErrorString(e));
}

int device_state(int device, DeviceState** out) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return SPMM_ERR_UNSUPPORTED;
    }
    if (device < 0 || device >= n) return SPMM_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> lock(g_states_mu);
    if (g_states.size() < static_cast<size_t>(n)) g_states.resize(n);
    if (!g_states[device]) {
        auto st = std::make_unique<DeviceState>();
        st->device = device;
        int prev = 0;
        SPMM_CUDA_TRY(cudaGetDevice(&prev));
        SPMM_CUDA_TRY(cudaSetDevice(device));
        SPMM_CUDA_TRY(cudaDeviceGetAttribute(&st->sm_count, cudaDevAttrMultiProcessorCount, device));
        SPMM_CUDA_TRY(cudaDeviceGetAttribute(&st->l2_bytes, cudaDevAttrL2CacheSize, device));
        SPMM_CUDA_TRY(cudaDeviceGetAttribute(&st->cc_major, cudaDevAttrComputeCapabilityMajor, device));
        SPMM_CUDA_TRY(cudaDeviceGetAttribute(&st->cc_minor, cudaDevAttrComputeCapabilityMinor, device));
        SPMM_CUDA_TRY(cudaMalloc(&st->err, sizeof(DeviceErrorRecord)));
        SPMM_CUDA_TRY(cudaMemset(st->err, 0, sizeof(DeviceErrorRecord)));
        SPMM_CUDA_TRY(cudaDeviceSynchronize());
        SPMM_CUDA_TRY(cudaSetDevice(prev));
        g_states[device] = std::move(st);
    }
    *out = g_states[device].get();
    return SPMM_OK;
}

int current_device_state(DeviceState** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return SPMM_ERR_UNSUPPORTED;
    }
    return device_state(dev, out);
}

int ensure_device_buffer(void** buf, size_t* cur, size_t bytes, bool zero, cudaStream_t stream) {
    if (bytes <= *cur) return SPMM_OK;
    if (*buf) {
        // The old buffer may still be in use by queued work on any stream.
        SPMM_CUDA_TRY(cudaDeviceSynchronize());
        SPMM_CUDA_TRY(cudaFree(*buf));
        *buf = nullptr;
        *cur = 0;
    }
    const size_t grown = bytes + bytes / 4;
    if (cudaMalloc(buf, grown) != cudaSuccess) {
        cudaGetLastError();
        *buf = nullptr;
        return SPMM_ERR_NO_MEMORY;
    }
    *cur = grown;
    if (zero) {
        SPMM_CUDA_TRY(cudaMemsetAsync(*buf, 0, grown, stream));
    }
    return SPMM_OK;
}

namespace {

// Eight elements per thread: two 16-byte loads in, one 16-byte store out, when aligned.
template <bool BF16>
__global__ void convert_f32_kernel(const float* __restrict__ src, uint16_t* __restrict__ dst, long long n) {
    const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long n8 = n / 8;
    for (long long i = tid; i < n8; i += stride) {
        const float4 a = __ldcs(reinterpret_cast<const float4*>(src) + 2 * i);
        const float4 b = __ldcs(reinterpret_cast<const float4*>(src) + 2 * i + 1);
        uint4 o;
        if constexpr (BF16) {
            __nv_bfloat162 h0 = __floats2bfloat162_rn(a.x, a.y), h1 = __floats2bfloat162_rn(a.z, a.w);
            __nv_bfloat162 h2 = __floats2bfloat162_rn(b.x, b.y), h3 = __floats2bfloat162_rn(b.z, b.w);
            o.x = *reinterpret_cast<unsigned*>(&h0);
            o.y = *reinterpret_cast<unsigned*>(&h1);
            o.z = *reinterpret_cast<unsigned*>(&h2);
            o.w = *reinterpret_cast<unsigned*>(&h3);
        } else {
            __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
            o.x = *reinterpret_cast<unsigned*>(&h0);
            o.y = *reinterpret_cast<unsigned*>(&h1);
            o.z = *reinterpret_cast<unsigned*>(&h2);
            o.w = *reinterpret_cast<unsigned*>(&h3);
        }
        __stcs(reinterpret_cast<uint4*>(dst) + i, o);
    }
    for (long long i = n8 * 8 + tid; i < n; i += stride) {
        if constexpr (BF16) {
            const __nv_bfloat16 h = __float2bfloat16_rn(src[i]);
            dst[i] = *reinterpret_cast<const uint16_t*>(&h);
        } else {
            const __half h = __float2half_rn(src[i]);
            dst[i] = *reinterpret_cast<const uint16_t*>(&h);
        }
    }
}

template <bool BF16>
__global__ void convert_f32_scalar_kernel(const float* __restrict__ src, uint16_t* __restrict__ dst, long long n) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        if constexpr (BF16) {
            const __nv_bfloat16 h = __float2bfloat16_rn(src[i]);
            dst[i] = *reinterpret_cast<const uint16_t*>(&h);
        } else {
            const __half h = __float2half_rn(src[i]);
            dst[i] = *reinterpret_cast<const uint16_t*>(&h);
        }
    }
}

}  // namespace
}  // namespace spmm_b200

using namespace spmm_b200;

extern "C" {

const char* spmm_status_string(int s) {
    switch (s) {
        case SPMM_OK: return "ok";
        case SPMM_ERR_INVALID_ARG: return "invalid argument";
        case SPMM_ERR_MISALIGNED: return "misaligned operand or unsupported N for this path";
        case SPMM_ERR_CUDA: return "CUDA runtime error";
        case SPMM_ERR_NCCL: return "NCCL error";
        case SPMM_ERR_TIMEOUT: return "device wait timed out";
        case SPMM_ERR_UNSUPPORTED: return "unsupported (no suitable device or feature)";
        case SPMM_ERR_NO_MEMORY: return "out of memory";
        case SPMM_ERR_BAD_INDEX: return "index out of range seen on the device";
        case SPMM_ERR_IO: return "I/O error";
        case SPMM_ERR_TOO_LARGE: return "request exceeds a fixed capacity";
        default: return "unknown status";
    }
}

int spmm_version(void) { return 100; }

int spmm_convert_f32(const float* src, uint16_t* dst, int64_t n, int32_t dtype, void* stream) {
    if (n < 0 || (n > 0 && (!src || !dst)) || (dtype != SPMM_DTYPE_F16 && dtype != SPMM_DTYPE_BF16))
        return SPMM_ERR_INVALID_ARG;
    if (n == 0) return SPMM_OK;
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    const cudaStream_t s = as_stream(stream);
    const bool vec = (reinterpret_cast<uintptr_t>(src) % 16 == 0) && (reinterpret_cast<uintptr_t>(dst) % 16 == 0);
    const long long work = vec ? (n / 8 + 1) : n;
    const long long blocks = std::min<long long>((work + 255) / 256, static_cast<long long>(st->sm_count) * 16);
    const int grid = static_cast<int>(std::max<long long>(blocks, 1));
    if (vec) {
        if (dtype == SPMM_DTYPE_BF16) convert_f32_kernel<true><<<grid, 256, 0, s>>>(src, dst, n);
        else convert_f32_kernel<false><<<grid, 256, 0, s>>>(src, dst, n);
    } else {
        if (dtype == SPMM_DTYPE_BF16) convert_f32_scalar_kernel<true><<<grid, 256, 0, s>>>(src, dst, n);
        else convert_f32_scalar_kernel<false><<<grid, 256, 0, s>>>(src, dst, n);
    }
    SPMM_CUDA_TRY(cudaGetLastError());
    return SPMM_OK;
}

int spmm_device_error(int32_t device, int32_t* code, int64_t* detail, int32_t clear) {
    DeviceState* st = nullptr;
    SPMM_TRY(device_state(device, &st));
    int prev = 0;
    SPMM_CUDA_TRY(cudaGetDevice(&prev));
    SPMM_CUDA_TRY(cudaSetDevice(device));
    DeviceErrorRecord rec{};
    int rc = SPMM_OK;
    if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&rec, st->err, sizeof(rec), cudaMemcpyDeviceToHost) != cudaSuccess) {
        rc = SPMM_ERR_CUDA;
    } else if (clear) {
        if (cudaMemset(st->err, 0, sizeof(rec)) != cudaSuccess) rc = SPMM_ERR_CUDA;
        // A kernel that hit a bad index may have left merge-path counters behind.
        if (rc == SPMM_OK && rec.code != 0 && st->csr_ws && st->csr_ws_bytes) {
            if (cudaMemset(st->csr_ws, 0, st->csr_ws_bytes) != cudaSuccess) rc = SPMM_ERR_CUDA;
        }
        if (rc == SPMM_OK && cudaDeviceSynchronize() != cudaSuccess) rc = SPMM_ERR_CUDA;
    }
    cudaSetDevice(prev);
    if (code) *code = rec.code;
    if (detail) *detail = rec.detail;
    return rc;
}

}  // extern "C"
