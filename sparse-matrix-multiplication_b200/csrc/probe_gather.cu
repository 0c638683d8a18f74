// Measurement helper for bench.py (lib/libspmm_probe.so, not part of the SpMM C ABI): the
// random-row gather ceiling of this GPU, i.e. how fast SMs can pull whole rows of a dense
// FP32 row-major matrix from the memory system when the rows are picked at random.
//
// The FP32 CSR kernels move one full B row (4 * N bytes) per nonzero; with uniformly random
// columns nothing is reused in L1, so the rate at which whole random rows reach the SMs bounds
// them, not HBM. This kernel does only that: same residency as the CSR kernels (4 CTAs x 8
// warps per SM), one warp per row fetch, each lane two 16-byte loads of a 256-float row (or one
// of a 128-float row), eight loads per lane in flight, rows picked by a counter hash over a buffer of `rows` rows
// (choose a footprint inside L2 for the L2 ceiling, or the real B's size). The loaded values
// are summed and one float per thread is stored so that nothing is optimised away.

#include <cuda_runtime.h>

#include <cstdint>

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

// ROWF floats per row: 256 (1 KB, two 16-byte loads per lane) or 128 (512 B, one per lane); U rows
// per warp in flight, so that every lane has eight 16-byte loads outstanding either way.
template <int ROWF, int U>
__global__ void __launch_bounds__(kThreads, 4) gather_probe_kernel(const float* __restrict__ buf, uint32_t rows,
                                                                   long long fetches, uint32_t seed,
                                                                   float* __restrict__ out) {
    constexpr int L = ROWF / 128;  // 16-byte loads per lane per row
    const int lane = threadIdx.x & 31;
    const long long warp = (static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const long long nwarps = (static_cast<long long>(gridDim.x) * kThreads) >> 5;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    long long f = warp * U;
    for (; f + U <= fetches; f += nwarps * U) {
        float4 b[U][L];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint32_t h = mix32(static_cast<uint32_t>(f + u) * 0x9e3779b9u + seed);
            const uint32_t r = static_cast<uint32_t>((static_cast<uint64_t>(h) * rows) >> 32);
            const float4* row = reinterpret_cast<const float4*>(buf + static_cast<size_t>(r) * ROWF);
#pragma unroll
            for (int l = 0; l < L; ++l) b[u][l] = __ldg(row + 32 * l + lane);
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int l = 0; l < L; ++l) {
                s0 += b[u][l].x;
                s1 += b[u][l].y;
                s2 += b[u][l].z;
                s3 += b[u][l].w;
            }
    }
    out[static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x] = s0 + s1 + s2 + s3;
}

}  // namespace

extern "C" {

// Fetch `fetches` random 1 KB rows (256 floats) of `buf` (rows x 256, 16-byte aligned) on
// `stream` (spmm_probe_gather), or rows of 128 or 256 floats (spmm_probe_gather_rows). `out`
// needs grid_ctas * 256 floats, grid_ctas = sm_count * 4 (see spmm_probe_ctas). Returns 0, or a
// cudaError_t value (1 for bad arguments).
int spmm_probe_ctas(int* ctas) {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 1;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 1;
    *ctas = sms * 4;
    return 0;
}

// Rows of `row_floats` floats (128 or 256): `buf` is rows x row_floats, 16-byte aligned.
int spmm_probe_gather_rows(const float* buf, int row_floats, uint32_t rows, long long fetches, uint32_t seed,
                           float* out, void* stream) {
    if (!buf || !out || rows == 0 || fetches < 0 || (reinterpret_cast<uintptr_t>(buf) & 15)) return 1;
    if (row_floats != 128 && row_floats != 256) return 1;
    int ctas = 0;
    if (spmm_probe_ctas(&ctas)) return 1;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (row_floats == 256) gather_probe_kernel<256, 4><<<ctas, kThreads, 0, s>>>(buf, rows, fetches, seed, out);
    else gather_probe_kernel<128, 8><<<ctas, kThreads, 0, s>>>(buf, rows, fetches, seed, out);
    return static_cast<int>(cudaGetLastError());
}

int spmm_probe_gather(const float* buf, uint32_t rows, long long fetches, uint32_t seed, float* out, void* stream) {
    return spmm_probe_gather_rows(buf, 256, rows, fetches, seed, out, stream);
}

}  // extern "C"
