// Error macros and the event timer used by the drivers. Same names and behaviour as the
// reference's src/utils.h: a failing CUDA / cuSPARSE call prints and exits.
#pragma once

#include <cuda_runtime.h>
#include <cusparse.h>

#include <cstdio>
#include <cstdlib>

#define CUDA_CHECK(call)                                                                            \
    do {                                                                                            \
        cudaError_t cuda_check_err_ = (call);                                                       \
        if (cuda_check_err_ != cudaSuccess) {                                                       \
            std::fprintf(stderr, "CUDA error %s at %s:%d: %s\n", #call, __FILE__, __LINE__,        \
                         cudaGetErrorString(cuda_check_err_));                                      \
            std::exit(EXIT_FAILURE);                                                                \
        }                                                                                           \
    } while (0)

#define CUSPARSE_CHECK(call)                                                                        \
    do {                                                                                            \
        cusparseStatus_t cusparse_check_st_ = (call);                                               \
        if (cusparse_check_st_ != CUSPARSE_STATUS_SUCCESS) {                                        \
            std::fprintf(stderr, "cuSPARSE error %s at %s:%d: %s\n", #call, __FILE__, __LINE__,     \
                         cusparseGetErrorString(cusparse_check_st_));                               \
            std::exit(EXIT_FAILURE);                                                                \
        }                                                                                           \
    } while (0)

constexpr int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Elapsed time between two events recorded on the legacy default stream.
class GpuTimer {
public:
    GpuTimer() {
        cudaEventCreate(&begin_);
        cudaEventCreate(&end_);
    }
    ~GpuTimer() {
        cudaEventDestroy(begin_);
        cudaEventDestroy(end_);
    }
    GpuTimer(const GpuTimer&) = delete;
    GpuTimer& operator=(const GpuTimer&) = delete;
    void start() { cudaEventRecord(begin_); }
    void stop() {
        cudaEventRecord(end_);
        cudaEventSynchronize(end_);
    }
    float elapsed_ms() {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, begin_, end_);
        return ms;
    }

private:
    cudaEvent_t begin_{};
    cudaEvent_t end_{};
};
