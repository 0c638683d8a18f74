// C++ API of the B200 SpMM engine: multi-GPU row split and the managed-memory path. Drop-in
// for the reference's src/spmm_multigpu.h.
//
// C = A * B splits by rows of A with no cross-device reduction: each device gets an
// nnz-balanced row range of A and a full copy of B (sent once to device 0, then broadcast
// over NVLink with NCCL) and writes its rows of C.
#pragma once

#include <vector>

#include "csr.h"

namespace spmm {

int gpu_count();

struct MultiGpuResult {
    float time_ms = 0.f;   // max over devices of the median kernel time
    int num_gpus = 0;
    std::vector<int> rows; // rows per device
    std::vector<int> nnz;  // nonzeros per device
};

// num_gpus is clamped to [1, visible devices]. Uploads and the broadcast of B are outside
// the timed loop.
MultiGpuResult spmm_multigpu(const CSR& h_A, const float* h_B, float* h_C, int N, int num_gpus, int warmup, int iters);

// A, B, C in cudaMallocManaged memory prefetched to the current device; median kernel ms.
float spmm_unified(const CSR& h_A, const float* h_B, float* h_C, int N, int warmup, int iters);

}  // namespace spmm
