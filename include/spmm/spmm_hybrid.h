// C++ API of the B200 SpMM engine: automatic CUDA-core / tensor-core dispatch. Drop-in for
// the reference's src/spmm_hybrid.h.
//
// The BSR fill-in ratio (stored 16x16 block elements / nonzeros) decides: near 1 the blocks
// are dense and the tcgen05 BSR kernel wins; large fill-in means the blocks are mostly
// padding and the CSR kernel wins.
#pragma once

#include "csr.h"

namespace spmm {

enum class Backend {
    CSR_TILED,   // CSR on the CUDA cores
    TENSOR_WMMA  // BSR-16 on the tensor cores (tcgen05 on B200)
};

struct HybridPlan {
    Backend backend = Backend::CSR_TILED;
    double fill_in_ratio = 0.0;
    double block_density = 0.0;
    float threshold = 0.0f;
    bool n_aligned = false;  // N % 16 == 0
    const char* reason = "";
};

// Tensor cores iff N % 16 == 0, N > 0 and fill-in <= fill_in_threshold. The default is the
// crossover measured on B200 (the reference's T4 default was 2.0).
HybridPlan hybrid_choose(const CSR& h_A, int N, float fill_in_threshold = 6.0f);

// "csr" or "wmma".
const char* backend_name(Backend b);

// Runs the chosen back end on host A/B/C: warmup + iters launches, returns the median kernel
// time in ms and leaves C (M x N row-major) in h_C.
float spmm_hybrid_run(const HybridPlan& plan, const CSR& h_A, const float* h_B, float* h_C, int N, int warmup,
                      int iters);

}  // namespace spmm
