// C++ launcher spmm_memopt: C(M x N) = A(M x K, CSR, device) * B(K x N, row-major, device),
// FP32, on the legacy default stream, asynchronous; allocates nothing per call beyond the
// library's per-device workspace. Drop-in for the reference's src/kernels/spmm_memopt.h.
// On B200 it runs the engine's sm_100a CSR kernel with SPMM_CSR_ROWWARP (one warp per row).
#pragma once

#include "../csr.h"

namespace spmm {

void spmm_memopt(const CSR& d_A, const float* d_B, float* d_C, int N);

}  // namespace spmm
