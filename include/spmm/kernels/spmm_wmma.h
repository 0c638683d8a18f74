// C++ launchers of the tensor-core path. Drop-in for the reference's src/kernels/spmm_wmma.h.
// On B200 spmm_wmma runs the engine's tcgen05 BSR-16 kernel (TMEM accumulators, TMA
// operand loads); N must be a multiple of 8 with 16-byte aligned operands for that path,
// other shapes run a CUDA-core BSR kernel.
#pragma once

#include <cuda_fp16.h>

#include "../bsr.h"

namespace spmm {

// d_dst[i] = FP16(d_src[i]), round to nearest even; device pointers, default stream.
void float_to_half(const float* d_src, half* d_dst, int n_elements);

// d_C (M x N, FP32) = d_bsr (FP16 blocks) * d_B_fp16 (K x N, FP16), FP32 accumulation.
void spmm_wmma(const BSR& d_bsr, const half* d_B_fp16, float* d_C, int N);

}  // namespace spmm
