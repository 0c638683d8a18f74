// C++ API of the B200 SpMM engine: BSR with 16x16 blocks. Drop-in for the reference's
// src/bsr.h: same structs, constant and functions.
#pragma once

#include <cuda_fp16.h>

#include <vector>

#include "csr.h"

namespace spmm {

// Block edge of the block-sparse format (one tensor-core K step for 16-bit inputs).
constexpr int BSR_BLOCK = 16;

// Host BSR: every non-empty 16x16 block stored dense, row-major, zero padded.
struct BSR_host {
    int num_rows = 0;    // M
    int num_cols = 0;    // K
    int block_rows = 0;  // ceil(M / 16)
    int block_cols = 0;  // ceil(K / 16)
    int num_blocks = 0;  // non-empty blocks
    int nnz = 0;         // nonzeros of the source CSR
    std::vector<int> row_ptr;   // block_rows + 1
    std::vector<int> col_idx;   // num_blocks, sorted per block-row
    std::vector<half> values;   // num_blocks * 256
};

// Device BSR (raw device pointers).
struct BSR {
    int num_rows = 0;
    int num_cols = 0;
    int block_rows = 0;
    int block_cols = 0;
    int num_blocks = 0;
    int nnz = 0;
    int* row_ptr = nullptr;
    int* col_idx = nullptr;
    half* values = nullptr;
};

struct BSR_stats {
    int num_blocks;         // non-empty blocks
    long stored_elements;   // num_blocks * 256
    int original_nnz;       // CSR nonzeros
    double fill_in_ratio;   // stored_elements / original_nnz
    double block_density;   // num_blocks / (block_rows * block_cols)
};

// CSR (host) -> BSR_host, FP32 values rounded to FP16 (nearest even).
BSR_host bsr_from_csr_host(const CSR& h_csr);
BSR bsr_to_device(const BSR_host& h);
void bsr_free_device(BSR& d);
BSR_stats bsr_compute_stats(const BSR_host& h);

}  // namespace spmm
