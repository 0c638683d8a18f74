// C++ API of the B200 SpMM engine: CSR matrices. Drop-in for the reference's src/csr.h
// (Adityaa-Saha17/Sparse-Matrix-Multiplication): same namespace, struct layout, function
// names and signatures, implemented in libspmm.so on top of the C ABI in spmm_c.h.
#pragma once

#include <string>
#include <vector>

namespace spmm {

// 0-based CSR with int32 indices and FP32 values; columns sorted inside each row.
// Host or device memory, depending on who made it (reference: src/csr.h:7-14).
struct CSR {
    int num_rows = 0;
    int num_cols = 0;
    int nnz = 0;
    int* row_ptr = nullptr;  // num_rows + 1
    int* col_idx = nullptr;  // nnz
    float* values = nullptr; // nnz
};

// malloc'd host arrays; exits with a message when the allocation fails.
CSR csr_alloc_host(int rows, int cols, int nnz);
void csr_free_host(CSR& m);

// Triplets -> CSR, ordered by (row, col). Duplicate coordinates are kept, as the
// reference does. Throws std::runtime_error on a size mismatch.
CSR csr_from_coo_host(int rows, int cols, const std::vector<int>& row_indices, const std::vector<int>& col_indices,
                      const std::vector<float>& values);

// Bernoulli(density) matrix from mt19937(seed) with U[-1,1) values; the same matrix the
// reference generator produces. Throws on a density outside [0, 1].
CSR generate_uniform_random_csr(int rows, int cols, float density, int seed);

// Rows [row_begin, row_end) as a new host CSR with row_ptr rebased to 0.
CSR csr_row_slice_host(const CSR& m, int row_begin, int row_end);

// Binary file: int32 rows, cols, nnz; row_ptr; col_idx; float values.
CSR csr_read_binary_host(const std::string& path);
void csr_write_binary_host(const CSR& m, const std::string& path);

// Device copies (cudaMalloc + synchronous copy) and their release.
CSR csr_to_device(const CSR& host);
void csr_free_device(CSR& device);

}  // namespace spmm
