// TEST INFRASTRUCTURE ONLY -- builds oracle/_ref/libref.so from the reference's own
// sources where they lie (nothing is copied into this repository). The reference keeps
// nnz_balanced_bounds, generate_dense_row_major and compare in anonymous namespaces, so
// this file textually includes those translation units to reach them; `main` of the
// harness is renamed out of the way. Everything is exported as plain C for ctypes.
//
// Used by tests/ to pin the oracle restatement against the reference itself, and on a GPU
// box to run the reference's recompiled kernels as a same-box comparison. Build:
//   make -C oracle ref            (needs the reference checkout; see oracle/Makefile)

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#define main spmm_reference_harness_main
#include "bench/harness.cu"
#undef main
#include "spmm_multigpu.cu"

#include "kernels/spmm_baseline.h"
#include "kernels/spmm_memopt.h"
#include "kernels/spmm_memopt_v2.h"
#include "kernels/spmm_tiled.h"
#include "kernels/spmm_tiled_v2.h"
#include "kernels/spmm_tiled_v3.h"
#include "kernels/spmm_tiled_v4.h"
#include "kernels/spmm_wmma.h"

namespace {
template <typename T>
T* dup(const T* src, size_t n) {
    T* p = static_cast<T*>(std::malloc(sizeof(T) * (n > 0 ? n : 1)));
    if (n) std::memcpy(p, src, sizeof(T) * n);
    return p;
}
}  // namespace

extern "C" {

void ref_free(void* p) { std::free(p); }

int ref_gen_uniform_csr(int rows, int cols, float density, int seed, int** rp, int** ci, float** v,
                        int* nnz) {
    spmm::CSR m = spmm::generate_uniform_random_csr(rows, cols, density, seed);
    *rp = dup(m.row_ptr, static_cast<size_t>(rows) + 1);
    *ci = dup(m.col_idx, static_cast<size_t>(m.nnz));
    *v = dup(m.values, static_cast<size_t>(m.nnz));
    *nnz = m.nnz;
    spmm::csr_free_host(m);
    return 0;
}

void ref_gen_dense(int rows, int cols, int seed, float* out) {
    std::vector<float> v = generate_dense_row_major(rows, cols, seed);
    std::memcpy(out, v.data(), sizeof(float) * v.size());
}

int ref_csr_from_coo(int rows, int cols, int n, const int* r, const int* c, const float* v,
                     int** rp, int** ci, float** vo) {
    std::vector<int> rv(r, r + n), cv(c, c + n);
    std::vector<float> vv(v, v + n);
    spmm::CSR m = spmm::csr_from_coo_host(rows, cols, rv, cv, vv);
    *rp = dup(m.row_ptr, static_cast<size_t>(rows) + 1);
    *ci = dup(m.col_idx, static_cast<size_t>(m.nnz));
    *vo = dup(m.values, static_cast<size_t>(m.nnz));
    spmm::csr_free_host(m);
    return 0;
}

int ref_bsr_from_csr(int M, int K, int nnz, const int* rp, const int* ci, const float* v, int* block_rows,
                     int* block_cols, int* num_blocks, int** brp, int** bci, uint16_t** bval,
                     long* stored, double* fill_in, double* density) {
    spmm::CSR m;
    m.num_rows = M;
    m.num_cols = K;
    m.nnz = nnz;
    m.row_ptr = const_cast<int*>(rp);
    m.col_idx = const_cast<int*>(ci);
    m.values = const_cast<float*>(v);
    spmm::BSR_host h = spmm::bsr_from_csr_host(m);
    spmm::BSR_stats s = spmm::bsr_compute_stats(h);
    *block_rows = h.block_rows;
    *block_cols = h.block_cols;
    *num_blocks = h.num_blocks;
    *brp = dup(h.row_ptr.data(), h.row_ptr.size());
    *bci = dup(h.col_idx.data(), h.col_idx.size());
    *bval = dup(reinterpret_cast<const uint16_t*>(h.values.data()), h.values.size());
    *stored = s.stored_elements;
    *fill_in = s.fill_in_ratio;
    *density = s.block_density;
    return 0;
}

void ref_nnz_balanced_bounds(int rows, int nnz, const int* rp, int G, int* out) {
    spmm::CSR m;
    m.num_rows = rows;
    m.nnz = nnz;
    m.row_ptr = const_cast<int*>(rp);
    std::vector<int> b = spmm::nnz_balanced_bounds(m, G);
    for (int g = 0; g <= G; ++g) out[g] = b[g];
}

void ref_compare(const float* ours, const float* ref, long n, float* max_abs, float* max_rel, float* rel_l2) {
    std::vector<float> a(ours, ours + n), b(ref, ref + n);
    ErrorStats s = compare(a, b);
    *max_abs = s.max_abs;
    *max_rel = s.max_rel;
    *rel_l2 = s.rel_l2;
}

// The reference's own kernels recompiled for this GPU, driven on device buffers.
// kernel: 0 baseline, 1 memopt, 2 memopt_v2, 3 tiled, 4 tiled_v2, 5 tiled_v3, 6 tiled_v4.
int ref_spmm_csr_device(int kernel, int M, int K, int nnz, int* d_rp, int* d_ci, float* d_v,
                        const float* d_B, float* d_C, int N) {
    spmm::CSR a;
    a.num_rows = M;
    a.num_cols = K;
    a.nnz = nnz;
    a.row_ptr = d_rp;
    a.col_idx = d_ci;
    a.values = d_v;
    switch (kernel) {
        case 0: spmm::spmm_baseline(a, d_B, d_C, N); break;
        case 1: spmm::spmm_memopt(a, d_B, d_C, N); break;
        case 2: spmm::spmm_memopt_v2(a, d_B, d_C, N); break;
        case 3: spmm::spmm_tiled(a, d_B, d_C, N); break;
        case 4: if (N % 128) return -1; spmm::spmm_tiled_v2(a, d_B, d_C, N); break;
        case 5: spmm::spmm_tiled_v3(a, d_B, d_C, N); break;
        case 6: spmm::spmm_tiled_v4(a, d_B, d_C, N); break;
        default: return -1;
    }
    return 0;
}

int ref_spmm_wmma_device(int M, int K, int block_rows, int block_cols, int num_blocks, int nnz, int* d_rp,
                         int* d_ci, void* d_vals, const void* d_B16, float* d_C, int N) {
    spmm::BSR b;
    b.num_rows = M;
    b.num_cols = K;
    b.block_rows = block_rows;
    b.block_cols = block_cols;
    b.num_blocks = num_blocks;
    b.nnz = nnz;
    b.row_ptr = d_rp;
    b.col_idx = d_ci;
    b.values = static_cast<half*>(d_vals);
    spmm::spmm_wmma(b, static_cast<const half*>(d_B16), d_C, N);
    return 0;
}

}  // extern "C"
