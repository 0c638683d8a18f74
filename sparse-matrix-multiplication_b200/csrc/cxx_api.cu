// libspmm.so: the reference-compatible C++ API (include/spmm/*.h) implemented on the C ABI
// of libspmm_b200.so (include/spmm_c.h). Host C++ only -- every computation goes through
// the C entry points. Errors follow the reference's conventions: CUDA failures print and
// exit, host validation throws std::runtime_error, spmm_tiled_v2 aborts on N % 128 != 0.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "spmm/bsr.h"
#include "spmm/csr.h"
#include "spmm/kernels/spmm_baseline.h"
#include "spmm/kernels/spmm_memopt.h"
#include "spmm/kernels/spmm_memopt_v2.h"
#include "spmm/kernels/spmm_tiled.h"
#include "spmm/kernels/spmm_tiled_v2.h"
#include "spmm/kernels/spmm_tiled_v3.h"
#include "spmm/kernels/spmm_tiled_v4.h"
#include "spmm/kernels/spmm_wmma.h"
#include "spmm/spmm_hybrid.h"
#include "spmm/spmm_multigpu.h"
#include "spmm/utils.h"
#include "spmm_c.h"

namespace spmm {
namespace {

spmm_csr_view view_of(const CSR& m) {
    return spmm_csr_view{m.num_rows, m.num_cols, m.nnz, m.row_ptr, m.col_idx, m.values};
}

CSR adopt(const spmm_csr_host& h) {
    CSR m;
    m.num_rows = h.rows;
    m.num_cols = h.cols;
    m.nnz = h.nnz;
    m.row_ptr = h.row_ptr;
    m.col_idx = h.col_idx;
    m.values = h.values;
    return m;
}

// A failure of a device entry point is fatal, like CUDA_CHECK in the reference.
void device_check(int status, const char* what) {
    if (status == SPMM_OK) return;
    std::fprintf(stderr, "spmm error in %s: %s\n", what, spmm_status_string(status));
    std::exit(EXIT_FAILURE);
}

void csr_launch(const CSR& d_A, const float* d_B, float* d_C, int N, int algo, const char* name) {
    const spmm_csr_view v = view_of(d_A);
    device_check(spmm_csr_f32(&v, d_B, d_C, N, algo, nullptr), name);
}

}  // namespace

// ------------------------------------------------------------------ csr.h

CSR csr_alloc_host(int rows, int cols, int nnz) {
    spmm_csr_host h{};
    if (spmm_csr_host_alloc(rows, cols, nnz, &h) != SPMM_OK) {
        std::fprintf(stderr, "csr_alloc_host: out of memory\n");
        std::exit(EXIT_FAILURE);
    }
    return adopt(h);
}

void csr_free_host(CSR& m) {
    std::free(m.row_ptr);
    std::free(m.col_idx);
    std::free(m.values);
    m.row_ptr = nullptr;
    m.col_idx = nullptr;
    m.values = nullptr;
    m.nnz = m.num_rows = m.num_cols = 0;
}

CSR csr_from_coo_host(int rows, int cols, const std::vector<int>& row_indices, const std::vector<int>& col_indices,
                      const std::vector<float>& values) {
    const int n = static_cast<int>(values.size());
    if (n != static_cast<int>(row_indices.size()) || n != static_cast<int>(col_indices.size()))
        throw std::runtime_error("csr_from_coo_host: triplet size mismatch");
    spmm_csr_host h{};
    const int rc = spmm_csr_from_coo_host(rows, cols, n, row_indices.data(), col_indices.data(), values.data(), &h);
    if (rc == SPMM_ERR_NO_MEMORY) {
        std::fprintf(stderr, "csr_alloc_host: out of memory\n");
        std::exit(EXIT_FAILURE);
    }
    if (rc != SPMM_OK) throw std::runtime_error("csr_from_coo_host: invalid triplets");
    return adopt(h);
}

CSR generate_uniform_random_csr(int rows, int cols, float density, int seed) {
    if (density < 0.f || density > 1.f) throw std::runtime_error("generate_uniform_random_csr: invalid density");
    spmm_csr_host h{};
    const int rc = spmm_generate_uniform_csr(rows, cols, density, seed, &h);
    if (rc == SPMM_ERR_NO_MEMORY) {
        std::fprintf(stderr, "csr_alloc_host: out of memory\n");
        std::exit(EXIT_FAILURE);
    }
    if (rc != SPMM_OK) throw std::runtime_error("generate_uniform_random_csr: invalid density");
    return adopt(h);
}

CSR csr_row_slice_host(const CSR& m, int row_begin, int row_end) {
    if (row_begin < 0 || row_end > m.num_rows || row_begin > row_end)
        throw std::runtime_error("csr_row_slice_host: invalid row range");
    const spmm_csr_view v = view_of(m);
    spmm_csr_host h{};
    if (spmm_csr_row_slice_host(&v, row_begin, row_end, &h) != SPMM_OK)
        throw std::runtime_error("csr_row_slice_host: invalid row range");
    return adopt(h);
}

CSR csr_read_binary_host(const std::string& path) {
    // Distinguish the reference's three failure messages.
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) throw std::runtime_error("csr_read_binary_host: cannot open " + path);
    int hdr[3];
    const bool have_header = std::fread(hdr, sizeof(int), 3, f) == 3;
    std::fclose(f);
    if (!have_header) throw std::runtime_error("csr_read_binary_host: short read on header");
    spmm_csr_host h{};
    const int rc = spmm_csr_read_binary(path.c_str(), &h);
    if (rc == SPMM_ERR_NO_MEMORY) {
        std::fprintf(stderr, "csr_alloc_host: out of memory\n");
        std::exit(EXIT_FAILURE);
    }
    if (rc != SPMM_OK) throw std::runtime_error("csr_read_binary_host: short read on body");
    return adopt(h);
}

void csr_write_binary_host(const CSR& m, const std::string& path) {
    const spmm_csr_view v = view_of(m);
    if (spmm_csr_write_binary(&v, path.c_str()) != SPMM_OK)
        throw std::runtime_error("csr_write_binary_host: cannot open " + path);
}

CSR csr_to_device(const CSR& host) {
    CSR d;
    d.num_rows = host.num_rows;
    d.num_cols = host.num_cols;
    d.nnz = host.nnz;
    CUDA_CHECK(cudaMalloc(&d.row_ptr, sizeof(int) * (host.num_rows + 1)));
    CUDA_CHECK(cudaMalloc(&d.col_idx, sizeof(int) * host.nnz));
    CUDA_CHECK(cudaMalloc(&d.values, sizeof(float) * host.nnz));
    CUDA_CHECK(cudaMemcpy(d.row_ptr, host.row_ptr, sizeof(int) * (host.num_rows + 1), cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(d.col_idx, host.col_idx, sizeof(int) * host.nnz, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(d.values, host.values, sizeof(float) * host.nnz, cudaMemcpyHostToDevice));
    return d;
}

void csr_free_device(CSR& d) {
    if (d.row_ptr) CUDA_CHECK(cudaFree(d.row_ptr));
    if (d.col_idx) CUDA_CHECK(cudaFree(d.col_idx));
    if (d.values) CUDA_CHECK(cudaFree(d.values));
    d.row_ptr = nullptr;
    d.col_idx = nullptr;
    d.values = nullptr;
    d.nnz = d.num_rows = d.num_cols = 0;
}

// ------------------------------------------------------------------ bsr.h

BSR_host bsr_from_csr_host(const CSR& h_csr) {
    const spmm_csr_view v = view_of(h_csr);
    spmm_bsr_host b{};
    const int rc = spmm_csr_to_bsr16_host(&v, SPMM_DTYPE_F16, &b);
    if (rc != SPMM_OK) throw std::runtime_error(std::string("bsr_from_csr_host: ") + spmm_status_string(rc));
    BSR_host h;
    h.num_rows = b.rows;
    h.num_cols = b.cols;
    h.block_rows = b.block_rows;
    h.block_cols = b.block_cols;
    h.num_blocks = b.num_blocks;
    h.nnz = b.nnz;
    h.row_ptr.assign(b.row_ptr, b.row_ptr + b.block_rows + 1);
    h.col_idx.assign(b.col_idx, b.col_idx + b.num_blocks);
    h.values.resize(static_cast<size_t>(b.num_blocks) * BSR_BLOCK * BSR_BLOCK);
    if (!h.values.empty()) std::memcpy(static_cast<void*>(h.values.data()), b.values, h.values.size() * sizeof(half));
    spmm_bsr_host_free(&b);
    return h;
}

BSR bsr_to_device(const BSR_host& h) {
    BSR d;
    d.num_rows = h.num_rows;
    d.num_cols = h.num_cols;
    d.block_rows = h.block_rows;
    d.block_cols = h.block_cols;
    d.num_blocks = h.num_blocks;
    d.nnz = h.nnz;
    const size_t rp = (h.block_rows + 1) * sizeof(int);
    const size_t ci = h.num_blocks * sizeof(int);
    const size_t vb = static_cast<size_t>(h.num_blocks) * BSR_BLOCK * BSR_BLOCK * sizeof(half);
    CUDA_CHECK(cudaMalloc(&d.row_ptr, rp));
    CUDA_CHECK(cudaMalloc(&d.col_idx, ci));
    CUDA_CHECK(cudaMalloc(&d.values, vb));
    CUDA_CHECK(cudaMemcpy(d.row_ptr, h.row_ptr.data(), rp, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(d.col_idx, h.col_idx.data(), ci, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(d.values, h.values.data(), vb, cudaMemcpyHostToDevice));
    return d;
}

void bsr_free_device(BSR& d) {
    if (d.row_ptr) CUDA_CHECK(cudaFree(d.row_ptr));
    if (d.col_idx) CUDA_CHECK(cudaFree(d.col_idx));
    if (d.values) CUDA_CHECK(cudaFree(d.values));
    d.row_ptr = nullptr;
    d.col_idx = nullptr;
    d.values = nullptr;
}

BSR_stats bsr_compute_stats(const BSR_host& h) {
    const spmm_bsr_view v{h.num_rows, h.num_cols, h.block_rows, h.block_cols, h.num_blocks, h.nnz,
                          h.row_ptr.data(), h.col_idx.data(), reinterpret_cast<const uint16_t*>(h.values.data()),
                          SPMM_DTYPE_F16};
    spmm_bsr_stats s{};
    spmm_bsr_compute_stats(&v, &s);
    BSR_stats out;
    out.num_blocks = s.num_blocks;
    out.stored_elements = static_cast<long>(s.stored_elements);
    out.original_nnz = s.original_nnz;
    out.fill_in_ratio = s.fill_in_ratio;
    out.block_density = s.block_density;
    return out;
}

// ------------------------------------------------------------------ launchers

void spmm_baseline(const CSR& d_A, const float* d_B, float* d_C, int N) {
    csr_launch(d_A, d_B, d_C, N, SPMM_CSR_ROWWARP, "spmm_baseline");
}
void spmm_memopt(const CSR& d_A, const float* d_B, float* d_C, int N) {
    csr_launch(d_A, d_B, d_C, N, SPMM_CSR_ROWWARP, "spmm_memopt");
}
void spmm_memopt_v2(const CSR& d_A, const float* d_B, float* d_C, int N) {
    csr_launch(d_A, d_B, d_C, N, SPMM_CSR_ROWWARP, "spmm_memopt_v2");
}
void spmm_tiled(const CSR& d_A, const float* d_B, float* d_C, int N) {
    csr_launch(d_A, d_B, d_C, N, SPMM_CSR_MERGE, "spmm_tiled");
}
void spmm_tiled_v2(const CSR& d_A, const float* d_B, float* d_C, int N) {
    if (N % 128 != 0) {
        std::fprintf(stderr,
                     "spmm_tiled_v2: N=%d is not a multiple of COL_TILE=128. Use spmm_tiled for general N, or pad N "
                     "up.\n",
                     N);
        std::abort();
    }
    csr_launch(d_A, d_B, d_C, N, SPMM_CSR_MERGE, "spmm_tiled_v2");
}
void spmm_tiled_v3(const CSR& d_A, const float* d_B, float* d_C, int N) {
    csr_launch(d_A, d_B, d_C, N, SPMM_CSR_MERGE, "spmm_tiled_v3");
}
void spmm_tiled_v4(const CSR& d_A, const float* d_B, float* d_C, int N) {
    csr_launch(d_A, d_B, d_C, N, SPMM_CSR_MERGE, "spmm_tiled_v4");
}

void float_to_half(const float* d_src, half* d_dst, int n_elements) {
    device_check(spmm_convert_f32(d_src, reinterpret_cast<uint16_t*>(d_dst), n_elements, SPMM_DTYPE_F16, nullptr),
                 "float_to_half");
}

void spmm_wmma(const BSR& d_bsr, const half* d_B_fp16, float* d_C, int N) {
    const spmm_bsr_view v{d_bsr.num_rows, d_bsr.num_cols, d_bsr.block_rows, d_bsr.block_cols, d_bsr.num_blocks,
                          d_bsr.nnz, d_bsr.row_ptr, d_bsr.col_idx, reinterpret_cast<const uint16_t*>(d_bsr.values),
                          SPMM_DTYPE_F16};
    device_check(spmm_bsr16(&v, d_B_fp16, d_C, N, nullptr), "spmm_wmma");
}

// ------------------------------------------------------------------ hybrid

HybridPlan hybrid_choose(const CSR& h_A, int N, float fill_in_threshold) {
    const spmm_csr_view v = view_of(h_A);
    spmm_hybrid_plan p{};
    const int rc = spmm_hybrid_choose(&v, N, fill_in_threshold, &p);
    if (rc != SPMM_OK) throw std::runtime_error(std::string("hybrid_choose: ") + spmm_status_string(rc));
    HybridPlan plan;
    plan.backend = p.backend == SPMM_BACKEND_TC ? Backend::TENSOR_WMMA : Backend::CSR_TILED;
    plan.fill_in_ratio = p.fill_in_ratio;
    plan.block_density = p.block_density;
    plan.threshold = p.threshold;
    plan.n_aligned = p.n_aligned != 0;
    plan.reason = p.reason;
    return plan;
}

const char* backend_name(Backend b) {
    return spmm_backend_name(b == Backend::TENSOR_WMMA ? SPMM_BACKEND_TC : SPMM_BACKEND_CSR);
}

float spmm_hybrid_run(const HybridPlan& plan, const CSR& h_A, const float* h_B, float* h_C, int N, int warmup,
                      int iters) {
    spmm_hybrid_plan p{};
    p.backend = plan.backend == Backend::TENSOR_WMMA ? SPMM_BACKEND_TC : SPMM_BACKEND_CSR;
    p.fill_in_ratio = plan.fill_in_ratio;
    p.block_density = plan.block_density;
    p.threshold = plan.threshold;
    p.n_aligned = plan.n_aligned;
    p.reason = plan.reason;
    const spmm_csr_view v = view_of(h_A);
    float ms = 0.f;
    device_check(spmm_hybrid_run(&p, &v, h_B, h_C, N, warmup, iters, &ms), "spmm_hybrid_run");
    return ms;
}

// ------------------------------------------------------------------ multi-GPU

int gpu_count() { return spmm_gpu_count(); }

MultiGpuResult spmm_multigpu(const CSR& h_A, const float* h_B, float* h_C, int N, int num_gpus, int warmup, int iters) {
    const int visible = spmm_gpu_count();
    int g = num_gpus > visible ? visible : num_gpus;
    if (g < 1) g = 1;
    MultiGpuResult r;
    r.rows.assign(g, 0);
    r.nnz.assign(g, 0);
    const spmm_csr_view v = view_of(h_A);
    int used = 0;
    float bcast = 0.f;
    device_check(spmm_multigpu_run(&v, h_B, h_C, N, g, warmup, iters, &r.time_ms, &used, r.rows.data(), r.nnz.data(),
                                   &bcast),
                 "spmm_multigpu");
    r.num_gpus = used;
    r.rows.resize(used);
    r.nnz.resize(used);
    return r;
}

float spmm_unified(const CSR& h_A, const float* h_B, float* h_C, int N, int warmup, int iters) {
    const spmm_csr_view v = view_of(h_A);
    float ms = 0.f;
    device_check(spmm_unified_run(&v, h_B, h_C, N, warmup, iters, &ms), "spmm_unified");
    return ms;
}

}  // namespace spmm
