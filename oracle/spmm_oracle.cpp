// TEST INFRASTRUCTURE ONLY -- NOT PART OF THE PRODUCT.
//
// CPU restatement of the reference SpMM path (Adityaa-Saha17/Sparse-Matrix-Multiplication),
// used as the parity oracle by tests/, by __graft_entry__.smoke() and as bench.py's
// cpu_baseline leg. The product library never links, loads or calls this file.
//
// Every function cites the reference file:line whose behaviour it restates. The code is
// written independently: it follows the reference's *semantics* (draw order, sort keys,
// rounding, accumulation order), not its text.
//
// Parity pins (checked by tests/test_oracle_golden.py):
//   * generator nnz per (size, density) cell at seed 42: scripts/roofline.py:59-154,
//     README.md:233 (4096^2, d=0.01 -> 167686);
//   * BSR-16 block counts / fill-in / block density: reports/tensor_core_wmma.md:43-56;
//   * bit-identical CSR, BSR and bounds against the reference's own host code compiled
//     into oracle/_ref/ (oracle/Makefile target `ref`) when that build is present.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <random>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

void orc_free(void* p) { std::free(p); }

// ---------------------------------------------------------------------------------------
// COO -> CSR: index sort by (row, col), then count + inclusive scan; duplicates are kept.
// Restates src/csr.cu:44-72 (note: csr.h:20 claims de-duplication, the code does none).
// ---------------------------------------------------------------------------------------
int orc_csr_from_coo(int rows, int cols, int n, const int* ri, const int* ci, const float* vi,
                     int** row_ptr, int** col_idx, float** values) {
    (void)cols;
    std::vector<int> order(n);
    for (int i = 0; i < n; ++i) order[i] = i;
    // Same comparator as the reference so that std::sort (same libstdc++) yields the same
    // permutation even for duplicate coordinates.
    std::sort(order.begin(), order.end(), [&](int a, int b) {
        if (ri[a] != ri[b]) return ri[a] < ri[b];
        return ci[a] < ci[b];
    });
    int* rp = static_cast<int*>(std::calloc(rows + 1, sizeof(int)));
    int* cp = static_cast<int*>(std::malloc(sizeof(int) * (n > 0 ? n : 1)));
    float* vp = static_cast<float*>(std::malloc(sizeof(float) * (n > 0 ? n : 1)));
    if (!rp || !cp || !vp) return -1;
    for (int i = 0; i < n; ++i) {
        const int p = order[i];
        cp[i] = ci[p];
        vp[i] = vi[p];
        rp[ri[p] + 1] += 1;
    }
    for (int r = 0; r < rows; ++r) rp[r + 1] += rp[r];
    *row_ptr = rp;
    *col_idx = cp;
    *values = vp;
    return 0;
}

// ---------------------------------------------------------------------------------------
// Uniform Bernoulli generator. Restates src/csr.cu:74-103: one mt19937(seed) stream; for each
// cell in row-major order draw U[0,1) as float and keep the cell when it is < density, in
// which case the very next draw is its value U[-1,1). Uses libstdc++'s own distributions,
// exactly as the reference does, so the stream is the reference's stream.
// ---------------------------------------------------------------------------------------
int orc_gen_uniform_csr(int rows, int cols, float density, int seed,
                        int** row_ptr, int** col_idx, float** values, int* nnz_out) {
    if (density < 0.f || density > 1.f) return -2;
    std::mt19937 rng(static_cast<uint32_t>(seed));
    std::uniform_real_distribution<float> keep(0.f, 1.f);
    std::uniform_real_distribution<float> val(-1.f, 1.f);
    int* rp = static_cast<int*>(std::malloc(sizeof(int) * (rows + 1)));
    std::vector<int> cs;
    std::vector<float> vs;
    rp[0] = 0;
    for (int r = 0; r < rows; ++r) {
        for (int c = 0; c < cols; ++c) {
            if (keep(rng) < density) {
                cs.push_back(c);
                vs.push_back(val(rng));
            }
        }
        rp[r + 1] = static_cast<int>(cs.size());
    }
    // The generator emits cells already ordered by (row, col) with unique keys, so the
    // reference's COO->CSR sort is the identity on this input.
    const size_t n = cs.size();
    int* cp = static_cast<int*>(std::malloc(sizeof(int) * (n > 0 ? n : 1)));
    float* vp = static_cast<float*>(std::malloc(sizeof(float) * (n > 0 ? n : 1)));
    if (n) {
        std::memcpy(cp, cs.data(), sizeof(int) * n);
        std::memcpy(vp, vs.data(), sizeof(float) * n);
    }
    *row_ptr = rp;
    *col_idx = cp;
    *values = vp;
    *nnz_out = static_cast<int>(n);
    return 0;
}

// Dense B: mt19937(seed), U[-1,1) per element in row-major order.
// Restates src/bench/harness.cu:114-120 (and src/bench/spmm_run.cu, same helper).
void orc_gen_dense(int rows, int cols, int seed, float* out) {
    std::mt19937 rng(static_cast<uint32_t>(seed));
    std::uniform_real_distribution<float> uni(-1.f, 1.f);
    const size_t n = static_cast<size_t>(rows) * cols;
    for (size_t i = 0; i < n; ++i) out[i] = uni(rng);
}

// Row slice [b, e) rebased to 0. Restates src/csr.cu:105-123.
int orc_row_slice(const int* row_ptr, const int* col_idx, const float* values, int b, int e,
                  int** rp_out, int** ci_out, float** v_out, int* nnz_out) {
    if (b < 0 || b > e) return -1;
    const int rows = e - b;
    const int start = row_ptr[b], stop = row_ptr[e];
    const int n = stop - start;
    int* rp = static_cast<int*>(std::malloc(sizeof(int) * (rows + 1)));
    int* cp = static_cast<int*>(std::malloc(sizeof(int) * (n > 0 ? n : 1)));
    float* vp = static_cast<float*>(std::malloc(sizeof(float) * (n > 0 ? n : 1)));
    for (int r = 0; r <= rows; ++r) rp[r] = row_ptr[b + r] - start;
    if (n > 0) {
        std::memcpy(cp, col_idx + start, sizeof(int) * n);
        std::memcpy(vp, values + start, sizeof(float) * n);
    }
    *rp_out = rp;
    *ci_out = cp;
    *v_out = vp;
    *nnz_out = n;
    return 0;
}

// ---------------------------------------------------------------------------------------
// FP32 -> FP16 bits, round to nearest even (what __float2half does). The oracle relies on
// the compiler's _Float16 conversion (libgcc, correctly rounded), independent of CUDA.
// ---------------------------------------------------------------------------------------
uint16_t orc_f32_to_f16(float x) {
    _Float16 h = static_cast<_Float16>(x);
    uint16_t bits;
    std::memcpy(&bits, &h, 2);
    return bits;
}

float orc_f16_to_f32(uint16_t bits) {
    _Float16 h;
    std::memcpy(&h, &bits, 2);
    return static_cast<float>(h);
}

// FP32 -> BF16 bits, round to nearest even (NaN kept quiet).
uint16_t orc_f32_to_bf16(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return static_cast<uint16_t>((u >> 16) | 0x40u);
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return static_cast<uint16_t>(u >> 16);
}

float orc_bf16_to_f32(uint16_t bits) {
    uint32_t u = static_cast<uint32_t>(bits) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

void orc_convert_f32(const float* src, uint16_t* dst, long n, int to_bf16) {
    for (long i = 0; i < n; ++i) dst[i] = to_bf16 ? orc_f32_to_bf16(src[i]) : orc_f32_to_f16(src[i]);
}

// ---------------------------------------------------------------------------------------
// CSR -> BSR-16. Restates src/bsr.cu:30-109: per block-row the sorted unique block-column
// list, exclusive scan into row_ptr, zero-filled FP32 staging written at
// (block, r%16, c%16) -- a later duplicate overwrites an earlier one -- then FP32->FP16 RN.
// values_out holds FP16 bits; block b occupies [b*256, (b+1)*256), row-major inside.
// ---------------------------------------------------------------------------------------
int orc_bsr_from_csr(int M, int K, const int* row_ptr, const int* col_idx, const float* values,
                     int* block_rows_out, int* block_cols_out, int* num_blocks_out,
                     int** brp_out, int** bci_out, uint16_t** bval_out) {
    const int BS = 16;
    const int br_n = (M + BS - 1) / BS;
    const int bc_n = (K + BS - 1) / BS;
    std::vector<std::vector<int>> cols(br_n);
    for (int r = 0; r < M; ++r)
        for (int p = row_ptr[r]; p < row_ptr[r + 1]; ++p) cols[r / BS].push_back(col_idx[p] / BS);
    for (auto& v : cols) {
        std::sort(v.begin(), v.end());
        v.erase(std::unique(v.begin(), v.end()), v.end());
    }
    int* brp = static_cast<int*>(std::malloc(sizeof(int) * (br_n + 1)));
    brp[0] = 0;
    for (int b = 0; b < br_n; ++b) brp[b + 1] = brp[b] + static_cast<int>(cols[b].size());
    const int nb = brp[br_n];
    int* bci = static_cast<int*>(std::malloc(sizeof(int) * (nb > 0 ? nb : 1)));
    for (int b = 0; b < br_n; ++b)
        for (size_t i = 0; i < cols[b].size(); ++i) bci[brp[b] + i] = cols[b][i];
    std::vector<float> stage(static_cast<size_t>(nb) * 256, 0.f);
    for (int r = 0; r < M; ++r) {
        const int b = r / BS;
        for (int p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
            const int c = col_idx[p];
            const int local = static_cast<int>(std::lower_bound(cols[b].begin(), cols[b].end(), c / BS) -
                                               cols[b].begin());
            stage[static_cast<size_t>(brp[b] + local) * 256 + (r % BS) * BS + (c % BS)] = values[p];
        }
    }
    uint16_t* bv = static_cast<uint16_t*>(std::malloc(sizeof(uint16_t) * (stage.size() > 0 ? stage.size() : 1)));
    for (size_t i = 0; i < stage.size(); ++i) bv[i] = orc_f32_to_f16(stage[i]);
    *block_rows_out = br_n;
    *block_cols_out = bc_n;
    *num_blocks_out = nb;
    *brp_out = brp;
    *bci_out = bci;
    *bval_out = bv;
    return 0;
}

// Fill-in statistics. Restates src/bsr.cu:149-162.
void orc_bsr_stats(int num_blocks, int nnz, int block_rows, int block_cols, long* stored,
                   double* fill_in, double* block_density) {
    *stored = static_cast<long>(num_blocks) * 256;
    *fill_in = nnz > 0 ? static_cast<double>(*stored) / nnz : 0.0;
    const long total = static_cast<long>(block_rows) * block_cols;
    *block_density = total > 0 ? static_cast<double>(num_blocks) / total : 0.0;
}

// nnz-balanced row bounds. Restates src/spmm_multigpu.cu:26-40: bounds[g] is the first row
// r (the scan resumes where g-1 stopped) with row_ptr[r] >= floor(nnz*g/G), then a
// monotone fix-up; bounds[0] = 0, bounds[G] = rows.
void orc_nnz_balanced_bounds(const int* row_ptr, int rows, long nnz, int G, int* bounds) {
    for (int g = 0; g <= G; ++g) bounds[g] = 0;
    bounds[G] = rows;
    int r = 0;
    for (int g = 1; g < G; ++g) {
        const long target = (nnz * g) / G;
        while (r < rows && row_ptr[r] < target) ++r;
        bounds[g] = r;
    }
    for (int g = 1; g <= G; ++g) bounds[g] = std::max(bounds[g], bounds[g - 1]);
}

static void set_threads(int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

int orc_max_threads() {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

// ---------------------------------------------------------------------------------------
// CSR x dense, FP32, the reference's per-element semantics: for every (i, j) the sum runs
// sequentially over p = row_ptr[i] .. row_ptr[i+1]-1 as sum = fma(v_p, B[col_p, j], sum)
// starting from +0 (src/kernels/spmm_baseline.cu:19-24; nvcc contracts `sum += v*b` into an
// FMA). Rows are independent, so OpenMP over rows changes nothing in the arithmetic.
// schedule_dynamic selects a dynamic schedule (used for skewed row lengths).
// ---------------------------------------------------------------------------------------
void orc_spmm_csr_f32(int M, int N, const int* row_ptr, const int* col_idx, const float* values,
                      const float* B, float* C, int threads, int schedule_dynamic) {
    set_threads(threads);
    if (schedule_dynamic) {
#pragma omp parallel for schedule(dynamic, 16)
        for (int i = 0; i < M; ++i) {
            float* c = C + static_cast<size_t>(i) * N;
            for (int j = 0; j < N; ++j) c[j] = 0.f;
            for (int p = row_ptr[i]; p < row_ptr[i + 1]; ++p) {
                const float v = values[p];
                const float* b = B + static_cast<size_t>(col_idx[p]) * N;
                for (int j = 0; j < N; ++j) c[j] = std::fmaf(v, b[j], c[j]);
            }
        }
    } else {
#pragma omp parallel for schedule(static)
        for (int i = 0; i < M; ++i) {
            float* c = C + static_cast<size_t>(i) * N;
            for (int j = 0; j < N; ++j) c[j] = 0.f;
            for (int p = row_ptr[i]; p < row_ptr[i + 1]; ++p) {
                const float v = values[p];
                const float* b = B + static_cast<size_t>(col_idx[p]) * N;
                for (int j = 0; j < N; ++j) c[j] = std::fmaf(v, b[j], c[j]);
            }
        }
    }
}

// The reference's FP32 semantics with one documented change, the one the engine's merge-path
// kernel makes for long rows: a row with more than S nonzeros is cut wherever r + p is a
// multiple of S (r = row, p = global nonzero index); each piece is its own sequential FMA
// chain from +0 and the pieces are added left to right in FP32. Rows with <= S nonzeros are
// computed exactly as orc_spmm_csr_f32 does. Lets the tests demand bit equality everywhere.
void orc_spmm_csr_f32_split(int M, int N, const int* row_ptr, const int* col_idx, const float* values,
                            const float* B, float* C, int S, int threads) {
    set_threads(threads);
#pragma omp parallel for schedule(dynamic, 16)
    for (int i = 0; i < M; ++i) {
        float* c = C + static_cast<size_t>(i) * N;
        const int rs = row_ptr[i], re = row_ptr[i + 1];
        std::vector<float> piece(N);
        for (int j = 0; j < N; ++j) c[j] = 0.f;
        bool first = true;
        int p0 = rs;
        while (p0 < re || first) {
            int p1 = re;
            if (re - rs > S) {
                const long next_cut = (static_cast<long>(i) + p0) / S * S + S - i;  // next multiple of S
                if (next_cut < re) p1 = static_cast<int>(next_cut);
            }
            for (int j = 0; j < N; ++j) piece[j] = 0.f;
            for (int p = p0; p < p1; ++p) {
                const float v = values[p];
                const float* b = B + static_cast<size_t>(col_idx[p]) * N;
                for (int j = 0; j < N; ++j) piece[j] = std::fmaf(v, b[j], piece[j]);
            }
            if (first) {
                for (int j = 0; j < N; ++j) c[j] = piece[j];
            } else {
                for (int j = 0; j < N; ++j) c[j] = c[j] + piece[j];
            }
            first = false;
            p0 = p1;
            if (p0 >= re) break;
        }
    }
}

// Same product with FP64 accumulation of exact FP32 products (the tolerance reference).
void orc_spmm_csr_f64(int M, int N, const int* row_ptr, const int* col_idx, const float* values,
                      const float* B, double* C, int threads) {
    set_threads(threads);
#pragma omp parallel for schedule(dynamic, 16)
    for (int i = 0; i < M; ++i) {
        double* c = C + static_cast<size_t>(i) * N;
        for (int j = 0; j < N; ++j) c[j] = 0.0;
        for (int p = row_ptr[i]; p < row_ptr[i + 1]; ++p) {
            const double v = values[p];
            const float* b = B + static_cast<size_t>(col_idx[p]) * N;
            for (int j = 0; j < N; ++j) c[j] += v * static_cast<double>(b[j]);
        }
    }
}

// BSR-16 x dense with 16-bit operands widened exactly and FP64 accumulation. Semantics of
// src/kernels/spmm_wmma.cu:63-89: C[br*16+r, n] = sum over blocks b of block-row br of
// sum_k A_b[r, k] * B[col_b*16 + k, n]; rows >= M and B rows >= K contribute nothing.
// dtype 0 = FP16 bits, 1 = BF16 bits (A and B share the type).
void orc_spmm_bsr_f64(int M, int K, int N, int block_rows, const int* brp, const int* bci,
                      const uint16_t* bval, const uint16_t* B16, int dtype, double* C, int threads) {
    set_threads(threads);
    auto widen = [dtype](uint16_t h) -> double {
        return dtype ? static_cast<double>(orc_bf16_to_f32(h)) : static_cast<double>(orc_f16_to_f32(h));
    };
#pragma omp parallel for schedule(dynamic, 4)
    for (int br = 0; br < block_rows; ++br) {
        std::vector<double> acc(static_cast<size_t>(16) * N, 0.0);
        for (int b = brp[br]; b < brp[br + 1]; ++b) {
            const int bc = bci[b];
            for (int r = 0; r < 16; ++r) {
                for (int k = 0; k < 16; ++k) {
                    const int kk = bc * 16 + k;
                    if (kk >= K) continue;
                    const double a = widen(bval[static_cast<size_t>(b) * 256 + r * 16 + k]);
                    if (a == 0.0) continue;
                    const uint16_t* brow = B16 + static_cast<size_t>(kk) * N;
                    double* arow = acc.data() + static_cast<size_t>(r) * N;
                    for (int n = 0; n < N; ++n) arow[n] += a * widen(brow[n]);
                }
            }
        }
        for (int r = 0; r < 16; ++r) {
            const int row = br * 16 + r;
            if (row >= M) break;
            std::memcpy(C + static_cast<size_t>(row) * N, acc.data() + static_cast<size_t>(r) * N,
                        sizeof(double) * N);
        }
    }
}

// Error metrics of src/bench/harness.cu:173-196: max |d|; max |d|/|ref| over cells with
// |ref| > 1e-3 * max|ref| (FP32 arithmetic as in the reference); rel_l2 in FP64.
void orc_compare(const float* ours, const float* ref, long n, float* max_abs, float* max_rel,
                 float* rel_l2) {
    float ref_max = 0.f;
    for (long i = 0; i < n; ++i) ref_max = std::max(ref_max, std::fabs(ref[i]));
    const float floor_ = 1e-3f * ref_max;
    float ma = 0.f, mr = 0.f;
    double es = 0.0, rs = 0.0;
    for (long i = 0; i < n; ++i) {
        const float d = std::fabs(ours[i] - ref[i]);
        ma = std::max(ma, d);
        const float a = std::fabs(ref[i]);
        if (a > floor_) mr = std::max(mr, d / a);
        es += static_cast<double>(d) * d;
        rs += static_cast<double>(a) * a;
    }
    *max_abs = ma;
    *max_rel = mr;
    *rel_l2 = rs > 0.0 ? static_cast<float>(std::sqrt(es / rs)) : 0.f;
}

}  // extern "C"
