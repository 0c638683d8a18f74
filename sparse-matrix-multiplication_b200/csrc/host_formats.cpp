// Host-side format utilities of libspmm_b200.so: CSR allocation, COO->CSR, the seeded
// generators, row slicing, the binary CSR file format, CSR->BSR-16 conversion, fill-in
// statistics and the nnz-balanced row partition. Plain C++17, no CUDA.
//
// These reproduce the reference's host behaviour exactly (same outputs bit for bit), because
// the configs, the hybrid decision and the multi-GPU split are all defined by it:
//   generator     src/csr.cu:74-103        COO->CSR      src/csr.cu:44-72
//   row slice     src/csr.cu:105-123       binary IO     src/csr.cu:125-150
//   CSR->BSR      src/bsr.cu:30-109        stats         src/bsr.cu:149-162
//   bounds        src/spmm_multigpu.cu:26-40
//   dense B       src/bench/harness.cu:114-120

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <thread>
#include <vector>

#include "spmm_c.h"

namespace {

// ---------------------------------------------------------------------------------------
// MT19937 (Matsumoto & Nishimura, 1998), producing the tempered output in blocks of 624
// words. The state recurrence, seeding and tempering are the published algorithm; the
// block layout lets the generator scan words with a plain compare loop.
// ---------------------------------------------------------------------------------------
class MersenneBlock {
public:
    static constexpr int kN = 624;
    static constexpr int kM = 397;

    explicit MersenneBlock(uint32_t seed) {
        s_[0] = seed;
        for (int i = 1; i < kN; ++i) s_[i] = 1812433253u * (s_[i - 1] ^ (s_[i - 1] >> 30)) + static_cast<uint32_t>(i);
    }

    // Advance the state by one full block and write the 624 tempered outputs.
    __attribute__((always_inline)) void next_block(uint32_t* out) {
        constexpr uint32_t kUpper = 0x80000000u, kLower = 0x7fffffffu, kA = 0x9908b0dfu;
        int i = 0;
        for (; i < kN - kM; ++i) {
            const uint32_t y = (s_[i] & kUpper) | (s_[i + 1] & kLower);
            s_[i] = s_[i + kM] ^ (y >> 1) ^ ((y & 1u) ? kA : 0u);
        }
        for (; i < kN - 1; ++i) {
            const uint32_t y = (s_[i] & kUpper) | (s_[i + 1] & kLower);
            s_[i] = s_[i + kM - kN] ^ (y >> 1) ^ ((y & 1u) ? kA : 0u);
        }
        {
            const uint32_t y = (s_[kN - 1] & kUpper) | (s_[0] & kLower);
            s_[kN - 1] = s_[kM - 1] ^ (y >> 1) ^ ((y & 1u) ? kA : 0u);
        }
        for (int k = 0; k < kN; ++k) {
            uint32_t y = s_[k];
            y ^= y >> 11;
            y ^= (y << 7) & 0x9d2c5680u;
            y ^= (y << 15) & 0xefc60000u;
            y ^= y >> 18;
            out[k] = y;
        }
    }

private:
    uint32_t s_[kN];
};

// A word stream over MersenneBlock.
class WordStream {
public:
    explicit WordStream(uint32_t seed) : gen_(seed) {}
    uint32_t next() {
        if (pos_ == MersenneBlock::kN) refill();
        return buf_[pos_++];
    }
    // Number of words left in the current block (refilling first if it is empty).
    int available() {
        if (pos_ == MersenneBlock::kN) refill();
        return MersenneBlock::kN - pos_;
    }
    const uint32_t* cursor() const { return buf_ + pos_; }
    void skip(int n) { pos_ += n; }

private:
    void refill() {
        gen_.next_block(buf_);
        pos_ = 0;
    }
    MersenneBlock gen_;
    uint32_t buf_[MersenneBlock::kN];
    int pos_ = MersenneBlock::kN;
};

// U[0,1) float from one 32-bit word, as the C++ standard library's canonical generator
// does it for float and a 32-bit engine: float(x) / 2^32, with 1.0 replaced by the largest
// float below 1.
inline float canonical01(uint32_t x) {
    const float r = static_cast<float>(x) / 4294967296.0f;
    return r >= 1.0f ? 0x1.fffffep-1f : r;
}

// U[a,b) as the standard library computes it: canonical * (b - a) + a.
inline float uniform_ab(uint32_t x, float a, float b) { return canonical01(x) * (b - a) + a; }

// True when any of the 32 words is below T (T <= 2^32; compared in signed space so the loop
// vectorises with plain SSE2 compares).
__attribute__((always_inline)) inline bool any_below32(const uint32_t* w, uint64_t T) {
    if (T > 0xffffffffull) return true;
    const int32_t ts = static_cast<int32_t>(static_cast<uint32_t>(T) ^ 0x80000000u);
    int hit = 0;
    for (int k = 0; k < 32; ++k) hit |= static_cast<int32_t>(w[k] ^ 0x80000000u) < ts;
    return hit != 0;
}

// Smallest word value x with canonical01(x) >= density (words below it are "kept").
uint64_t keep_threshold(float density) {
    uint64_t lo = 0, hi = 1ull << 32;  // answer in [lo, hi]
    while (lo < hi) {
        const uint64_t mid = lo + (hi - lo) / 2;
        if (canonical01(static_cast<uint32_t>(mid)) < density) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

bool alloc_csr(int32_t rows, int32_t cols, int32_t nnz, spmm_csr_host* out) {
    out->rows = rows;
    out->cols = cols;
    out->nnz = nnz;
    out->row_ptr = static_cast<int32_t*>(std::malloc(sizeof(int32_t) * (static_cast<size_t>(rows) + 1)));
    out->col_idx = static_cast<int32_t*>(std::malloc(sizeof(int32_t) * (nnz > 0 ? static_cast<size_t>(nnz) : 1)));
    out->values = static_cast<float*>(std::malloc(sizeof(float) * (nnz > 0 ? static_cast<size_t>(nnz) : 1)));
    if (!out->row_ptr || !out->col_idx || !out->values) {
        std::free(out->row_ptr);
        std::free(out->col_idx);
        std::free(out->values);
        out->row_ptr = nullptr;
        out->col_idx = nullptr;
        out->values = nullptr;
        return false;
    }
    return true;
}

// FP32 -> FP16 bits, IEEE round-to-nearest-even; NaN becomes the canonical 0x7fff.
uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t a = x & 0x7fffffffu;
    if (a > 0x7f800000u) return 0x7fffu;                 // NaN
    if (a >= 0x477ff000u) return static_cast<uint16_t>(sign | 0x7c00u);  // >= 65520 -> inf
    if (a < 0x38800000u) {                               // half subnormal or zero
        if (a < 0x33000000u) return static_cast<uint16_t>(sign);  // below 2^-25
        const uint32_t e = a >> 23;
        const uint32_t m = (a & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e;                 // 14..24
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return static_cast<uint16_t>(sign | q);
    }
    const uint32_t r = a - 0x38000000u;                  // rebias 127 -> 15
    uint32_t q = r >> 13;
    const uint32_t rem = r & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
    return static_cast<uint16_t>(sign | q);
}

// FP32 -> BF16 bits, round-to-nearest-even; NaN stays a (quiet) NaN.
uint16_t f32_to_bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return static_cast<uint16_t>((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(u >> 16);
}

}  // namespace

namespace {

// The generator's word loop, compiled twice (AVX2 and baseline x86-64) and picked at load
// time: the block twist and the skip test vectorise 8-wide with AVX2 (2.2x on the config-5
// matrix). Same words, same output either way.
__attribute__((target_clones("avx2", "default")))
int generate_uniform_core(int32_t rows, int32_t cols, float density, int32_t seed, spmm_csr_host* out) {
    const uint64_t T = keep_threshold(density);
    const uint64_t cells = static_cast<uint64_t>(rows) * static_cast<uint64_t>(cols);
    WordStream ws(static_cast<uint32_t>(seed));

    std::vector<int32_t> row_ptr(static_cast<size_t>(rows) + 1, 0);
    std::vector<int32_t> col;
    std::vector<float> val;
    const double expect = static_cast<double>(cells) * density;
    col.reserve(static_cast<size_t>(expect * 1.01 + 1024));
    val.reserve(col.capacity());

    int32_t cur_row = 0;  // rows < cur_row have their row_ptr end filled
    uint64_t cell = 0;
    while (cell < cells) {
        const int avail = ws.available();
        const uint64_t want = std::min<uint64_t>(static_cast<uint64_t>(avail), cells - cell);
        const uint32_t* w = ws.cursor();
        const int n = static_cast<int>(want);
        int j = 0;
        // Skip 32-word groups without a kept cell (a value word below T only stops the skip).
        while (j + 32 <= n && !any_below32(w + j, T)) j += 32;
        while (j < n && w[j] >= T) ++j;
        if (j == n) {
            ws.skip(n);
            cell += static_cast<uint64_t>(n);
            continue;
        }
        ws.skip(j + 1);  // the kept cell's Bernoulli word
        cell += static_cast<uint64_t>(j);
        const float v = uniform_ab(ws.next(), -1.f, 1.f);  // its value is the very next word
        const int32_t r = static_cast<int32_t>(cell / static_cast<uint64_t>(cols));
        const int32_t c = static_cast<int32_t>(cell % static_cast<uint64_t>(cols));
        while (cur_row < r) row_ptr[++cur_row] = static_cast<int32_t>(col.size());
        if (col.size() >= static_cast<size_t>(std::numeric_limits<int32_t>::max())) return SPMM_ERR_TOO_LARGE;
        col.push_back(c);
        val.push_back(v);
        cell += 1;
    }
    while (cur_row < rows) row_ptr[++cur_row] = static_cast<int32_t>(col.size());

    const int32_t nnz = static_cast<int32_t>(col.size());
    if (!alloc_csr(rows, cols, nnz, out)) return SPMM_ERR_NO_MEMORY;
    std::memcpy(out->row_ptr, row_ptr.data(), sizeof(int32_t) * row_ptr.size());
    if (nnz) {
        std::memcpy(out->col_idx, col.data(), sizeof(int32_t) * col.size());
        std::memcpy(out->values, val.data(), sizeof(float) * val.size());
    }
    return SPMM_OK;
}

__attribute__((target_clones("avx2", "default")))
void generate_dense_core(size_t n, int32_t seed, float* out) {
    WordStream ws(static_cast<uint32_t>(seed));
    for (size_t i = 0; i < n; ++i) out[i] = uniform_ab(ws.next(), -1.f, 1.f);
}

}  // namespace

extern "C" {

int spmm_csr_host_alloc(int32_t rows, int32_t cols, int32_t nnz, spmm_csr_host* out) {
    if (!out || rows < 0 || cols < 0 || nnz < 0) return SPMM_ERR_INVALID_ARG;
    return alloc_csr(rows, cols, nnz, out) ? SPMM_OK : SPMM_ERR_NO_MEMORY;
}

void spmm_csr_host_free(spmm_csr_host* m) {
    if (!m) return;
    std::free(m->row_ptr);
    std::free(m->col_idx);
    std::free(m->values);
    m->row_ptr = nullptr;
    m->col_idx = nullptr;
    m->values = nullptr;
    m->rows = m->cols = m->nnz = 0;
}

int spmm_csr_from_coo_host(int32_t rows, int32_t cols, int32_t n, const int32_t* ri, const int32_t* ci,
                           const float* vi, spmm_csr_host* out) {
    if (!out || rows < 0 || cols < 0 || n < 0 || (n > 0 && (!ri || !ci || !vi))) return SPMM_ERR_INVALID_ARG;
    for (int32_t i = 0; i < n; ++i)
        if (ri[i] < 0 || ri[i] >= rows) return SPMM_ERR_INVALID_ARG;
    // Permutation by (row, col) with the same comparison sequence as the reference, so that
    // even duplicate coordinates land in the same order.
    std::vector<int32_t> perm(static_cast<size_t>(n));
    for (int32_t i = 0; i < n; ++i) perm[i] = i;
    std::sort(perm.begin(), perm.end(), [ri, ci](int32_t a, int32_t b) {
        return ri[a] != ri[b] ? ri[a] < ri[b] : ci[a] < ci[b];
    });
    if (!alloc_csr(rows, cols, n, out)) return SPMM_ERR_NO_MEMORY;
    std::memset(out->row_ptr, 0, sizeof(int32_t) * (static_cast<size_t>(rows) + 1));
    for (int32_t i = 0; i < n; ++i) {
        const int32_t p = perm[i];
        out->col_idx[i] = ci[p];
        out->values[i] = vi[p];
        out->row_ptr[ri[p] + 1] += 1;
    }
    for (int32_t r = 0; r < rows; ++r) out->row_ptr[r + 1] += out->row_ptr[r];
    return SPMM_OK;
}


int spmm_generate_uniform_csr(int32_t rows, int32_t cols, float density, int32_t seed, spmm_csr_host* out) {
    if (!out || rows < 0 || cols < 0 || !(density >= 0.f && density <= 1.f)) return SPMM_ERR_INVALID_ARG;
    return generate_uniform_core(rows, cols, density, seed, out);
}

int spmm_generate_dense(int32_t rows, int32_t cols, int32_t seed, float* out) {
    if (rows < 0 || cols < 0 || (!out && rows && cols)) return SPMM_ERR_INVALID_ARG;
    generate_dense_core(static_cast<size_t>(rows) * static_cast<size_t>(cols), seed, out);
    return SPMM_OK;
}

int spmm_generate_uniform_csr_fast(int32_t rows, int32_t cols, float density, int64_t seed, int32_t threads,
                                   spmm_csr_host* out) {
    if (!out || rows < 0 || cols < 0 || !(density >= 0.f && density <= 1.f)) return SPMM_ERR_INVALID_ARG;
    const int nthreads = std::max(1, threads > 0 ? threads : static_cast<int>(std::thread::hardware_concurrency()));
    // Per row: gaps between kept columns are geometric with parameter p, drawn by inversion
    // from a counter-based stream (SplitMix64 over (seed, row, draw)), so rows are
    // independent and the result does not depend on the thread count.
    const double p = density;
    const double log1mp = p < 1.0 ? std::log1p(-p) : 0.0;
    auto mix = [](uint64_t z) {
        z += 0x9e3779b97f4a7c15ull;
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        return z ^ (z >> 31);
    };
    auto row_walk = [&](int32_t r, auto&& emit) {
        if (p <= 0.0 || cols == 0) return;
        uint64_t ctr = mix(static_cast<uint64_t>(seed) ^ mix(static_cast<uint64_t>(r) + 0x51ed27ull));
        int64_t c = -1;
        for (;;) {
            ctr = mix(ctr);
            if (p >= 1.0) {
                c += 1;
            } else {
                const double u = (static_cast<double>(ctr >> 11) + 0.5) * 0x1.0p-53;  // (0, 1)
                c += 1 + static_cast<int64_t>(std::floor(std::log(u) / log1mp));
            }
            if (c >= cols) return;
            ctr = mix(ctr);
            const float v = static_cast<float>((static_cast<double>(ctr >> 40) + 0.5) * 0x1.0p-24) * 2.0f - 1.0f;
            emit(static_cast<int32_t>(c), v);
        }
    };
    // Pass 1: counts per row (in parallel), pass 2: fill (in parallel).
    std::vector<int64_t> counts(static_cast<size_t>(rows) + 1, 0);
    auto run = [&](auto&& body) {
        std::vector<std::thread> pool;
        for (int t = 0; t < nthreads; ++t)
            pool.emplace_back([&, t] {
                for (int32_t r = t; r < rows; r += nthreads) body(r);
            });
        for (auto& th : pool) th.join();
    };
    run([&](int32_t r) {
        int64_t n = 0;
        row_walk(r, [&](int32_t, float) { ++n; });
        counts[r + 1] = n;
    });
    for (int32_t r = 0; r < rows; ++r) counts[r + 1] += counts[r];
    if (counts[rows] > std::numeric_limits<int32_t>::max()) return SPMM_ERR_TOO_LARGE;
    const int32_t nnz = static_cast<int32_t>(counts[rows]);
    if (!alloc_csr(rows, cols, nnz, out)) return SPMM_ERR_NO_MEMORY;
    for (int32_t r = 0; r <= rows; ++r) out->row_ptr[r] = static_cast<int32_t>(counts[r]);
    run([&](int32_t r) {
        int64_t k = counts[r];
        row_walk(r, [&](int32_t c, float v) {
            out->col_idx[k] = c;
            out->values[k] = v;
            ++k;
        });
    });
    return SPMM_OK;
}

int spmm_csr_row_slice_host(const spmm_csr_view* m, int32_t b, int32_t e, spmm_csr_host* out) {
    if (!m || !out || b < 0 || e > m->rows || b > e) return SPMM_ERR_INVALID_ARG;
    const int32_t start = m->row_ptr[b];
    const int32_t stop = m->row_ptr[e];
    const int32_t nnz = stop - start;
    if (nnz < 0) return SPMM_ERR_INVALID_ARG;
    if (!alloc_csr(e - b, m->cols, nnz, out)) return SPMM_ERR_NO_MEMORY;
    for (int32_t r = 0; r <= e - b; ++r) out->row_ptr[r] = m->row_ptr[b + r] - start;
    if (nnz > 0) {
        std::memcpy(out->col_idx, m->col_idx + start, sizeof(int32_t) * nnz);
        std::memcpy(out->values, m->values + start, sizeof(float) * nnz);
    }
    return SPMM_OK;
}

int spmm_csr_read_binary(const char* path, spmm_csr_host* out) {
    if (!path || !out) return SPMM_ERR_INVALID_ARG;
    std::FILE* f = std::fopen(path, "rb");
    if (!f) return SPMM_ERR_IO;
    int32_t hdr[3];
    if (std::fread(hdr, sizeof(int32_t), 3, f) != 3) {
        std::fclose(f);
        return SPMM_ERR_IO;
    }
    if (hdr[0] < 0 || hdr[1] < 0 || hdr[2] < 0) {
        std::fclose(f);
        return SPMM_ERR_IO;
    }
    if (!alloc_csr(hdr[0], hdr[1], hdr[2], out)) {
        std::fclose(f);
        return SPMM_ERR_NO_MEMORY;
    }
    const size_t nr = static_cast<size_t>(hdr[0]) + 1, nz = static_cast<size_t>(hdr[2]);
    const bool ok = std::fread(out->row_ptr, sizeof(int32_t), nr, f) == nr &&
                    std::fread(out->col_idx, sizeof(int32_t), nz, f) == nz &&
                    std::fread(out->values, sizeof(float), nz, f) == nz;
    std::fclose(f);
    if (!ok) {
        spmm_csr_host_free(out);
        return SPMM_ERR_IO;
    }
    return SPMM_OK;
}

int spmm_csr_write_binary(const spmm_csr_view* m, const char* path) {
    if (!m || !path) return SPMM_ERR_INVALID_ARG;
    std::FILE* f = std::fopen(path, "wb");
    if (!f) return SPMM_ERR_IO;
    const int32_t hdr[3] = {m->rows, m->cols, m->nnz};
    const size_t nr = static_cast<size_t>(m->rows) + 1, nz = static_cast<size_t>(m->nnz);
    bool ok = std::fwrite(hdr, sizeof(int32_t), 3, f) == 3 && std::fwrite(m->row_ptr, sizeof(int32_t), nr, f) == nr;
    if (ok && nz) {
        ok = std::fwrite(m->col_idx, sizeof(int32_t), nz, f) == nz && std::fwrite(m->values, sizeof(float), nz, f) == nz;
    }
    ok = (std::fclose(f) == 0) && ok;
    return ok ? SPMM_OK : SPMM_ERR_IO;
}

int spmm_csr_validate_host(const spmm_csr_view* m, int32_t* bad_row) {
    if (bad_row) *bad_row = -1;
    if (!m || m->rows < 0 || m->cols < 0 || m->nnz < 0 || !m->row_ptr) return SPMM_ERR_INVALID_ARG;
    if (m->nnz > 0 && (!m->col_idx || !m->values)) return SPMM_ERR_INVALID_ARG;
    if (m->row_ptr[0] != 0 || m->row_ptr[m->rows] != m->nnz) {
        if (bad_row) *bad_row = m->row_ptr[0] != 0 ? 0 : m->rows;
        return SPMM_ERR_INVALID_ARG;
    }
    for (int32_t r = 0; r < m->rows; ++r) {
        const int32_t a = m->row_ptr[r], b = m->row_ptr[r + 1];
        bool bad = b < a;
        for (int32_t p = a; !bad && p < b; ++p) bad = m->col_idx[p] < 0 || m->col_idx[p] >= m->cols;
        if (bad) {
            if (bad_row) *bad_row = r;
            return SPMM_ERR_INVALID_ARG;
        }
    }
    return SPMM_OK;
}

int spmm_csr_to_bsr16_host(const spmm_csr_view* A, int32_t dtype, spmm_bsr_host* out) {
    if (!A || !out || (dtype != SPMM_DTYPE_F16 && dtype != SPMM_DTYPE_BF16)) return SPMM_ERR_INVALID_ARG;
    if (A->rows < 0 || A->cols < 0 || !A->row_ptr) return SPMM_ERR_INVALID_ARG;
    constexpr int32_t kB = 16;
    const int32_t M = A->rows, K = A->cols;
    const int32_t nbr = (M + kB - 1) / kB, nbc = (K + kB - 1) / kB;

    // Pass 1: sorted unique block-columns of every block-row.
    std::vector<int32_t> brp(static_cast<size_t>(nbr) + 1, 0);
    std::vector<std::vector<int32_t>> lists(static_cast<size_t>(nbr));
    for (int32_t br = 0; br < nbr; ++br) {
        auto& L = lists[br];
        const int32_t r1 = std::min(M, (br + 1) * kB);
        for (int32_t r = br * kB; r < r1; ++r)
            for (int32_t p = A->row_ptr[r]; p < A->row_ptr[r + 1]; ++p) L.push_back(A->col_idx[p] / kB);
        std::sort(L.begin(), L.end());
        L.erase(std::unique(L.begin(), L.end()), L.end());
        brp[br + 1] = brp[br] + static_cast<int32_t>(L.size());
    }
    const int32_t nb = brp[nbr];

    out->rows = M;
    out->cols = K;
    out->block_rows = nbr;
    out->block_cols = nbc;
    out->num_blocks = nb;
    out->nnz = A->nnz;
    out->dtype = dtype;
    out->row_ptr = static_cast<int32_t*>(std::malloc(sizeof(int32_t) * (static_cast<size_t>(nbr) + 1)));
    out->col_idx = static_cast<int32_t*>(std::malloc(sizeof(int32_t) * (nb > 0 ? static_cast<size_t>(nb) : 1)));
    const size_t nvals = static_cast<size_t>(nb) * kB * kB;
    out->values = static_cast<uint16_t*>(std::malloc(sizeof(uint16_t) * (nvals > 0 ? nvals : 1)));
    std::vector<float> stage(nvals, 0.f);
    if (!out->row_ptr || !out->col_idx || !out->values) {
        spmm_bsr_host_free(out);
        return SPMM_ERR_NO_MEMORY;
    }
    std::memcpy(out->row_ptr, brp.data(), sizeof(int32_t) * brp.size());
    for (int32_t br = 0; br < nbr; ++br)
        std::copy(lists[br].begin(), lists[br].end(), out->col_idx + brp[br]);

    // Pass 2: scatter every nonzero into its block (a later duplicate overwrites).
    for (int32_t r = 0; r < M; ++r) {
        const int32_t br = r / kB;
        const auto& L = lists[br];
        for (int32_t p = A->row_ptr[r]; p < A->row_ptr[r + 1]; ++p) {
            const int32_t c = A->col_idx[p];
            const int32_t local = static_cast<int32_t>(std::lower_bound(L.begin(), L.end(), c / kB) - L.begin());
            stage[static_cast<size_t>(brp[br] + local) * kB * kB + (r % kB) * kB + (c % kB)] = A->values[p];
        }
    }
    // Pass 3: round to the 16-bit type.
    if (dtype == SPMM_DTYPE_F16) {
        for (size_t i = 0; i < nvals; ++i) out->values[i] = f32_to_f16_bits(stage[i]);
    } else {
        for (size_t i = 0; i < nvals; ++i) out->values[i] = f32_to_bf16_bits(stage[i]);
    }
    return SPMM_OK;
}

void spmm_bsr_host_free(spmm_bsr_host* b) {
    if (!b) return;
    std::free(b->row_ptr);
    std::free(b->col_idx);
    std::free(b->values);
    b->row_ptr = nullptr;
    b->col_idx = nullptr;
    b->values = nullptr;
}

int spmm_bsr_compute_stats(const spmm_bsr_view* b, spmm_bsr_stats* out) {
    if (!b || !out) return SPMM_ERR_INVALID_ARG;
    out->num_blocks = b->num_blocks;
    out->stored_elements = static_cast<int64_t>(b->num_blocks) * 256;
    out->original_nnz = b->nnz;
    out->fill_in_ratio = b->nnz > 0 ? static_cast<double>(out->stored_elements) / b->nnz : 0.0;
    const int64_t total = static_cast<int64_t>(b->block_rows) * b->block_cols;
    out->block_density = total > 0 ? static_cast<double>(b->num_blocks) / static_cast<double>(total) : 0.0;
    return SPMM_OK;
}

int spmm_nnz_balanced_bounds(const int32_t* row_ptr, int32_t rows, int64_t nnz, int32_t G, int32_t* out) {
    if (!out || G < 1 || rows < 0 || (!row_ptr && rows > 0)) return SPMM_ERR_INVALID_ARG;
    for (int32_t g = 0; g < G; ++g) out[g] = 0;
    out[G] = rows;
    int32_t r = 0;
    for (int32_t g = 1; g < G; ++g) {
        const int64_t target = (nnz * g) / G;
        while (r < rows && row_ptr[r] < target) ++r;
        out[g] = r;
    }
    for (int32_t g = 1; g <= G; ++g) out[g] = std::max(out[g], out[g - 1]);
    return SPMM_OK;
}

}  // extern "C"
