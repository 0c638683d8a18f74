/*
 * spmm_c.h -- C ABI of the B200 SpMM engine (libspmm_b200.so).
 *
 * Computes C[M x N] = A[M x K] * B[K x N] with A sparse (CSR FP32, or BSR 16x16 FP16/BF16)
 * and B, C dense row-major. Plain C: POD views, plain pointers and sizes, an opaque
 * `void* stream` (a cudaStream_t; NULL = legacy default stream). No C++ types cross this
 * boundary, so cgo / ctypes / JNI bindings can be written directly against it.
 *
 * Every entry point returns an int status: SPMM_OK (0) or a negative SPMM_ERR_* code
 * (spmm_status_string() names it). Nothing prints or exits; the C++ API in include/spmm/
 * maps the codes back to the reference's exit/throw behaviour.
 *
 * Each declaration cites the reference interface it replaces as
 * (reference: <path in Adityaa-Saha17/Sparse-Matrix-Multiplication>:<line>).
 */
#ifndef SPMM_C_H
#define SPMM_C_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status codes */
#define SPMM_OK 0
#define SPMM_ERR_INVALID_ARG (-1)  /* bad size, null pointer, malformed CSR/BSR            */
#define SPMM_ERR_MISALIGNED (-2)   /* an operand's alignment / N does not fit this path    */
#define SPMM_ERR_CUDA (-3)         /* a CUDA runtime call failed                           */
#define SPMM_ERR_NCCL (-4)         /* an NCCL call failed                                  */
#define SPMM_ERR_TIMEOUT (-5)      /* a device-side wait ran out of its iteration budget   */
#define SPMM_ERR_UNSUPPORTED (-6)  /* no device / feature for this request                 */
#define SPMM_ERR_NO_MEMORY (-7)    /* host or device allocation failed                     */
#define SPMM_ERR_BAD_INDEX (-8)    /* the device saw an index outside its declared range   */
#define SPMM_ERR_IO (-9)           /* file open / short read / short write                 */
#define SPMM_ERR_TOO_LARGE (-10)   /* the request exceeds a fixed capacity                 */

const char* spmm_status_string(int status);
int spmm_version(void); /* major*10000 + minor*100 + patch */

/* ---------------------------------------------------------------- formats */

/* Read-only CSR view (0-based, int32 indices, columns sorted within a row).
 * (reference: src/csr.h:7-14, struct spmm::CSR) */
typedef struct spmm_csr_view {
    int32_t rows, cols, nnz;
    const int32_t* row_ptr; /* rows + 1 */
    const int32_t* col_idx; /* nnz */
    const float* values;    /* nnz */
} spmm_csr_view;

/* Host CSR whose arrays the library malloc'd; release with spmm_csr_host_free. */
typedef struct spmm_csr_host {
    int32_t rows, cols, nnz;
    int32_t* row_ptr;
    int32_t* col_idx;
    float* values;
} spmm_csr_host;

#define SPMM_DTYPE_F16 0
#define SPMM_DTYPE_BF16 1

/* BSR with 16x16 blocks; block b holds values[b*256 .. b*256+255], row-major inside the
 * block, as FP16 or BF16 bits. (reference: src/bsr.h:22-60, BSR_BLOCK / BSR_host / BSR) */
typedef struct spmm_bsr_view {
    int32_t rows, cols;             /* original M, K                       */
    int32_t block_rows, block_cols; /* ceil(M/16), ceil(K/16)              */
    int32_t num_blocks;             /* non-empty blocks                    */
    int32_t nnz;                    /* original nonzeros                   */
    const int32_t* row_ptr;         /* block_rows + 1                      */
    const int32_t* col_idx;         /* num_blocks, sorted per block-row    */
    const uint16_t* values;         /* num_blocks * 256                    */
    int32_t dtype;                  /* SPMM_DTYPE_F16 / SPMM_DTYPE_BF16    */
} spmm_bsr_view;

typedef struct spmm_bsr_host {
    int32_t rows, cols, block_rows, block_cols, num_blocks, nnz, dtype;
    int32_t* row_ptr;
    int32_t* col_idx;
    uint16_t* values;
} spmm_bsr_host;

/* (reference: src/bsr.h:62-68, struct spmm::BSR_stats) */
typedef struct spmm_bsr_stats {
    int32_t num_blocks;
    int64_t stored_elements;
    int32_t original_nnz;
    double fill_in_ratio;
    double block_density;
} spmm_bsr_stats;

/* ---------------------------------------------------------------- host utilities */

/* (reference: src/csr.h:17-18, csr_alloc_host / csr_free_host) */
int spmm_csr_host_alloc(int32_t rows, int32_t cols, int32_t nnz, spmm_csr_host* out);
void spmm_csr_host_free(spmm_csr_host* m);

/* COO -> CSR, sorted by (row, col); duplicates are kept, as the reference does.
 * (reference: src/csr.h:20-21, csr_from_coo_host; src/csr.cu:44-72) */
int spmm_csr_from_coo_host(int32_t rows, int32_t cols, int32_t n, const int32_t* row_idx,
                           const int32_t* col_idx, const float* values, spmm_csr_host* out);

/* Uniform Bernoulli(density) CSR from mt19937(seed), bit-identical to the reference
 * generator's output. (reference: src/csr.h:23-25; src/csr.cu:74-103) */
int spmm_generate_uniform_csr(int32_t rows, int32_t cols, float density, int32_t seed,
                              spmm_csr_host* out);

/* Dense rows x cols row-major U[-1,1) from mt19937(seed).
 * (reference: src/bench/harness.cu:114-120, generate_dense_row_major) */
int spmm_generate_dense(int32_t rows, int32_t cols, int32_t seed, float* out);

/* Fast uniform CSR generator, NOT bit-compatible with spmm_generate_uniform_csr: each row
 * draws the gaps between its kept columns from a geometric(density) distribution (so the
 * expected nnz is rows * cols * density, as for the Bernoulli generator) and its values
 * from U[-1,1), both from a counter-based stream keyed by (seed, row). Columns are strictly
 * increasing in each row. The output depends on (rows, cols, density, seed) only, not on
 * `threads` (0 = all hardware threads). No counterpart in the reference: it exists to make
 * config-5-sized inputs in well under a second instead of scanning rows*cols words. */
int spmm_generate_uniform_csr_fast(int32_t rows, int32_t cols, float density, int64_t seed,
                                   int32_t threads, spmm_csr_host* out);

/* Rows [row_begin, row_end) of a host CSR, row_ptr rebased to 0.
 * (reference: src/csr.h:27-30, csr_row_slice_host; src/csr.cu:105-123) */
int spmm_csr_row_slice_host(const spmm_csr_view* m, int32_t row_begin, int32_t row_end,
                            spmm_csr_host* out);

/* Binary CSR file: int32 rows, cols, nnz; row_ptr; col_idx; float values (little endian).
 * (reference: src/csr.h:32-35; src/csr.cu:125-150) */
int spmm_csr_read_binary(const char* path, spmm_csr_host* out);
int spmm_csr_write_binary(const spmm_csr_view* m, const char* path);

/* Structural check of a host CSR (row_ptr[0]==0, monotone, row_ptr[rows]==nnz,
 * 0 <= col < cols). Returns SPMM_OK or SPMM_ERR_INVALID_ARG; *bad_row gets the first
 * offending row (or -1). Not in the reference (it trusts its inputs). */
int spmm_csr_validate_host(const spmm_csr_view* m, int32_t* bad_row);

/* CSR -> BSR-16 on the host, bit-identical to the reference conversion (FP16: RN-even;
 * BF16: RN-even). (reference: src/bsr.h:71-73, bsr_from_csr_host; src/bsr.cu:30-109) */
int spmm_csr_to_bsr16_host(const spmm_csr_view* A, int32_t dtype, spmm_bsr_host* out);
void spmm_bsr_host_free(spmm_bsr_host* b);

/* (reference: src/bsr.h:79-80, bsr_compute_stats; src/bsr.cu:149-162) */
int spmm_bsr_compute_stats(const spmm_bsr_view* b, spmm_bsr_stats* out);

/* CSR -> BSR-16 on the GPU, bit-identical to spmm_csr_to_bsr16_host (the reference's
 * bsr_from_csr_host, src/bsr.cu:30-109, which runs on the host). Device pointers, two steps:
 *   count: fills d_bsr_row_ptr (block_rows + 1 ints) and returns *num_blocks (synchronises
 *          `stream`); with num_blocks the fill-in ratio is num_blocks * 256 / nnz.
 *   fill : writes d_col_idx (num_blocks ints) and d_values (num_blocks * 256 16-bit values,
 *          4-byte aligned).
 * Needs columns sorted within each row and K <= 1,048,576 (SPMM_ERR_UNSUPPORTED otherwise:
 * use the host conversion); an index outside [0, K) gives SPMM_ERR_BAD_INDEX.
 * (replaces the host-side conversion the reference runs twice per hybrid run,
 *  src/spmm_hybrid.cu:38,78) */
int spmm_csr_to_bsr16_device_count(const spmm_csr_view* dA, int32_t* d_bsr_row_ptr, int32_t* num_blocks,
                                   void* stream);
int spmm_csr_to_bsr16_device_fill(const spmm_csr_view* dA, const int32_t* d_bsr_row_ptr, int32_t* d_col_idx,
                                  uint16_t* d_values, int32_t dtype, void* stream);

/* nnz-balanced row partition into G ranges: out[0..G], out[g]..out[g+1] is range g.
 * Bit-identical to the reference's partition. (reference: src/spmm_multigpu.cu:26-40) */
int spmm_nnz_balanced_bounds(const int32_t* row_ptr, int32_t rows, int64_t nnz, int32_t G,
                             int32_t* out);

/* ---------------------------------------------------------------- device compute */

/* CSR algorithms (all compute the same product; they differ in work distribution). */
#define SPMM_CSR_AUTO 0     /* = SPMM_CSR_MERGE                                            */
#define SPMM_CSR_ROWWARP 1  /* one warp per row, vectorised B-row loads, no row splitting  */
#define SPMM_CSR_MERGE 2    /* nnz-balanced merge-path chunks; long rows split + fix-up   */

/* Tuning knobs; zero fields take the library default. chunk = merge-path items per warp
 * (a multiple of 32, 64..8192); it also sets the long-row threshold. col_pass = width of a
 * column slab (the grid walks N slab by slab so a slab's B columns stay in L2): 0 = auto,
 * else 32/64/128/256. b_policy: 0 = plain non-coherent B loads (default; measured fastest
 * on B200 in an interleaved A/B over configs 1, 2, 4, 5), 1 = with an L2 evict-last hint,
 * 2 = evict-last and no L1 allocation. k_phases (SPMM_CSR_ROWWARP only; 0 = auto): cut
 * A's columns into this many equal ranges and run one launch per range in order, each
 * continuing every C element's FMA chain from the value the previous launch left in C, so
 * only 1/k_phases of B has to stay L2-resident at a time (1..8; direct calls take 0 as 1,
 * plans choose). Results are bit-identical for every k_phases. */
typedef struct spmm_csr_tuning {
    int32_t chunk;
    int32_t col_pass;
    int32_t b_policy;
    int32_t k_phases;
    int32_t schedule; /* merge-path chunk scheduling: 0 = auto (static), 1 = static: warp w takes
                         chunk w, 2 = dynamic: a resident grid takes chunks from a counter */
    int32_t phase_mode; /* column phases (k_phases > 1): 0 = auto, 1 = one launch per phase,
                           2 = every phase in one launch (each warp takes its rows through the
                           phases in order, one wave of resident warps); bit-identical */
    int32_t reserved[2];
} spmm_csr_tuning;

/* C = A * B, FP32, on `stream`; A, B, C are device pointers. Asynchronous.
 * Per output element the sum runs in nonzero order with FP32 FMA (the reference's
 * semantics); a row longer than the chunk is cut at merge-path chunk boundaries and its
 * pieces are added left to right (deterministic, run to run and across streams).
 * Uses a library-owned per-device workspace (allocated on first use, grown on demand);
 * calls that use it concurrently on different streams of one device race -- use
 * spmm_csr_f32_ws for that.
 * (reference: the 7 launchers `void spmm_X(const CSR&, const float*, float*, int)`,
 *  src/kernels/spmm_baseline.h:16 ... src/kernels/spmm_tiled_v4.h:63) */
int spmm_csr_f32(const spmm_csr_view* A, const float* B, float* C, int32_t N, int32_t algo,
                 void* stream);

/* Same, with explicit tuning and a caller-owned workspace. ws_bytes must be at least
 * spmm_csr_f32_workspace_size(); the workspace must be all-zero before its first use and
 * is left all-zero by every call. ws may be NULL when the size is 0. */
int spmm_csr_f32_workspace_size(const spmm_csr_view* A, int32_t N, int32_t algo,
                                const spmm_csr_tuning* tune, size_t* bytes);
int spmm_csr_f32_ws(const spmm_csr_view* A, const float* B, float* C, int32_t N, int32_t algo,
                    const spmm_csr_tuning* tune, void* ws, size_t ws_bytes, void* stream);

/* Chunk size (merge-path items per warp) that the given call would use on the current
 * device; rows longer than it are split at multiples of it (in row + nonzero index). */
int spmm_csr_f32_chunk(const spmm_csr_view* A, int32_t N, int32_t algo,
                       const spmm_csr_tuning* tune, int32_t* chunk);

/* spmm_csr_f32 for callers that must not allocate device memory (no counterpart in the
 * reference, whose launchers need no scratch). Hosts that hand all device memory to their
 * own allocator or a fixed budget, or loops that cannot take cudaMalloc's implicit device
 * synchronisation, cannot use spmm_csr_f32, which allocates its workspace on first use.
 * This variant allocates nothing: its scratch is a 16 MiB array compiled into the library
 * (held by every GPU that loads the library until the process exits). Calls whose workspace
 * would exceed 16 MiB -- about ((M + nnz) / chunk) * 8.1 * N bytes, exactly what
 * spmm_csr_f32_workspace_size reports -- return SPMM_ERR_TOO_LARGE. The first call on a device looks
 * up the array's device address; make it before any stream capture. All calls on a device
 * share the array, so calls that overlap on the GPU race; the counters that must start at
 * zero are cleared on `stream` before each launch. Bad indices are replaced by a safe one but
 * not reported (spmm_device_error does not see this path): validate A beforehand. Same
 * results as spmm_csr_f32 with the same algo, bit for bit. Arguments are checked as
 * spmm_csr_f32 checks them (SPMM_ERR_INVALID_ARG / SPMM_ERR_MISALIGNED) before the size check
 * and before anything is queued. The array's address is looked up once per device and kept:
 * do not call this entry point after cudaDeviceReset in the same process. */
int spmm_csr_f32_noalloc(const spmm_csr_view* A, const float* B, float* C, int32_t N, int32_t algo,
                         void* stream);

/* Inspector / executor form of spmm_csr_f32 (no counterpart in the reference, whose
 * launchers re-derive everything per call). spmm_csr_plan_create reads A's device row_ptr
 * once (one small kernel, synchronises `stream`) and picks the work distribution:
 * SPMM_CSR_ROWWARP when the longest row is at most max(4 * (M + nnz) / resident warps, 256),
 * else SPMM_CSR_MERGE. With ROWWARP and tune->k_phases == 0 it also picks column phases by the
 * size of B (cols * N * 4 bytes) against the L2 and the bytes a launch gathers (nnz * N * 4):
 * 3 phases when B is 0.8x to 1.2x the L2 and the launch gathers at least 4 GB; about one phase
 * per half L2 of B when B exceeds 1.2x the L2 and the launch gathers at least 12 GB; else one.
 * It computes the phase split positions once (one pass over col_idx) and allocates the plan's
 * workspace.
 * spmm_csr_plan_execute launches only (no allocation, asynchronous); A's arrays must stay
 * valid and unchanged. Results equal spmm_csr_f32 with the chosen algo bit for bit. */
typedef struct spmm_csr_plan spmm_csr_plan;
int spmm_csr_plan_create(const spmm_csr_view* A, int32_t N, const spmm_csr_tuning* tune, void* stream,
                         spmm_csr_plan** plan);
int spmm_csr_plan_execute(const spmm_csr_plan* plan, const float* B, float* C, void* stream);
int spmm_csr_plan_info(const spmm_csr_plan* plan, int32_t* algo, int32_t* max_row, size_t* ws_bytes);
/* Number of column phases the plan runs. */
int spmm_csr_plan_k_phases(const spmm_csr_plan* plan, int32_t* k_phases);
/* Kernel launches per spmm_csr_plan_execute: one per phase, or one for all of them
 * (phase_mode 2), 0 for an empty product. */
int spmm_csr_plan_launches(const spmm_csr_plan* plan, int32_t* launches);
void spmm_csr_plan_destroy(spmm_csr_plan* plan);

/* End-to-end call on HOST buffers: copies A and B to the current device (pinned or
 * pageable host memory), computes, copies C back, synchronises `stream`. Device buffers
 * are cached by the library between calls. With SPMM_CSR_ROWWARP and at least 64 MiB to move,
 * the call is pipelined: rows in 8 nnz-balanced groups on library-owned streams, so each
 * group's (col, val) copy, its launch and its C copy back overlap the other groups' (B first,
 * as every group reads all of it); the result is bit-identical to the unpipelined call. */
int spmm_csr_f32_host(const spmm_csr_view* hA, const float* hB, float* hC, int32_t N,
                      int32_t algo, void* stream);

/* FP32 -> FP16 / BF16 (round to nearest even), n elements, device pointers.
 * (reference: src/kernels/spmm_wmma.h:32, float_to_half) */
int spmm_convert_f32(const float* src, uint16_t* dst, int64_t n, int32_t dtype, void* stream);

/* BSR-16 x dense 16-bit B (same dtype as the blocks) -> FP32 C, on the tensor cores
 * (tcgen05, TMEM accumulators). Device pointers. Asynchronous.
 * (reference: src/kernels/spmm_wmma.h:39, spmm_wmma) */
int spmm_bsr16(const spmm_bsr_view* A, const void* B16, float* C, int32_t N, void* stream);

/* Inspector / executor form of spmm_bsr16 (no counterpart in the reference). Plan creation
 * (synchronises `stream`) merges, once, the block-column lists of every group of block-rows a
 * tensor-core CTA handles and stores the result as a fixed-stride schedule in device memory
 * (at most 256 MiB; larger schedules, or operands the tensor-core path does not take, leave the
 * plan on the per-call path). Execution then skips the row-pointer and column-list reads and the
 * merge, one dependent memory round trip and a serial loop fewer per CTA. A's arrays must stay
 * valid and unchanged; B16 and C may change per call. Same results as spmm_bsr16. */
typedef struct spmm_bsr_plan spmm_bsr_plan;
int spmm_bsr16_plan_create(const spmm_bsr_view* A, int32_t N, void* stream, spmm_bsr_plan** plan);
int spmm_bsr16_plan_execute(const spmm_bsr_plan* plan, const void* B16, float* C, void* stream);
/* Block-rows per CTA (0 = not on the tensor-core path), schedule steps of the longest group,
 * schedule bytes (0 = no schedule). */
int spmm_bsr16_plan_info(const spmm_bsr_plan* plan, int32_t* group, int32_t* max_steps,
                         size_t* schedule_bytes);
/* Block stride of the plan's grouped A copies (0: one copy per block). With stride S, a step whose
 * G blocks sit at p, p + S, ..., p + (G-1) S in the value array (block-diagonal, evenly filled
 * bands) loads them in one TMA copy instead of G. */
int spmm_bsr16_plan_a_stride(const spmm_bsr_plan* plan, int32_t* a_stride);
void spmm_bsr16_plan_destroy(spmm_bsr_plan* plan);

/* BSR-16 path variants for measurement: 0 = auto, 1 = tcgen05, 2 = CUDA-core fallback. */
int spmm_bsr16_algo(const spmm_bsr_view* A, const void* B16, float* C, int32_t N, int32_t algo,
                    void* stream);

/* First error recorded by a kernel on `device` since the last clear (SPMM_OK if none):
 * bad index, device wait timeout. Synchronises the device. *detail gets the offending
 * index / site. clear != 0 resets the record. */
int spmm_device_error(int32_t device, int32_t* code, int64_t* detail, int32_t clear);

/* ---------------------------------------------------------------- hybrid dispatch */

#define SPMM_BACKEND_CSR 0 /* CUDA-core CSR (the reference's Backend::CSR_TILED)   */
#define SPMM_BACKEND_TC 1  /* BSR-16 tensor cores (the reference's TENSOR_WMMA)     */

/* (reference: src/spmm_hybrid.h:33-40, struct HybridPlan) */
typedef struct spmm_hybrid_plan {
    int32_t backend;
    double fill_in_ratio;
    double block_density;
    float threshold;
    int32_t n_aligned;
    const char* reason; /* static string */
} spmm_hybrid_plan;

/* Default fill-in threshold: 6.0, the CSR / tensor-core crossover measured on B200 by
 * sparse-matrix-multiplication_b200/sweep.py (the reference's T4 default is 2.0). */
float spmm_hybrid_default_threshold(void);

/* TC iff N % 16 == 0 && N > 0 && fill_in <= threshold. threshold <= 0 selects the default.
 * (reference: src/spmm_hybrid.h:48, hybrid_choose; src/spmm_hybrid.cu:32-56) */
int spmm_hybrid_choose(const spmm_csr_view* hA, int32_t N, float threshold,
                       spmm_hybrid_plan* out);

/* (reference: src/spmm_hybrid.h:51, backend_name) */
const char* spmm_backend_name(int32_t backend);

/* Host A/B/C; warmup + iters launches on the current device; *ms = median kernel time.
 * (reference: src/spmm_hybrid.h:62-64, spmm_hybrid_run; src/spmm_hybrid.cu:58-125) */
int spmm_hybrid_run(const spmm_hybrid_plan* plan, const spmm_csr_view* hA, const float* hB,
                    float* hC, int32_t N, int32_t warmup, int32_t iters, float* ms);

/* ---------------------------------------------------------------- multi-GPU */

/* (reference: src/spmm_multigpu.h:32, gpu_count) */
int spmm_gpu_count(void);

/* nnz-balanced row split over num_gpus devices (clamped to the visible count), one host thread
 * per device running the per-rank path below (spmm_rank_run: each device copies its rows of A
 * and 1/num_gpus of B's rows, an NCCL all-gather over NVLink completes B on every device, the
 * rows of C come back into hC, row-disjoint). *time_ms = max over devices of the median kernel
 * time on the resident operands (the reference's semantics); *bcast_ms = the time of the
 * all-gather of B alone (max over devices). rows_out / nnz_out (may be NULL) receive
 * num_gpus entries.
 * (reference: src/spmm_multigpu.h:49-52, spmm_multigpu; src/spmm_multigpu.cu:44-120) */
int spmm_multigpu_run(const spmm_csr_view* hA, const float* hB, float* hC, int32_t N,
                      int32_t num_gpus, int32_t warmup, int32_t iters, float* time_ms,
                      int32_t* used_gpus, int32_t* rows_out, int32_t* nnz_out, float* bcast_ms);

/* ---------------------------------------------------------------- multi-GPU, one process per GPU
 *
 * The same row split for programs that run one process (or one long-lived host thread) per
 * GPU, as torchrun and MPI jobs do. Every rank holds the whole host A and B and receives its
 * own rows of C; the ranks exchange B over NVLink through an NCCL communicator, so B crosses
 * the host links once in total instead of once per GPU. (reference: the per-GPU worker of
 * src/spmm_multigpu.cu:66-109, which spmm_multigpu_run above runs as threads of one call) */

#define SPMM_COMM_ID_BYTES 128
typedef struct spmm_comm spmm_comm;

/* A new communicator id (the bytes of an ncclUniqueId). Make it on one rank and hand the same
 * bytes to every rank over any host channel (a TCP store, MPI, a shared file). */
int spmm_comm_unique_id(uint8_t id[SPMM_COMM_ID_BYTES]);

/* Join communicator `id` as `rank` of `world`, on the current device. Every rank calls it; it
 * returns once all have joined, or SPMM_ERR_TIMEOUT after timeout_ms (<= 0: 300 s) when a rank
 * never joins (the half-made communicator is then aborted). The same timeout bounds every
 * later host wait on this communicator; a communicator that timed out is aborted and every
 * further call on it returns SPMM_ERR_NCCL. */
int spmm_comm_init(const uint8_t id[SPMM_COMM_ID_BYTES], int32_t world, int32_t rank, int32_t timeout_ms,
                   spmm_comm** out);

/* Wrap an NCCL communicator the caller already owns (an ncclComm_t passed as void*); its size,
 * rank and device are read from it. spmm_comm_destroy then frees the wrapper only. */
int spmm_comm_wrap(void* nccl_comm, int32_t timeout_ms, spmm_comm** out);
int spmm_comm_info(const spmm_comm* comm, int32_t* world, int32_t* rank, int32_t* device);
void spmm_comm_destroy(spmm_comm* comm);

/* This rank's share of C = A * B under the reference's row split: rows [bounds[rank],
 * bounds[rank + 1]) of spmm_nnz_balanced_bounds(A, world) (reference:
 * src/spmm_multigpu.cu:26-40, 60-64). hA is the WHOLE host matrix, the same on every rank;
 * comm = NULL is a world of one on the current device (no NCCL). Allocates the rank's device
 * buffers (its rows of A, all of B, its rows of C), copies its rows of A once and inspects
 * them (spmm_csr_plan_create). Local: no collective. Synchronises `stream`. */
typedef struct spmm_rank_plan spmm_rank_plan;
int spmm_rank_plan_create(spmm_comm* comm, const spmm_csr_view* hA, int32_t N, void* stream, spmm_rank_plan** out);

/* The rank's rows [row_begin, row_end) and nonzeros; the rows of B it copies from the host
 * itself, [b_row_begin, b_row_end) (B's rows in `world` shares of K * r / world); the CSR
 * algorithm its plan picked and the kernel launches one spmm_rank_execute makes. Any pointer
 * may be NULL. */
int spmm_rank_plan_info(const spmm_rank_plan* plan, int32_t* row_begin, int32_t* row_end, int32_t* nnz,
                        int32_t* b_row_begin, int32_t* b_row_end, int32_t* algo, int32_t* launches);

/* One end-to-end multiply on host buffers; collective (every rank calls it, in the same order):
 * the rank's rows of A and its share of B's rows go host -> device; the ranks all-gather B over
 * NVLink (NCCL; ncclAllGather for equal shares, grouped send/recv otherwise); the kernels run on
 * the rank's rows; its rows of C come back into hC_rows ((row_end - row_begin) x N row-major: a
 * caller that holds the whole M x N C passes C + row_begin * N). hA must be the matrix the plan
 * was made for: its values may change between calls, its structure may not (a row_ptr that
 * differs at the rank's boundaries is refused). hB is the whole K x N B.
 * With SPMM_B200_B_PIECES=P (2..16) in the environment when the plan is made, the share is copied
 * in P pieces and each piece goes to the other ranks (grouped send/recv) as soon as it has landed.
 * Pipelined (one-warp-per-row plans): the all-gather overlaps the copy of A's rows, each of 8
 * nnz-balanced row groups is launched once its rows have landed, and each group's rows of C go
 * back while later groups compute. Bit-identical to spmm_rank_execute and to spmm_csr_f32 with
 * the plan's algorithm on the rank's rows. Returns once hC_rows holds the result (the wait is
 * bounded by the communicator's timeout). Pinned host buffers make the copies asynchronous. */
int spmm_rank_run(spmm_rank_plan* plan, const spmm_csr_view* hA, const float* hB, float* hC_rows, void* stream);

/* spmm_rank_run without the wait, for a stream of multiplies: issues the same copies, exchange,
 * kernels and copies back, and returns. The next run or submit on the plan overlaps this one where
 * the buffers allow: its copies in wait only for this run's kernels, its kernels for this run's
 * copies back, so one run's copies back can share the host links with the next run's copies in.
 * hA, hB and hC_rows must stay valid and unchanged, and hC_rows is not written in full, until
 * spmm_rank_wait returns (give consecutive submits different hC_rows). Collective, like
 * spmm_rank_run. (no counterpart in the reference, whose multi-GPU call is synchronous) */
int spmm_rank_submit(spmm_rank_plan* plan, const spmm_csr_view* hA, const float* hB, float* hC_rows, void* stream);

/* Waits (bounded by the communicator's timeout) until the last run issued on the plan has put its
 * rows of C on the host, and makes `stream` wait for it too. */
int spmm_rank_wait(spmm_rank_plan* plan, void* stream);

/* The kernels alone, on the device-resident operands the last spmm_rank_run left behind (the
 * rank's rows of A and the gathered B), into the plan's device C. Asynchronous, not collective;
 * on the device it starts after the last run's copies back, whatever the stream. */
int spmm_rank_execute(spmm_rank_plan* plan, void* stream);

/* The all-gather of B alone (device to device over NVLink, from the shares already on every
 * rank's device). Collective, asynchronous on `stream`, after the last run's copies back. */
int spmm_rank_gather_b(spmm_rank_plan* plan, void* stream);

/* The plan's device buffers: B (K x N, gathered) and the rank's rows of C. */
int spmm_rank_plan_buffers(const spmm_rank_plan* plan, float** dB, float** dC);
/* Waits for the plan's queued work (bounded: past the communicator's timeout it is aborted, so
 * that a run waiting on a rank that is gone ends) and frees the plan. */
void spmm_rank_plan_destroy(spmm_rank_plan* plan);

/* Managed-memory single-GPU path: A, B, C in cudaMallocManaged memory, prefetched to the
 * current device. *ms = median kernel time.
 * (reference: src/spmm_multigpu.h:57-58, spmm_unified; src/spmm_multigpu.cu:122-182) */
int spmm_unified_run(const spmm_csr_view* hA, const float* hB, float* hC, int32_t N,
                     int32_t warmup, int32_t iters, float* ms);

/* spmm_unified_run for matrices larger than the device (no counterpart in the reference, whose
 * unified path prefetches everything and leaves the rest to demand paging). device_budget =
 * bytes of device memory to plan with (0 = 90 % of what is free now). When B does not fit
 * beside A, C and the split positions, A's columns are cut into phases (at most 32; *phases_used
 * reports the count, 1 = no phases): per phase, B's rows of that column range are prefetched to
 * the device, the phase's kernel continues every C element's FMA chain, and the rows are
 * prefetched back to the host before the next phase. Results equal the one-warp-per-row kernel
 * (the reference's sequential chain per element) bit for bit; *ms is the median time of a whole
 * pass, migrations included. */
int spmm_unified_run_ex(const spmm_csr_view* hA, const float* hB, float* hC, int32_t N,
                        size_t device_budget, int32_t warmup, int32_t iters, float* ms,
                        int32_t* phases_used);

#ifdef __cplusplus
}
#endif

#endif /* SPMM_C_H */
