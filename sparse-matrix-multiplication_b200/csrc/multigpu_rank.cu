// The multi-GPU row split for programs that run one process (or one long-lived host thread) per
// GPU: a communicator over NCCL and a per-rank plan that holds the rank's share of the product.
//
// The reference runs its split inside one call with one host thread per GPU
// (src/spmm_multigpu.cu:44-120): rows cut by nnz_balanced_bounds (:26-40), every GPU gets its
// slice of A and the whole of B from the host, runs tiled_v3 and copies its rows of C back
// (:66-109). Here each rank does the same for its own rows, with three differences of design:
//   * B crosses the host links once in total: every rank copies an equal share of B's rows
//     and the ranks all-gather the rest over NVLink (NCCL), while A's rows are still arriving;
//   * the rank's rows run in nnz-balanced row groups, each launched as soon as its rows have
//     landed, and each group's rows of C go back while later groups compute;
//   * every host wait is bounded (a rank that never joins or stops answering gives
//     SPMM_ERR_TIMEOUT and the communicator is aborted, instead of a process that hangs).

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <new>
#include <thread>
#include <vector>

#include "common.cuh"
#include "nccl_api.cuh"

struct spmm_comm {
    ncclComm_t comm = nullptr;
    int world = 1;
    int rank = 0;
    int device = 0;
    bool owned = false;   // made by spmm_comm_init (destroyed with the wrapper)
    bool broken = false;  // aborted after a timeout or an asynchronous NCCL error
    int timeout_ms = 300000;
};

namespace spmm_b200 {
namespace {

constexpr int kRankGroups = 8;  // row groups of one rank's pipelined run
// Pieces of a rank's B share in an end-to-end run (world > 1). One piece: the share crosses the
// host link, then one ncclAllGather (or grouped send/recv for unequal shares) completes B. More
// pieces: each piece is sent to every other rank (grouped send/recv) as soon as it has landed,
// while the next piece is still being copied.
constexpr int kBPieces = 1;

// Pieces of B's share per end-to-end run: SPMM_B200_B_PIECES (1..16) when set, else kBPieces.
int b_pieces_setting() {
    const char* e = std::getenv("SPMM_B200_B_PIECES");
    if (e && e[0]) {
        const int v = std::atoi(e);
        if (v >= 1 && v <= 16) return v;
    }
    return kBPieces;
}

using Clock = std::chrono::steady_clock;

double elapsed_ms(Clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
}

// Let the host breathe between polls once a wait has lasted a while.
void backoff(int polls) {
    if (polls < 2000) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(50));
}

void abort_comm(spmm_comm* c) {
    if (c && c->comm && !c->broken) {
        nccl().comm_abort(c->comm);
        c->broken = true;
    }
}

// Wait for a non-blocking communicator to leave ncclInProgress (an init or a group that is
// still being enqueued). Bounded by the communicator's timeout; aborts it when that runs out.
int wait_comm_ready(spmm_comm* c) {
    const auto t0 = Clock::now();
    for (int polls = 0;; ++polls) {
        ncclResult_t st = ncclSuccess;
        if (nccl().comm_get_async_error(c->comm, &st) != ncclSuccess) st = ncclInternalError;
        if (st == ncclSuccess) return SPMM_OK;
        if (st != ncclInProgress) {
            abort_comm(c);
            return SPMM_ERR_NCCL;
        }
        if (elapsed_ms(t0) > c->timeout_ms) {
            abort_comm(c);
            return SPMM_ERR_TIMEOUT;
        }
        backoff(polls);
    }
}

// Wait for `ev` on the host. While it is pending, the communicator (if any) is checked for
// asynchronous errors; past the timeout the communicator is aborted (NCCL's kernels then
// leave) and SPMM_ERR_TIMEOUT is returned.
int wait_event(cudaEvent_t ev, spmm_comm* c, int timeout_ms) {
    const auto t0 = Clock::now();
    for (int polls = 0;; ++polls) {
        const cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return SPMM_OK;
        if (e != cudaErrorNotReady) {
            note_cuda_error(e, "cudaEventQuery", __FILE__, __LINE__);
            return SPMM_ERR_CUDA;
        }
        if (c && c->comm) {
            ncclResult_t st = ncclSuccess;
            nccl().comm_get_async_error(c->comm, &st);
            if (st != ncclSuccess && st != ncclInProgress) {
                abort_comm(c);
                return SPMM_ERR_NCCL;
            }
        }
        if (elapsed_ms(t0) > timeout_ms) {
            abort_comm(c);
            return SPMM_ERR_TIMEOUT;
        }
        backoff(polls);
    }
}

__global__ void rebase_row_ptr_kernel(int* __restrict__ rp, int n, int base) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) rp[i] -= base;
}

}  // namespace
}  // namespace spmm_b200

using namespace spmm_b200;

struct spmm_rank_plan {
    spmm_comm* comm = nullptr;  // null: a world of one
    int world = 1, rank = 0, device = 0;
    int32_t M = 0, K = 0, N = 0, nnz_all = 0;
    int32_t r0 = 0, r1 = 0;  // this rank's rows of A and C
    int32_t p0 = 0, p1 = 0;  // their positions in the whole A
    std::vector<int32_t> b_bounds;  // world + 1: the rows of B each rank uploads
    std::vector<int32_t> groups;    // row groups inside the rank (relative rows), pipelined runs
    std::vector<int32_t> group_pos; // their first positions (relative), groups.size() entries
    int* d_rp = nullptr;
    int* d_ci = nullptr;
    float* d_v = nullptr;
    float* d_B = nullptr;
    float* d_C = nullptr;
    spmm_csr_view dview{};
    spmm_csr_plan* cplan = nullptr;
    int32_t algo = SPMM_CSR_ROWWARP;
    int32_t launches = 1;  // kernel launches of one spmm_rank_execute
    int32_t b_pieces = 1;  // pieces of the B share copied and exchanged one after another
    bool pipelined = false;
    cudaStream_t s_in = nullptr, s_comm = nullptr, s_k = nullptr, s_out = nullptr;
    // [0] start, [1] B share landed, [2] B gathered, [3 + g] rows of group g landed,
    // [3 + G + g] group g computed, [3 + 2G] end, [4 + 2G + j] piece j of the B share landed.
    std::vector<cudaEvent_t> ev;

    // Cross-step ordering of submitted runs: a run's copies into the device buffers wait for the
    // previous run's kernels (kdone), its kernels for the previous run's copies back (end).
    cudaEvent_t kdone = nullptr;
    bool submitted = false;  // a run has been issued since the plan was made
    bool pending = false;    // the last run was submitted and no host wait has seen it end

    int rows() const { return r1 - r0; }
    int nnz() const { return p1 - p0; }
    int timeout_ms() const { return comm ? comm->timeout_ms : 300000; }
    int groups_count() const { return static_cast<int>(groups.size()) - 1; }
    cudaEvent_t end_event() const { return ev[3 + 2 * groups_count()]; }
};

namespace spmm_b200 {
namespace {

// Waits for everything queued on the plan's streams. Each wait is bounded by the plan's timeout:
// a collective that waits on a rank that is gone is ended by aborting the communicator (NCCL's
// kernels then leave), so the synchronisations that follow cannot wait for ever.
int drain(spmm_rank_plan* p) {
    int rc = SPMM_OK;
    for (cudaStream_t x : {p->s_in, p->s_comm, p->s_k, p->s_out}) {
        if (!x) continue;
        cudaEvent_t e = nullptr;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess) {
            int r = cudaEventRecord(e, x) == cudaSuccess ? wait_event(e, p->comm, p->timeout_ms()) : SPMM_ERR_CUDA;
            if (rc == SPMM_OK) rc = r;
            cudaEventDestroy(e);
        } else {
            cudaGetLastError();
        }
    }
    for (cudaStream_t x : {p->s_in, p->s_comm, p->s_k, p->s_out})
        if (x) cudaStreamSynchronize(x);
    return rc;
}

void release(spmm_rank_plan* p) {
    if (!p) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    drain(p);
    if (p->cplan) spmm_csr_plan_destroy(p->cplan);
    for (cudaEvent_t e : p->ev)
        if (e) cudaEventDestroy(e);
    if (p->kdone) cudaEventDestroy(p->kdone);
    for (cudaStream_t s : {p->s_in, p->s_comm, p->s_k, p->s_out})
        if (s) cudaStreamDestroy(s);
    cudaFree(p->d_rp);
    cudaFree(p->d_ci);
    cudaFree(p->d_v);
    cudaFree(p->d_B);
    cudaFree(p->d_C);
    cudaSetDevice(prev);
    delete p;
}

bool host_view_ok(const spmm_csr_view* A) {
    return A && A->rows >= 0 && A->cols >= 0 && A->nnz >= 0 && A->row_ptr &&
           (A->nnz == 0 || (A->col_idx && A->values));
}

// Every rank's share of B's rows: K * r / world (shares differ by at most one row).
void b_shares(int32_t K, int world, std::vector<int32_t>* out) {
    out->resize(world + 1);
    for (int r = 0; r <= world; ++r) (*out)[r] = static_cast<int32_t>(static_cast<int64_t>(K) * r / world);
}

// The all-gather of B on `s`: in place, the rank's share already at its rows. Equal shares
// use ncclAllGather; unequal ones a group of point-to-point copies (an all-gather-v).
int gather_b_issue(spmm_rank_plan* p, cudaStream_t s) {
    if (p->world == 1) return SPMM_OK;
    spmm_comm* c = p->comm;
    if (c->broken) return SPMM_ERR_NCCL;
    const NcclApi& nc = nccl();
    const size_t N = static_cast<size_t>(p->N);
    const int32_t* bb = p->b_bounds.data();
    const size_t share = static_cast<size_t>(bb[1] - bb[0]);
    bool equal = true;
    for (int r = 0; r < p->world; ++r) equal = equal && static_cast<size_t>(bb[r + 1] - bb[r]) == share;
    NvtxRange range("spmm_rank: all-gather B");
    if (nc.group_start() != ncclSuccess) return SPMM_ERR_NCCL;
    bool ok = true;
    if (equal) {
        if (share * N != 0) {
            float* mine = p->d_B + static_cast<size_t>(bb[p->rank]) * N;
            ok = nc.all_gather(mine, p->d_B, share * N, ncclFloat, c->comm, s) == ncclSuccess;
        }
    } else {
        const float* mine = p->d_B + static_cast<size_t>(bb[p->rank]) * N;
        const size_t my_count = static_cast<size_t>(bb[p->rank + 1] - bb[p->rank]) * N;
        for (int r = 0; r < p->world && ok; ++r) {
            if (r == p->rank) continue;
            const size_t their = static_cast<size_t>(bb[r + 1] - bb[r]) * N;
            if (my_count) ok = nc.send(mine, my_count, ncclFloat, r, c->comm, s) == ncclSuccess;
            if (ok && their)
                ok = nc.recv(p->d_B + static_cast<size_t>(bb[r]) * N, their, ncclFloat, r, c->comm, s) == ncclSuccess;
        }
    }
    const ncclResult_t end = nc.group_end();
    if (!ok || (end != ncclSuccess && end != ncclInProgress)) {
        abort_comm(c);
        return SPMM_ERR_NCCL;
    }
    return end == ncclInProgress ? wait_comm_ready(c) : SPMM_OK;
}

// Rows [lo, hi) of piece j of rank r's share of B (the share cut into P near-equal pieces).
void share_piece(const spmm_rank_plan* p, int r, int j, int P, int32_t* lo, int32_t* hi) {
    const int64_t b0 = p->b_bounds[r], len = p->b_bounds[r + 1] - b0;
    *lo = static_cast<int32_t>(b0 + len * j / P);
    *hi = static_cast<int32_t>(b0 + len * (j + 1) / P);
}

// Piece j of every rank's share to every other rank (point-to-point, grouped), on `s`: the
// exchange of a piece starts as soon as this rank's copy of it has landed, while the next
// piece is still crossing the host link.
int exchange_piece_issue(spmm_rank_plan* p, int j, int P, cudaStream_t s) {
    spmm_comm* c = p->comm;
    if (c->broken) return SPMM_ERR_NCCL;
    const NcclApi& nc = nccl();
    const size_t N = static_cast<size_t>(p->N);
    int32_t mlo = 0, mhi = 0;
    share_piece(p, p->rank, j, P, &mlo, &mhi);
    const size_t mine = static_cast<size_t>(mhi - mlo) * N;
    NvtxRange range("spmm_rank: exchange B piece");
    if (nc.group_start() != ncclSuccess) return SPMM_ERR_NCCL;
    bool ok = true;
    for (int r = 0; r < p->world && ok; ++r) {
        if (r == p->rank) continue;
        int32_t lo = 0, hi = 0;
        share_piece(p, r, j, P, &lo, &hi);
        const size_t theirs = static_cast<size_t>(hi - lo) * N;
        if (mine) ok = nc.send(p->d_B + static_cast<size_t>(mlo) * N, mine, ncclFloat, r, c->comm, s) == ncclSuccess;
        if (ok && theirs)
            ok = nc.recv(p->d_B + static_cast<size_t>(lo) * N, theirs, ncclFloat, r, c->comm, s) == ncclSuccess;
    }
    const ncclResult_t end = nc.group_end();
    if (!ok || (end != ncclSuccess && end != ncclInProgress)) {
        abort_comm(c);
        return SPMM_ERR_NCCL;
    }
    return end == ncclInProgress ? wait_comm_ready(c) : SPMM_OK;
}

// Makes `s` wait on the device for the last run's copies back when no host wait has seen them end
// (a submitted run): kernels or copies issued on `s` next may overwrite what those copies read.
// Inside a stream capture the wait is an external-event node of the graph.
int order_after_last_run(spmm_rank_plan* p, cudaStream_t s) {
    if (!p->pending) return SPMM_OK;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    SPMM_CUDA_TRY(cudaStreamIsCapturing(s, &cs));
    const unsigned flags = cs == cudaStreamCaptureStatusActive ? cudaEventWaitExternal : cudaEventWaitDefault;
    SPMM_CUDA_TRY(cudaStreamWaitEvent(s, p->end_event(), flags));
    return SPMM_OK;
}

int check_plan_device(const spmm_rank_plan* p) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return SPMM_ERR_UNSUPPORTED;
    }
    return dev == p->device ? SPMM_OK : SPMM_ERR_INVALID_ARG;
}

// Issues one end-to-end run. `join`: the caller's stream waits for the run's last copy back
// (spmm_rank_run); without it (spmm_rank_submit) the caller's stream is only the run's start,
// so that the next submitted run's copies in can overlap this run's copies back.
int run_issue(spmm_rank_plan* p, const spmm_csr_view* hA, const float* hB, float* hC, cudaStream_t s,
              DeviceState* st, bool join) {
    const size_t N = static_cast<size_t>(p->N);
    const int G = p->groups_count();
    cudaEvent_t* ev = p->ev.data();
    const bool prev = p->submitted;
    SPMM_CUDA_TRY(cudaEventRecord(ev[0], s));
    for (cudaStream_t x : {p->s_in, p->s_comm, p->s_k, p->s_out}) SPMM_CUDA_TRY(cudaStreamWaitEvent(x, ev[0], 0));
    // The device buffers this run overwrites are still read by the previous run's kernels
    // (A's rows, B) and copies back (C): wait for those, not for the whole previous run.
    if (prev) {
        SPMM_CUDA_TRY(cudaStreamWaitEvent(p->s_in, p->kdone, 0));
        SPMM_CUDA_TRY(cudaStreamWaitEvent(p->s_comm, p->kdone, 0));
        SPMM_CUDA_TRY(cudaStreamWaitEvent(p->s_k, p->end_event(), 0));
    }
    p->submitted = true;
    const int P = p->b_pieces;
    cudaEvent_t* ev_piece = ev + 4 + 2 * G;
    {
        // B first, in P pieces: the exchange of B can start once every rank's piece has landed,
        // and with P > 1 the exchange of one piece overlaps the host copy of the next.
        NvtxRange range("spmm_rank: B share H2D");
        for (int j = 0; j < P; ++j) {
            int32_t lo = 0, hi = 0;
            share_piece(p, p->rank, j, P, &lo, &hi);
            if (static_cast<size_t>(hi - lo) * N != 0)
                SPMM_CUDA_TRY(cudaMemcpyAsync(p->d_B + static_cast<size_t>(lo) * N, hB + static_cast<size_t>(lo) * N,
                                              sizeof(float) * static_cast<size_t>(hi - lo) * N, cudaMemcpyHostToDevice,
                                              p->s_in));
            SPMM_CUDA_TRY(cudaEventRecord(ev_piece[j], p->s_in));
        }
        SPMM_CUDA_TRY(cudaEventRecord(ev[1], p->s_in));
    }
    if (p->world > 1) {
        if (P == 1) {
            SPMM_CUDA_TRY(cudaStreamWaitEvent(p->s_comm, ev[1], 0));
            SPMM_TRY(gather_b_issue(p, p->s_comm));
        } else {
            for (int j = 0; j < P; ++j) {
                SPMM_CUDA_TRY(cudaStreamWaitEvent(p->s_comm, ev_piece[j], 0));
                SPMM_TRY(exchange_piece_issue(p, j, P, p->s_comm));
            }
        }
        SPMM_CUDA_TRY(cudaEventRecord(ev[2], p->s_comm));
    } else {
        SPMM_CUDA_TRY(cudaEventRecord(ev[2], p->s_in));
    }
    {
        // A's rows of this rank: row_ptr (rebased to the rank's first position), then each
        // group's (column, value) pairs.
        NvtxRange range("spmm_rank: A rows H2D");
        const int rows = p->rows();
        SPMM_CUDA_TRY(cudaMemcpyAsync(p->d_rp, hA->row_ptr + p->r0, sizeof(int) * (static_cast<size_t>(rows) + 1),
                                      cudaMemcpyHostToDevice, p->s_in));
        if (p->p0 != 0) {
            const int blocks = std::min((rows + 1 + 255) / 256, st->sm_count * 4);
            rebase_row_ptr_kernel<<<std::max(blocks, 1), 256, 0, p->s_in>>>(p->d_rp, rows + 1, p->p0);
            SPMM_CUDA_TRY(cudaGetLastError());
        }
        for (int g = 0; g < G; ++g) {
            const size_t q0 = static_cast<size_t>(p->group_pos[g]), q1 = static_cast<size_t>(p->group_pos[g + 1]);
            if (q1 > q0) {
                SPMM_CUDA_TRY(cudaMemcpyAsync(p->d_ci + q0, hA->col_idx + p->p0 + q0, sizeof(int) * (q1 - q0),
                                              cudaMemcpyHostToDevice, p->s_in));
                SPMM_CUDA_TRY(cudaMemcpyAsync(p->d_v + q0, hA->values + p->p0 + q0, sizeof(float) * (q1 - q0),
                                              cudaMemcpyHostToDevice, p->s_in));
            }
            SPMM_CUDA_TRY(cudaEventRecord(ev[3 + g], p->s_in));
        }
    }
    {
        NvtxRange range("spmm_rank: launches");
        SPMM_CUDA_TRY(cudaStreamWaitEvent(p->s_k, ev[2], 0));
        for (int g = 0; g < G; ++g) {
            SPMM_CUDA_TRY(cudaStreamWaitEvent(p->s_k, ev[3 + g], 0));
            if (p->pipelined) {
                const int g0 = p->groups[g], g1 = p->groups[g + 1];
                if (g1 > g0) {
                    // Rows g0..g1 as their own view; row_ptr keeps the rank's positions.
                    spmm_csr_view part = p->dview;
                    part.rows = g1 - g0;
                    part.row_ptr = p->d_rp + g0;
                    SPMM_TRY(csr_f32_launch(&part, p->d_B, p->d_C + static_cast<size_t>(g0) * N, p->N,
                                            SPMM_CSR_ROWWARP, nullptr, nullptr, 0, p->s_k, st));
                }
            } else if (g == G - 1) {
                SPMM_TRY(spmm_csr_plan_execute(p->cplan, p->d_B, p->d_C, p->s_k));
            }
            SPMM_CUDA_TRY(cudaEventRecord(ev[3 + G + g], p->s_k));
        }
        SPMM_CUDA_TRY(cudaEventRecord(p->kdone, p->s_k));
    }
    {
        NvtxRange range("spmm_rank: C rows D2H");
        for (int g = 0; g < G; ++g) {
            SPMM_CUDA_TRY(cudaStreamWaitEvent(p->s_out, ev[3 + G + g], 0));
            const int g0 = p->groups[g], g1 = p->groups[g + 1];
            if (static_cast<size_t>(g1 - g0) * N != 0)
                SPMM_CUDA_TRY(cudaMemcpyAsync(hC + static_cast<size_t>(g0) * N, p->d_C + static_cast<size_t>(g0) * N,
                                              sizeof(float) * static_cast<size_t>(g1 - g0) * N, cudaMemcpyDeviceToHost,
                                              p->s_out));
        }
        SPMM_CUDA_TRY(cudaEventRecord(ev[3 + 2 * G], p->s_out));
        if (join) SPMM_CUDA_TRY(cudaStreamWaitEvent(s, ev[3 + 2 * G], 0));
    }
    return SPMM_OK;
}

int check_run_args(const spmm_rank_plan* p, const spmm_csr_view* hA, const float* hB, const float* hC_rows) {
    if (!p || !host_view_ok(hA)) return SPMM_ERR_INVALID_ARG;
    if (hA->rows != p->M || hA->cols != p->K || hA->nnz != p->nnz_all || hA->row_ptr[p->r0] != p->p0 ||
        hA->row_ptr[p->r1] != p->p1)
        return SPMM_ERR_INVALID_ARG;  // not the matrix the plan was made for
    const size_t N = static_cast<size_t>(p->N);
    if ((static_cast<size_t>(p->K) * N != 0 && !hB) || (static_cast<size_t>(p->rows()) * N != 0 && !hC_rows))
        return SPMM_ERR_INVALID_ARG;
    if (p->comm && p->comm->broken) return SPMM_ERR_NCCL;
    return SPMM_OK;
}

int issue_checked(spmm_rank_plan* p, const spmm_csr_view* hA, const float* hB, float* hC_rows, void* stream,
                  bool join) {
    if (!p) return SPMM_ERR_INVALID_ARG;
    SPMM_TRY(check_plan_device(p));
    SPMM_TRY(check_run_args(p, hA, hB, hC_rows));
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    const int rc = run_issue(p, hA, hB, hC_rows, as_stream(stream), st, join);
    if (rc != SPMM_OK) drain(p);  // whatever was queued still reads the caller's host buffers
    return rc;
}

}  // namespace
}  // namespace spmm_b200

extern "C" {

int spmm_comm_unique_id(uint8_t id[SPMM_COMM_ID_BYTES]) {
    if (!id) return SPMM_ERR_INVALID_ARG;
    const NcclApi& nc = nccl();
    if (!nc.ranks_ok) return SPMM_ERR_UNSUPPORTED;
    ncclUniqueId uid;
    if (nc.get_unique_id(&uid) != ncclSuccess) return SPMM_ERR_NCCL;
    static_assert(sizeof(uid) == SPMM_COMM_ID_BYTES, "ncclUniqueId size");
    std::memcpy(id, &uid, SPMM_COMM_ID_BYTES);
    return SPMM_OK;
}

int spmm_comm_init(const uint8_t id[SPMM_COMM_ID_BYTES], int32_t world, int32_t rank, int32_t timeout_ms,
                   spmm_comm** out) {
    if (!id || !out || world < 1 || rank < 0 || rank >= world) return SPMM_ERR_INVALID_ARG;
    *out = nullptr;
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    const NcclApi& nc = nccl();
    if (!nc.ranks_ok) return SPMM_ERR_UNSUPPORTED;
    spmm_comm* c = new (std::nothrow) spmm_comm();
    if (!c) return SPMM_ERR_NO_MEMORY;
    c->world = world;
    c->rank = rank;
    c->device = st->device;
    c->owned = true;
    if (timeout_ms > 0) c->timeout_ms = timeout_ms;
    ncclUniqueId uid;
    std::memcpy(&uid, id, SPMM_COMM_ID_BYTES);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // so that a rank that never joins gives a bounded wait, not a hang
    NvtxRange range("spmm_comm_init");
    const ncclResult_t r = nc.comm_init_rank_config(&c->comm, world, uid, rank, &cfg);
    int rc = SPMM_OK;
    if (r != ncclSuccess && r != ncclInProgress) rc = SPMM_ERR_NCCL;
    else rc = wait_comm_ready(c);
    if (rc != SPMM_OK) {
        if (c->comm && !c->broken) nc.comm_abort(c->comm);
        delete c;
        return rc;
    }
    *out = c;
    return SPMM_OK;
}

int spmm_comm_wrap(void* nccl_comm, int32_t timeout_ms, spmm_comm** out) {
    if (!nccl_comm || !out) return SPMM_ERR_INVALID_ARG;
    const NcclApi& nc = nccl();
    if (!nc.ranks_ok) return SPMM_ERR_UNSUPPORTED;
    spmm_comm* c = new (std::nothrow) spmm_comm();
    if (!c) return SPMM_ERR_NO_MEMORY;
    c->comm = static_cast<ncclComm_t>(nccl_comm);
    if (nc.comm_count(c->comm, &c->world) != ncclSuccess || nc.comm_user_rank(c->comm, &c->rank) != ncclSuccess ||
        nc.comm_cu_device(c->comm, &c->device) != ncclSuccess) {
        delete c;
        return SPMM_ERR_NCCL;
    }
    if (timeout_ms > 0) c->timeout_ms = timeout_ms;
    *out = c;
    return SPMM_OK;
}

int spmm_comm_info(const spmm_comm* c, int32_t* world, int32_t* rank, int32_t* device) {
    if (!c) return SPMM_ERR_INVALID_ARG;
    if (world) *world = c->world;
    if (rank) *rank = c->rank;
    if (device) *device = c->device;
    return c->broken ? SPMM_ERR_NCCL : SPMM_OK;
}

void spmm_comm_destroy(spmm_comm* c) {
    if (!c) return;
    if (c->owned && c->comm && !c->broken) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(c->device);
        nccl().comm_destroy(c->comm);
        cudaSetDevice(prev);
    }
    delete c;
}

int spmm_rank_plan_create(spmm_comm* comm, const spmm_csr_view* hA, int32_t N, void* stream, spmm_rank_plan** out) {
    if (!out || !host_view_ok(hA) || N < 0) return SPMM_ERR_INVALID_ARG;
    *out = nullptr;
    if (hA->row_ptr[0] != 0 || hA->row_ptr[hA->rows] != hA->nnz) return SPMM_ERR_INVALID_ARG;
    DeviceState* st = nullptr;
    SPMM_TRY(current_device_state(&st));
    if (comm && (comm->broken || comm->device != st->device)) return SPMM_ERR_INVALID_ARG;
    const cudaStream_t s = as_stream(stream);
    spmm_rank_plan* p = new (std::nothrow) spmm_rank_plan();
    if (!p) return SPMM_ERR_NO_MEMORY;
    p->comm = comm;
    p->world = comm ? comm->world : 1;
    p->rank = comm ? comm->rank : 0;
    p->device = st->device;
    p->M = hA->rows;
    p->K = hA->cols;
    p->N = N;
    p->nnz_all = hA->nnz;
    int rc = SPMM_OK;
    auto fail = [&](int code) {
        release(p);
        return code;
    };
    {
        // The reference's partition (bit-identical): this rank's rows and positions.
        std::vector<int32_t> bounds(p->world + 1);
        rc = spmm_nnz_balanced_bounds(hA->row_ptr, hA->rows, hA->nnz, p->world, bounds.data());
        if (rc != SPMM_OK) return fail(rc);
        p->r0 = bounds[p->rank];
        p->r1 = bounds[p->rank + 1];
        p->p0 = hA->row_ptr[p->r0];
        p->p1 = hA->row_ptr[p->r1];
    }
    b_shares(p->K, p->world, &p->b_bounds);
    const size_t rows = static_cast<size_t>(p->rows()), nnz = static_cast<size_t>(p->nnz());
    const size_t K = static_cast<size_t>(p->K), Nz = static_cast<size_t>(N);
    if (cudaMalloc(&p->d_rp, sizeof(int) * (rows + 1)) != cudaSuccess ||
        cudaMalloc(&p->d_ci, sizeof(int) * std::max<size_t>(nnz, 1)) != cudaSuccess ||
        cudaMalloc(&p->d_v, sizeof(float) * std::max<size_t>(nnz, 1)) != cudaSuccess ||
        cudaMalloc(&p->d_B, sizeof(float) * std::max<size_t>(K * Nz, 1)) != cudaSuccess ||
        cudaMalloc(&p->d_C, sizeof(float) * std::max<size_t>(rows * Nz, 1)) != cudaSuccess) {
        cudaGetLastError();
        return fail(SPMM_ERR_NO_MEMORY);
    }
    // The rank's rows once, so that the CSR plan can inspect them (row_ptr rebased to 0).
    std::vector<int32_t> rp(rows + 1);
    for (size_t i = 0; i <= rows; ++i) rp[i] = hA->row_ptr[p->r0 + i] - p->p0;
    if (cudaMemcpyAsync(p->d_rp, rp.data(), sizeof(int) * (rows + 1), cudaMemcpyHostToDevice, s) != cudaSuccess ||
        (nnz && (cudaMemcpyAsync(p->d_ci, hA->col_idx + p->p0, sizeof(int) * nnz, cudaMemcpyHostToDevice, s) !=
                     cudaSuccess ||
                 cudaMemcpyAsync(p->d_v, hA->values + p->p0, sizeof(float) * nnz, cudaMemcpyHostToDevice, s) !=
                     cudaSuccess)) ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(SPMM_ERR_CUDA);
    p->dview = spmm_csr_view{static_cast<int32_t>(rows), p->K, static_cast<int32_t>(nnz), p->d_rp, p->d_ci, p->d_v};
    rc = spmm_csr_plan_create(&p->dview, N, nullptr, stream, &p->cplan);
    if (rc != SPMM_OK) return fail(rc);
    spmm_csr_plan_info(p->cplan, &p->algo, nullptr, nullptr);
    spmm_csr_plan_launches(p->cplan, &p->launches);
    // Row groups: ROWWARP computes every row on its own, so any grouping of the rows into
    // launches gives the same bits, with or without the plan's column phases (each element's
    // chain is the same however its positions are cut); the pipelined run launches each group
    // unphased, since its kernels hide behind the copies. Merge plans run as one launch once
    // all rows have landed.
    p->pipelined = p->algo == SPMM_CSR_ROWWARP && rows >= 2 * kRankGroups && N > 0;
    const int G = p->pipelined ? kRankGroups : 1;
    p->groups.resize(G + 1);
    if (p->pipelined) {
        rc = spmm_nnz_balanced_bounds(rp.data(), static_cast<int32_t>(rows), static_cast<int64_t>(nnz), G,
                                      p->groups.data());
        if (rc != SPMM_OK) return fail(rc);
    } else {
        p->groups[0] = 0;
        p->groups[1] = static_cast<int32_t>(rows);
    }
    p->group_pos.resize(G + 1);
    for (int g = 0; g <= G; ++g) p->group_pos[g] = rp[p->groups[g]];
    for (cudaStream_t* x : {&p->s_in, &p->s_comm, &p->s_k, &p->s_out})
        if (cudaStreamCreateWithFlags(x, cudaStreamNonBlocking) != cudaSuccess) return fail(SPMM_ERR_CUDA);
    p->b_pieces = p->world > 1 ? b_pieces_setting() : 1;
    p->ev.assign(4 + 2 * G + p->b_pieces, nullptr);
    if (cudaEventCreateWithFlags(&p->kdone, cudaEventDisableTiming) != cudaSuccess) return fail(SPMM_ERR_CUDA);
    for (auto& e : p->ev)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return fail(SPMM_ERR_CUDA);
    *out = p;
    return SPMM_OK;
}

int spmm_rank_plan_info(const spmm_rank_plan* p, int32_t* row_begin, int32_t* row_end, int32_t* nnz,
                        int32_t* b_row_begin, int32_t* b_row_end, int32_t* algo, int32_t* launches) {
    if (!p) return SPMM_ERR_INVALID_ARG;
    if (row_begin) *row_begin = p->r0;
    if (row_end) *row_end = p->r1;
    if (nnz) *nnz = p->nnz();
    if (b_row_begin) *b_row_begin = p->b_bounds[p->rank];
    if (b_row_end) *b_row_end = p->b_bounds[p->rank + 1];
    if (algo) *algo = p->algo;
    if (launches) *launches = p->launches;
    return SPMM_OK;
}

int spmm_rank_run(spmm_rank_plan* p, const spmm_csr_view* hA, const float* hB, float* hC_rows, void* stream) {
    NvtxRange range("spmm_rank_run");
    SPMM_TRY(issue_checked(p, hA, hB, hC_rows, stream, true));
    p->pending = true;
    const int rc = wait_event(p->end_event(), p->comm, p->timeout_ms());
    if (rc == SPMM_OK) p->pending = false;
    return rc;
}

int spmm_rank_submit(spmm_rank_plan* p, const spmm_csr_view* hA, const float* hB, float* hC_rows, void* stream) {
    NvtxRange range("spmm_rank_submit");
    SPMM_TRY(issue_checked(p, hA, hB, hC_rows, stream, false));
    p->pending = true;
    return SPMM_OK;
}

int spmm_rank_wait(spmm_rank_plan* p, void* stream) {
    if (!p) return SPMM_ERR_INVALID_ARG;
    SPMM_TRY(check_plan_device(p));
    if (!p->submitted) return SPMM_OK;
    SPMM_CUDA_TRY(cudaStreamWaitEvent(as_stream(stream), p->end_event(), 0));
    const int rc = wait_event(p->end_event(), p->comm, p->timeout_ms());
    if (rc == SPMM_OK) p->pending = false;
    return rc;
}

int spmm_rank_execute(spmm_rank_plan* p, void* stream) {
    if (!p) return SPMM_ERR_INVALID_ARG;
    SPMM_TRY(check_plan_device(p));
    // On the device, after the last run's copies (it overwrites C, which they may still read).
    SPMM_TRY(order_after_last_run(p, as_stream(stream)));
    return spmm_csr_plan_execute(p->cplan, p->d_B, p->d_C, stream);
}

int spmm_rank_gather_b(spmm_rank_plan* p, void* stream) {
    if (!p) return SPMM_ERR_INVALID_ARG;
    SPMM_TRY(check_plan_device(p));
    if (p->comm && p->comm->broken) return SPMM_ERR_NCCL;
    SPMM_TRY(order_after_last_run(p, as_stream(stream)));
    return gather_b_issue(p, as_stream(stream));
}

int spmm_rank_plan_buffers(const spmm_rank_plan* p, float** dB, float** dC) {
    if (!p) return SPMM_ERR_INVALID_ARG;
    if (dB) *dB = p->d_B;
    if (dC) *dC = p->d_C;
    return SPMM_OK;
}

void spmm_rank_plan_destroy(spmm_rank_plan* p) { release(p); }

}  // extern "C"
