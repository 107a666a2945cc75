// shard.cu -- one cloud searched by the GPUs of a node, queries sharded.
//
// The reference searches a cloud on one GPU (FRNNEngine::search_gpu,
// python_interface/frnn_engine.cu:195-250).  Queries are independent and the
// point set is read-only, so the search splits over GPUs by query; the
// structure every query needs is built once.  One engine per GPU (one process
// per GPU), joined by an NCCL communicator (NVLink / NVSwitch within a node):
//
//   1. root: plan and build -- on the grid path the bounding box, the plan
//      (principal axes when they pay), the cell histogram, scan and
//      counting-sort scatter; on the tensor-core path the box and the fp16
//      scale; per 4,096-cell scan tile the sum of count * (count + 2) over
//      its cells (each query scans about its own cell's count of candidates
//      per shell cell) gives the partition of the cell-sorted queries into
//      slices of equal estimated work (frnn_shard_partition);
//   2. header broadcast (plan, sizes, slice bounds, the root's status), then
//      an all-reduce of every rank's status, so that a rank that cannot take
//      part makes every rank return the same error instead of waiting;
//   3. data broadcast in one NCCL group: the cell-sorted rows, their ids, the
//      cell starts (and the sorted projected coordinates of a principal-axis
//      grid); on the brute-force paths the cloud itself (every rank then
//      prepares its own fp16 tiles from it);
//   4. every rank searches its slice of the query order (sorted positions
//      on the grid path, 128-query tiles on the tensor-core path, input order
//      on SIMT brute force) with the engine's own kernels;
//   5. the slices go to the root (NCCL send / receive in one group), where one
//      kernel scatters them into the [K, N] results in original query order.
//
// Every wait on the host is bounded (FRNN_ERR_TIMEOUT after the shard's
// timeout; the communicator is then aborted and the shard unusable); an NCCL
// error reported by the communicator ends the call with FRNN_ERR_COMM.
// The only inter-GPU traffic is NCCL's: no kernel here touches another GPU's
// memory.
#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <type_traits>

#include "engine_state.h"
#include "frnn_internal.h"
#include "nccl_dyn.h"

using namespace frnn;
using namespace frnn::eng;

namespace {

constexpr int kMaxShardRanks = 64;

// Everything a rank needs to take part, sent by the root.
struct ShardHeader {
    int status;          // FRNN_OK, or the root's error (every rank returns it)
    int path;            // FRNN_PATH_GRID, _BRUTE or _BRUTE_TC
    int N, dim, K;
    float radius;
    int principal;       // the grid is on principal axes
    int nparts;
    GridPlan P;
    TcPlan tc;
    int bounds[kMaxShardRanks + 1];  // slice r = query order [bounds[r], bounds[r+1])
};
static_assert(std::is_trivially_copyable<ShardHeader>::value, "sent as bytes");

enum ShardStage { SH_BUILD = 0, SH_HEADER, SH_BCAST, SH_SEARCH, SH_GATHER, SH_SCATTER, SH_STAGES };

}  // namespace

struct frnn_shard {
    frnn_engine* e = nullptr;
    ncclComm_t comm = nullptr;
    int rank = 0, nranks = 1;
    bool broken = false;
    double timeout_s = 120.0;
    DevBuf d_hdr, d_stat, tile_work, tile_start, pts, st_idx, st_dist, res_idx, res_dist;
    ShardHeader* h_hdr = nullptr;   // pinned
    int* h_stat = nullptr;          // pinned, 16 ints
    uint64_t* h_work = nullptr;  // pinned, grows with the tile count
    int* h_tstart = nullptr;
    size_t h_tiles = 0;
    cudaEvent_t ev[2 * SH_STAGES] = {};
    bool ev_used[SH_STAGES] = {};
    long long bcast_bytes = 0, gather_bytes = 0;
    int last_rows = 0, last_path = 0;
};

namespace {

const char* nccl_text(ncclResult_t r) {
    const NcclApi* api = nccl_api();
    return api ? api->GetErrorString(r) : "NCCL not loaded";
}

int comm_fail(frnn_shard* sh, ncclResult_t r, const char* what) {
    return fail(sh->e, FRNN_ERR_COMM, std::string(what) + ": " + nccl_text(r));
}

#define SH_NCCL(sh, call, what)                                       \
    do {                                                              \
        ncclResult_t r__ = (call);                                    \
        if (r__ != ncclSuccess) return comm_fail(sh, r__, what);      \
    } while (0)

void sh_begin(frnn_shard* sh, int st) {
    if (sh->e->timing) cudaEventRecord(sh->ev[2 * st], sh->e->stream);
}
void sh_end(frnn_shard* sh, int st) {
    if (sh->e->timing) {
        cudaEventRecord(sh->ev[2 * st + 1], sh->e->stream);
        sh->ev_used[st] = true;
    }
}

// Wait for the engine stream with a deadline, watching the communicator:
// FRNN_ERR_COMM when NCCL reports an error, FRNN_ERR_TIMEOUT when the
// deadline passes (a peer that never joins); either way the communicator is
// aborted and the shard cannot be used again.
int wait_stream(frnn_shard* sh, const char* what) {
    const NcclApi* api = nccl_api();
    const auto t0 = std::chrono::steady_clock::now();
    for (long long it = 0;; ++it) {
        const cudaError_t q = cudaStreamQuery(sh->e->stream);
        if (q == cudaSuccess) return FRNN_OK;
        if (q != cudaErrorNotReady) return cuda_fail(sh->e, q, what);
        ncclResult_t ae = ncclSuccess;
        if (api->CommGetAsyncError(sh->comm, &ae) == ncclSuccess && ae != ncclSuccess && ae != ncclInProgress) {
            api->CommAbort(sh->comm);
            sh->comm = nullptr;
            sh->broken = true;
            return fail(sh->e, FRNN_ERR_COMM, std::string(what) + ": " + nccl_text(ae));
        }
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > sh->timeout_s) {
            api->CommAbort(sh->comm);
            sh->comm = nullptr;
            sh->broken = true;
            return fail(sh->e, FRNN_ERR_TIMEOUT,
                        std::string(what) + ": no progress within the shard timeout (a rank did not take part?)");
        }
        // spin first (the common wait is short), then back off
        if (it > 20000) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// Root side of step 5: slice r of the query order, [b[r], b[r+1]), arrived as
// [K, rows_r] at st + K*b[r] (the root's own slice at own); row j is query
// order position b[r] + j.  One thread per (original query q, slot k): the
// query's position is inv[q] on the grid path (cell order), q itself on the
// brute-force paths; the stores to out[k*N + q] are coalesced and the loads
// gather from a slice row that stays in L2 while its k is being written.
__global__ void shard_scatter_kernel(const int* __restrict__ st_idx, const float* __restrict__ st_dist,
                                     const int* __restrict__ own_idx, const float* __restrict__ own_dist,
                                     int own, const int* __restrict__ bounds, int nparts,
                                     const int* __restrict__ inv, int N, int* __restrict__ out_idx,
                                     float* __restrict__ out_dist) {
    __shared__ int b[kMaxShardRanks + 1];
    for (int i = threadIdx.x; i <= nparts; i += blockDim.x) b[i] = bounds[i];
    __syncthreads();
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= N) return;
    const int k = blockIdx.y;
    const int sq = inv ? __ldg(&inv[q]) : q;
    if ((unsigned)sq >= (unsigned)N) return;  // only after a scan gave up (FRNN_ERR_TIMEOUT)
    int lo = 0, hi = nparts;  // the part r with b[r] <= sq < b[r+1]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (b[mid] <= sq) lo = mid;
        else hi = mid;
    }
    const int r = lo, rows = b[r + 1] - b[r], j = sq - b[r];
    const long long src = (long long)k * rows + j;
    const long long dst = (long long)k * N + q;
    if (r == own) {
        out_idx[dst] = __ldg(&own_idx[src]);
        out_dist[dst] = __ldg(&own_dist[src]);
    } else {
        const long long base = (long long)b[r] * gridDim.y;  // K * b[r]
        out_idx[dst] = __ldg(&st_idx[base + src]);
        out_dist[dst] = __ldg(&st_dist[base + src]);
    }
}

int grow_pinned_tiles(frnn_shard* sh, size_t tiles) {
    if (sh->h_tiles >= tiles) return FRNN_OK;
    if (sh->h_work) cudaFreeHost(sh->h_work);
    if (sh->h_tstart) cudaFreeHost(sh->h_tstart);
    sh->h_work = nullptr;
    sh->h_tstart = nullptr;
    sh->h_tiles = 0;
    const size_t want = tiles + tiles / 8 + 64;
    if (cudaMallocHost(&sh->h_work, want * 8) != cudaSuccess ||
        cudaMallocHost(&sh->h_tstart, want * 4) != cudaSuccess) {
        cudaGetLastError();
        return fail(sh->e, FRNN_ERR_OOM, "pinned staging for the partition");
    }
    sh->h_tiles = want;
    return FRNN_OK;
}

// Step 1 on the root: plan, build and partition into h_hdr (status set).
int root_plan(frnn_shard* sh, const float* d_pts, int N, int dim, int K, float radius) {
    frnn_engine* e = sh->e;
    ShardHeader& H = *sh->h_hdr;
    H.path = self_search_path(e, N, dim);
    const int parts = sh->nranks;
    if (H.path == FRNN_PATH_GRID) {
        bool principal = false;
        int st = plan_grid_search(e, d_pts, N, dim, radius, &H.path, H.P, &principal);
        if (st != FRNN_OK) return st;
        H.principal = principal ? 1 : 0;
    }
    if (H.path == FRNN_PATH_BRUTE_TC) {
        int st = tc_plan(e, d_pts, N, dim, radius, &H.tc);
        if (st != FRNN_OK) return st;
        if (!H.tc.ok) H.path = FRNN_PATH_BRUTE;
    }
    if (H.path == FRNN_PATH_GRID) {
        const long long tiles = scan_tiles(H.P.cells);
        FRNN_GROW(e, sh->tile_work, (size_t)tiles * 8);
        FRNN_GROW(e, sh->tile_start, (size_t)tiles * 4);
        // inv: the root's scatter reads each query's row through it
        int st = build_points(e, d_pts, H.P, H.principal ? e->proj_u.as<float>() : nullptr, true,
                              sh->tile_work.as<unsigned long long>(), sh->tile_start.as<int>());
        if (st != FRNN_OK) return st;
        st = grow_pinned_tiles(sh, (size_t)tiles);
        if (st != FRNN_OK) return st;
        cudaStream_t s = e->stream;
        FRNN_CHECK(e, cudaMemcpyAsync(sh->h_work, sh->tile_work.p, (size_t)tiles * 8, cudaMemcpyDeviceToHost, s),
                   "tile work readback");
        FRNN_CHECK(e, cudaMemcpyAsync(sh->h_tstart, sh->tile_start.p, (size_t)tiles * 4, cudaMemcpyDeviceToHost, s),
                   "tile start readback");
        FRNN_CHECK(e, cudaMemcpyAsync(sh->h_stat, e->err_flag.p, sizeof(int), cudaMemcpyDeviceToHost, s),
                   "error flag readback");
        FRNN_CHECK(e, cudaStreamSynchronize(s), "partition sync");
        if (sh->h_stat[0] != 0) {
            cudaMemsetAsync(e->err_flag.p, 0, sizeof(int), s);
            cudaStreamSynchronize(s);
            return fail(e, FRNN_ERR_TIMEOUT, "a bounded device-side wait gave up");
        }
        if (frnn_shard_partition(sh->h_work, sh->h_tstart, tiles, N, parts, H.bounds) != FRNN_OK)
            return fail(e, FRNN_ERR_INVALID_ARG, "partition failed");
    } else if (H.path == FRNN_PATH_BRUTE_TC) {
        const int ntq = (N + 127) / 128;
        for (int r = 0; r <= parts; ++r) H.bounds[r] = std::min(N, (int)((long long)ntq * r / parts) * 128);
    } else {
        for (int r = 0; r <= parts; ++r) H.bounds[r] = (int)((long long)N * r / parts);
    }
    return FRNN_OK;
}

}  // namespace

extern "C" {

int frnn_shard_partition(const uint64_t* tile_work, const int* tile_start, int64_t tiles, int N, int nparts,
                         int* bounds) {
    if (!tile_work || !tile_start || !bounds || tiles < 1 || N < 0 || nparts < 1) return FRNN_ERR_INVALID_ARG;
    unsigned long long total = 0;
    for (int64_t t = 0; t < tiles; ++t) total += tile_work[t];
    bounds[0] = 0;
    bounds[nparts] = N;
    // boundary r sits at the tile edge nearest to the r/nparts quantile of the
    // cumulative work; tile edges are cell starts, so a slice never splits a cell
    int64_t t = 0;
    unsigned long long before = 0;  // work of tiles [0, t)
    for (int r = 1; r < nparts; ++r) {
        const long double target = (long double)total * r / nparts;
        while (t < tiles && (long double)(before + tile_work[t]) <= target) before += tile_work[t++];
        int pos = t < tiles ? tile_start[t] : N;
        if (t < tiles && target - (long double)before > 0.5L * (long double)tile_work[t])
            pos = t + 1 < tiles ? tile_start[t + 1] : N;  // nearer the end of tile t
        pos = std::min(std::max(pos, bounds[r - 1]), N);
        bounds[r] = pos;
    }
    return FRNN_OK;
}

}  // extern "C"

extern "C" {

int frnn_shard_unique_id(unsigned char* id_out) {
    if (!id_out) return FRNN_ERR_INVALID_ARG;
    const NcclApi* api = nccl_api();
    if (!api) return FRNN_ERR_COMM;
    ncclUniqueId id;
    if (api->GetUniqueId(&id) != ncclSuccess) return FRNN_ERR_COMM;
    std::memcpy(id_out, id.internal, FRNN_SHARD_ID_BYTES);
    return FRNN_OK;
}

int frnn_shard_create(frnn_engine* e, int nranks, int rank, const unsigned char* id, frnn_shard** out) {
    if (!out) return FRNN_ERR_INVALID_ARG;
    *out = nullptr;
    if (!e || !id || nranks < 1 || nranks > kMaxShardRanks || rank < 0 || rank >= nranks)
        return FRNN_ERR_INVALID_ARG;
    const NcclApi* api = nccl_api();
    if (!api) return fail(e, FRNN_ERR_COMM, "libnccl.so.2 could not be loaded");
    DeviceGuard g(e->device);
    frnn_shard* sh = new frnn_shard();
    sh->e = e;
    sh->rank = rank;
    sh->nranks = nranks;
    ncclUniqueId uid;
    std::memcpy(uid.internal, id, FRNN_SHARD_ID_BYTES);
    ncclResult_t r = api->CommInitRank(&sh->comm, nranks, uid, rank);
    if (r != ncclSuccess) {
        delete sh;
        return fail(e, FRNN_ERR_COMM, std::string("ncclCommInitRank: ") + nccl_text(r));
    }
    int st = FRNN_OK;
    if ((st = grow(e, sh->d_hdr, sizeof(ShardHeader), "shard header")) ||
        (st = grow(e, sh->d_stat, 64, "shard status"))) {
        frnn_shard_destroy(sh);
        return st;
    }
    if (cudaMallocHost(&sh->h_hdr, sizeof(ShardHeader)) != cudaSuccess ||
        cudaMallocHost(&sh->h_stat, 64) != cudaSuccess) {
        cudaGetLastError();
        frnn_shard_destroy(sh);
        return fail(e, FRNN_ERR_OOM, "pinned shard staging");
    }
    for (cudaEvent_t& ev : sh->ev)
        if (cudaEventCreate(&ev) != cudaSuccess) {
            cudaGetLastError();
            frnn_shard_destroy(sh);
            return fail(e, FRNN_ERR_CUDA, "shard events");
        }
    *out = sh;
    return FRNN_OK;
}

int frnn_shard_destroy(frnn_shard* sh) {
    if (!sh) return FRNN_OK;
    {
        DeviceGuard g(sh->e->device);
        cudaStreamSynchronize(sh->e->stream);
        const NcclApi* api = nccl_api();
        if (sh->comm && api) api->CommDestroy(sh->comm);
        for (DevBuf* b : {&sh->d_hdr, &sh->d_stat, &sh->tile_work, &sh->tile_start, &sh->pts, &sh->st_idx,
                          &sh->st_dist, &sh->res_idx, &sh->res_dist})
            if (b->p) cudaFree(b->p);
        if (sh->h_hdr) cudaFreeHost(sh->h_hdr);
        if (sh->h_stat) cudaFreeHost(sh->h_stat);
        if (sh->h_work) cudaFreeHost(sh->h_work);
        if (sh->h_tstart) cudaFreeHost(sh->h_tstart);
        for (cudaEvent_t ev : sh->ev)
            if (ev) cudaEventDestroy(ev);
    }
    delete sh;
    return FRNN_OK;
}

int frnn_shard_set_timeout(frnn_shard* sh, double seconds) {
    if (!sh || !(seconds > 0.0)) return FRNN_ERR_INVALID_ARG;
    sh->timeout_s = seconds;
    return FRNN_OK;
}

int frnn_search_sharded(frnn_shard* sh, int root, const float* d_points_soa, int N, int dim, int K,
                        float radius, int** d_idxs, float** d_dists) {
    if (!sh) return FRNN_ERR_INVALID_ARG;
    frnn_engine* e = sh->e;
    if (sh->broken) return fail(e, FRNN_ERR_STATE, "the shard's communicator was aborted by an earlier error");
    if (root < 0 || root >= sh->nranks) return fail(e, FRNN_ERR_INVALID_ARG, "root must be a rank of the shard");
    if (!d_idxs || !d_dists) return fail(e, FRNN_ERR_INVALID_ARG, "output pointers are null");
    *d_idxs = nullptr;
    *d_dists = nullptr;
    const NcclApi* api = nccl_api();
    DeviceGuard g(e->device);
    cudaStream_t s = e->stream;
    const bool is_root = sh->rank == root;
    const int parts = sh->nranks;
    e->last_N = -1;
    e->last_part_rows = -1;
    e->built.valid = false;
    e->last_overflow_map = 0;
    for (int i = 0; i < FRNN_STAGES; ++i) e->stage_used[i] = false;
    for (int i = 0; i < SH_STAGES; ++i) sh->ev_used[i] = false;
    sh->bcast_bytes = sh->gather_bytes = 0;
    sh->last_rows = 0;

    // local checks: every rank passes the same N, dim, K and radius; the root
    // passes the cloud (device memory on its GPU)
    int local = check_search_args(e, is_root ? (const void*)d_points_soa : (const void*)sh, N, dim, K, radius);
    if (local == FRNN_OK && is_root) local = check_device_ptr(e, d_points_soa);

    // 1. root: plan, build, partition
    ShardHeader& H = *sh->h_hdr;
    const size_t bounds_off = offsetof(ShardHeader, bounds);
    if (is_root) {
        std::memset(&H, 0, sizeof(H));
        H.N = N;
        H.dim = dim;
        H.K = K;
        H.radius = radius;
        H.nparts = parts;
        sh_begin(sh, SH_BUILD);
        H.status = local == FRNN_OK ? root_plan(sh, d_points_soa, N, dim, K, radius) : local;
        sh_end(sh, SH_BUILD);
        FRNN_CHECK(e, cudaMemcpyAsync(sh->d_hdr.p, &H, sizeof(H), cudaMemcpyHostToDevice, s), "header upload");
    }
    (void)bounds_off;
    // 2. header, then every rank's status
    sh_begin(sh, SH_HEADER);
    SH_NCCL(sh, api->Broadcast(sh->d_hdr.p, sh->d_hdr.p, sizeof(ShardHeader), ncclUint8, root, sh->comm, s),
            "header broadcast");
    FRNN_CHECK(e, cudaMemcpyAsync(&H, sh->d_hdr.p, sizeof(H), cudaMemcpyDeviceToHost, s), "header readback");
    int st = wait_stream(sh, "header broadcast");
    if (st != FRNN_OK) return st;
    if (H.status != FRNN_OK) {
        if (!is_root) fail(e, H.status, "the root's part of the sharded search failed");
        return H.status;
    }
    if (local == FRNN_OK && (H.N != N || H.dim != dim || H.K != K || H.radius != radius || H.nparts != parts))
        local = fail(e, FRNN_ERR_INVALID_ARG, "N, dim, K and radius must be the same on every rank");
    const int b0 = H.bounds[sh->rank], b1 = H.bounds[sh->rank + 1], rows = b1 - b0;
    const int path = H.path;
    const GridPlan& P = H.P;
    // buffers this rank needs (the root's build made its own)
    if (local == FRNN_OK && !is_root) {
        if (path == FRNN_PATH_GRID) {
            if ((local = grow(e, e->rows, ((size_t)N + kCollectRowPad) * P.row * 4, "rows")) == FRNN_OK &&
                (local = grow(e, e->ids, (size_t)N * 4, "ids")) == FRNN_OK &&
                (local = grow(e, e->starts, ((size_t)P.cells + 1) * 4, "starts")) == FRNN_OK && H.principal)
                local = grow(e, e->proj_s, (size_t)N * kProjStride * 4, "proj_s");
        } else {
            local = grow(e, sh->pts, (size_t)N * dim * 4, "points");
        }
    }
    if (local == FRNN_OK) local = grow(e, e->out_idx, (size_t)std::max(rows, 1) * K * 4, "out_idx");
    if (local == FRNN_OK) local = grow(e, e->out_dist, (size_t)std::max(rows, 1) * K * 4, "out_dist");
    if (local == FRNN_OK && is_root) {
        if ((local = grow(e, sh->st_idx, (size_t)N * K * 4, "staging")) == FRNN_OK &&
            (local = grow(e, sh->st_dist, (size_t)N * K * 4, "staging")) == FRNN_OK &&
            (local = grow(e, sh->res_idx, (size_t)N * K * 4, "results")) == FRNN_OK)
            local = grow(e, sh->res_dist, (size_t)N * K * 4, "results");
    }
    sh->h_stat[0] = local;
    FRNN_CHECK(e, cudaMemcpyAsync(sh->d_stat.p, sh->h_stat, sizeof(int), cudaMemcpyHostToDevice, s),
               "status upload");
    SH_NCCL(sh, api->AllReduce(sh->d_stat.p, sh->d_stat.p, 1, ncclInt32, ncclMax, sh->comm, s), "status all-reduce");
    FRNN_CHECK(e, cudaMemcpyAsync(sh->h_stat + 1, sh->d_stat.p, sizeof(int), cudaMemcpyDeviceToHost, s),
               "status readback");
    st = wait_stream(sh, "status all-reduce");
    if (st != FRNN_OK) return st;
    sh_end(sh, SH_HEADER);
    if (sh->h_stat[1] != FRNN_OK) {
        if (local == FRNN_OK) fail(e, sh->h_stat[1], "another rank could not take part in the sharded search");
        return sh->h_stat[1];
    }

    // 3. the data every rank searches
    sh_begin(sh, SH_BCAST);
    const float* pts = is_root ? d_points_soa : sh->pts.as<float>();
    SH_NCCL(sh, api->GroupStart(), "group start");
    if (path == FRNN_PATH_GRID) {
        const size_t nrow = (size_t)N * P.row, nc = (size_t)P.cells + 1;
        SH_NCCL(sh, api->Broadcast(e->rows.p, e->rows.p, nrow, ncclFloat32, root, sh->comm, s), "rows broadcast");
        SH_NCCL(sh, api->Broadcast(e->ids.p, e->ids.p, (size_t)N, ncclInt32, root, sh->comm, s), "ids broadcast");
        SH_NCCL(sh, api->Broadcast(e->starts.p, e->starts.p, nc, ncclInt32, root, sh->comm, s), "starts broadcast");
        sh->bcast_bytes = (long long)(nrow + N + nc) * 4;
        if (H.principal) {
            SH_NCCL(sh, api->Broadcast(e->proj_s.p, e->proj_s.p, (size_t)N * kProjStride, ncclFloat32, root,
                                       sh->comm, s),
                    "projection broadcast");
            sh->bcast_bytes += (long long)N * kProjStride * 4;
        }
    } else {
        SH_NCCL(sh, api->Broadcast(pts, (void*)pts, (size_t)N * dim, ncclFloat32, root, sh->comm, s),
                "points broadcast");
        sh->bcast_bytes = (long long)N * dim * 4;
    }
    SH_NCCL(sh, api->GroupEnd(), "group end");
    sh_end(sh, SH_BCAST);

    // 4. this rank's slice
    sh_begin(sh, SH_SEARCH);
    const float r2 = radius * radius;
    if (rows > 0) {
        if (path == FRNN_PATH_GRID) {
            st = search_built(e, P, H.principal != 0, K, r2, b0, b1, false, e->out_idx.as<int>(),
                              e->out_dist.as<float>());
        } else if (path == FRNN_PATH_BRUTE_TC) {
            st = tc_search(e, pts, N, dim, K, radius, H.tc, e->out_idx.as<int>(), e->out_dist.as<float>(),
                           b0 / 128, (b1 + 127) / 128);
        } else {
            FRNN_CHECK(e, launch_bruteforce(pts, N, dim, K, r2, b0, b1, e->out_idx.as<int>(),
                                            e->out_dist.as<float>(), rows, s),
                       "bruteforce launch");
            e->launches++;
        }
        if (st != FRNN_OK) return st;
    }
    sh_end(sh, SH_SEARCH);

    // 5. the slices to the root
    sh_begin(sh, SH_GATHER);
    SH_NCCL(sh, api->GroupStart(), "group start");
    if (is_root) {
        for (int r = 0; r < parts; ++r) {
            const int n_r = H.bounds[r + 1] - H.bounds[r];
            if (r == root || n_r == 0) continue;
            const size_t off = (size_t)K * H.bounds[r], cnt = (size_t)K * n_r;
            SH_NCCL(sh, api->Recv(sh->st_idx.as<int>() + off, cnt, ncclInt32, r, sh->comm, s), "idx receive");
            SH_NCCL(sh, api->Recv(sh->st_dist.as<float>() + off, cnt, ncclFloat32, r, sh->comm, s), "dist receive");
            sh->gather_bytes += (long long)cnt * 8;
        }
    } else if (rows > 0) {
        const size_t cnt = (size_t)K * rows;
        SH_NCCL(sh, api->Send(e->out_idx.p, cnt, ncclInt32, root, sh->comm, s), "idx send");
        SH_NCCL(sh, api->Send(e->out_dist.p, cnt, ncclFloat32, root, sh->comm, s), "dist send");
        sh->gather_bytes = (long long)cnt * 8;
    }
    SH_NCCL(sh, api->GroupEnd(), "group end");
    sh_end(sh, SH_GATHER);
    if (is_root) {
        sh_begin(sh, SH_SCATTER);
        dim3 grid((unsigned)((N + 255) / 256), (unsigned)K);
        shard_scatter_kernel<<<grid, 256, 0, s>>>(sh->st_idx.as<int>(), sh->st_dist.as<float>(), e->out_idx.as<int>(),
                                                  e->out_dist.as<float>(), root,
                                                  reinterpret_cast<const int*>(static_cast<const char*>(sh->d_hdr.p) +
                                                                               offsetof(ShardHeader, bounds)),
                                                  parts, path == FRNN_PATH_GRID ? e->inv.as<int>() : nullptr, N,
                                                  sh->res_idx.as<int>(), sh->res_dist.as<float>());
        FRNN_CHECK(e, cudaGetLastError(), "scatter launch");
        e->launches++;
        sh_end(sh, SH_SCATTER);
    }
    FRNN_CHECK(e, cudaMemcpyAsync(sh->h_stat + 2, e->err_flag.p, sizeof(int), cudaMemcpyDeviceToHost, s),
               "error flag readback");
    st = wait_stream(sh, "sharded search");
    if (st != FRNN_OK) return st;
    if (sh->h_stat[2] != 0) {
        cudaMemsetAsync(e->err_flag.p, 0, sizeof(int), s);
        cudaStreamSynchronize(s);
        return fail(e, FRNN_ERR_TIMEOUT, "a bounded device-side wait gave up");
    }
    sh->last_rows = rows;
    sh->last_path = path;
    e->last_path = path;
    e->last_g = path == FRNN_PATH_GRID ? P.g : 0;
    e->last_cells = path == FRNN_PATH_GRID ? P.cells : 0;
    e->last_principal = path == FRNN_PATH_GRID && H.principal;
    if (is_root) {
        *d_idxs = sh->res_idx.as<int>();
        *d_dists = sh->res_dist.as<float>();
    }
    return FRNN_OK;
}

int frnn_shard_last_stats(frnn_shard* sh, float* stage_ms, int n, int64_t* bcast_bytes, int64_t* gather_bytes,
                          int* rows) {
    if (!sh) return FRNN_ERR_INVALID_ARG;
    DeviceGuard g(sh->e->device);
    if (bcast_bytes) *bcast_bytes = sh->bcast_bytes;
    if (gather_bytes) *gather_bytes = sh->gather_bytes;
    if (rows) *rows = sh->last_rows;
    for (int i = 0; stage_ms && i < n; ++i) {
        stage_ms[i] = -1.0f;
        if (i < SH_STAGES && sh->ev_used[i]) {
            if (cudaEventSynchronize(sh->ev[2 * i + 1]) != cudaSuccess ||
                cudaEventElapsedTime(&stage_ms[i], sh->ev[2 * i], sh->ev[2 * i + 1]) != cudaSuccess) {
                cudaGetLastError();
                stage_ms[i] = -1.0f;
            }
        }
    }
    return FRNN_OK;
}

}  // extern "C"
