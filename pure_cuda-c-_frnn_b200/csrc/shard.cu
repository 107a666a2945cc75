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
//      scale.  On the grid path the candidates of every 64th cell-sorted
//      query (the point count of its 3^g shell, what a search scans) sample
//      the work along the query order, and frnn_shard_partition cuts it into
//      slices of equal estimated work;
//   2. header broadcast (plan, sizes, slice bounds, the root's status), then
//      an all-reduce of every rank's status, so that a rank that cannot take
//      part makes every rank return the same error instead of waiting;
//   3. data broadcast in one NCCL group: the cell-sorted rows, their ids, the
//      cell starts (and the sorted projected coordinates of a principal-axis
//      grid); on the brute-force paths the cloud itself (every rank then
//      prepares its own fp16 tiles from it);
//   4. every rank searches its slice of the query order (sorted positions
//      on the grid path, 128-query tiles on the tensor-core path, input order
//      on SIMT brute force) with the engine's own kernels, in a few chunks;
//   5. each finished chunk goes to the root at once (NCCL send / receive on a
//      high-priority communication stream) while the next chunk is searched,
//      and the root scatters every arrived chunk into the [K, N] results in
//      original query order -- so the gather overlaps the search and only the
//      last chunk's transfer remains after it.
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

// stages timed when the engine's timing is on: the root's plan and build, the
// header and status exchange, the data broadcast, the chunked slice search
// (engine stream), the root's receives and scatters (communication stream)
enum ShardStage { SH_BUILD = 0, SH_HEADER, SH_BCAST, SH_SEARCH, SH_GATHER, SH_STAGES };

// Chunks of a rank's slice: each is searched, then sent while the next one is
// searched.  Slices below kChunkMin queries are one chunk.
constexpr int kMaxChunks = 8;
constexpr int kChunkMin = 65536;
// Every kSampleStride-th cell-sorted query samples the search work.
constexpr int kSampleStride = 64;

// Chunk c of the slice [b0, b1) is [cb[c], cb[c+1]); on the tensor-core path
// every cut is a multiple of 128 (whole query tiles).  Every rank computes the
// same cuts for every slice.
int chunk_bounds(int b0, int b1, int path, int chunks, int* cb) {
    const int rows = b1 - b0;
    const int m = std::max(1, std::min(chunks, rows / kChunkMin));
    cb[0] = b0;
    for (int c = 1; c < m; ++c) {
        int x = b0 + (int)((long long)rows * c / m);
        if (path == FRNN_PATH_BRUTE_TC) x = std::min(b1, (x + 127) / 128 * 128);
        cb[c] = std::max(x, cb[c - 1]);
    }
    cb[m] = b1;
    return m;
}

}  // namespace

struct frnn_shard {
    frnn_engine* e = nullptr;
    ncclComm_t comm = nullptr;
    int rank = 0, nranks = 1;
    bool broken = false;
    double timeout_s = 120.0;
    DevBuf d_hdr, d_stat, work, pts, st_idx, st_dist, res_idx, res_dist;
    ShardHeader* h_hdr = nullptr;   // pinned
    int* h_stat = nullptr;          // pinned, 16 ints
    uint64_t* h_work = nullptr;     // pinned, grows with the sample count
    int* h_wstart = nullptr;
    size_t h_samples = 0;
    cudaStream_t cs = nullptr;      // communication stream (gather)
    int chunks = 1;                 // FRNN_SHARD_OPT_CHUNKS
    int comm_priority = 0;          // FRNN_SHARD_OPT_COMM_PRIORITY
    cudaEvent_t chunk_ev[kMaxChunks] = {}, comm_done = nullptr;
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

// Root side of step 5: one arrived chunk, [K, rows] at src (row j = query
// order position q0 + j), into out[k*N + q] with q = ids[q0 + j] on the grid
// path (cell order) or q0 + j on the brute-force paths.
__global__ void shard_scatter_kernel(const int* __restrict__ src_idx, const float* __restrict__ src_dist, int q0,
                                     int rows, const int* __restrict__ ids, int N, int* __restrict__ out_idx,
                                     float* __restrict__ out_dist) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= rows) return;
    const int k = blockIdx.y;
    const int q = ids ? __ldg(&ids[q0 + j]) : q0 + j;
    if ((unsigned)q >= (unsigned)N) return;  // only after a scan gave up (FRNN_ERR_TIMEOUT)
    const long long src = (long long)k * rows + j, dst = (long long)k * N + q;
    out_idx[dst] = __ldg(&src_idx[src]);
    out_dist[dst] = __ldg(&src_dist[src]);
}

cudaError_t launch_shard_scatter(const int* src_idx, const float* src_dist, int q0, int rows, int K, const int* ids,
                                 int N, int* out_idx, float* out_dist, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    dim3 grid((unsigned)((rows + 255) / 256), (unsigned)K);
    shard_scatter_kernel<<<grid, 256, 0, s>>>(src_idx, src_dist, q0, rows, ids, N, out_idx, out_dist);
    return cudaGetLastError();
}

// The work of the cell-sorted queries, sampled: for sorted position
// i * stride, the points in its cell's 3^g shell (the x-merged rows a grid
// search walks) plus a fixed charge per row.  work[i] covers the stride
// queries from there.
__global__ void sample_work_kernel(const float* __restrict__ rows, const float* __restrict__ proj_s,
                                   const int* __restrict__ starts, GridPlan P, int stride, int nsamples,
                                   unsigned long long* __restrict__ work) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nsamples) return;
    const long long sq = (long long)i * stride;
    int gc[kMaxGridAxes];
    for (int a = 0; a < P.g; ++a) {
        const float x = proj_s ? __ldg(&proj_s[sq * kProjStride + a]) : __ldg(&rows[sq * P.row + a]);
        gc[a] = cell_coord(x, P.origin[a], P.inv_cell, P.res[a]);
    }
    int nrows = 1;
    for (int a = 1; a < P.g; ++a) nrows *= 3;
    const int xlo = max(gc[0] - 1, 0), xhi = min(gc[0] + 1, P.res[0] - 1);
    unsigned long long total = 0;
    for (int t = 0; t < nrows; ++t) {
        int u = t;
        long long rb = 0;
        bool ok = true;
        for (int a = 1; a < P.g; ++a) {
            const int c = gc[a] + (u % 3) - 1;
            u /= 3;
            ok &= (c >= 0) & (c < P.res[a]);
            rb += (long long)c * P.stride[a];
        }
        if (ok) {
            const int s0 = __ldg(&starts[rb + xlo]), s1 = __ldg(&starts[rb + xhi + 1]);
            total += (unsigned long long)max(s1 - s0, 0);
        }
    }
    work[i] = (total + 8ull * nrows) * (unsigned long long)min((long long)stride, (long long)P.n - sq);
}

int grow_pinned_samples(frnn_shard* sh, size_t n) {
    if (sh->h_samples >= n) return FRNN_OK;
    if (sh->h_work) cudaFreeHost(sh->h_work);
    if (sh->h_wstart) cudaFreeHost(sh->h_wstart);
    sh->h_work = nullptr;
    sh->h_wstart = nullptr;
    sh->h_samples = 0;
    const size_t want = n + n / 8 + 64;
    if (cudaMallocHost(&sh->h_work, want * 8) != cudaSuccess ||
        cudaMallocHost(&sh->h_wstart, want * 4) != cudaSuccess) {
        cudaGetLastError();
        return fail(sh->e, FRNN_ERR_OOM, "pinned staging for the partition");
    }
    sh->h_samples = want;
    return FRNN_OK;
}

// Step 1 on the root: plan, build and partition into h_hdr.
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
        cudaStream_t s = e->stream;
        int st = build_points(e, d_pts, H.P, H.principal ? e->proj_u.as<float>() : nullptr, false);
        if (st != FRNN_OK) return st;
        if (parts > 1) {
            const int ns = (N + kSampleStride - 1) / kSampleStride;
            FRNN_GROW(e, sh->work, (size_t)ns * 8);
            st = grow_pinned_samples(sh, (size_t)ns);
            if (st != FRNN_OK) return st;
            sample_work_kernel<<<(ns + 127) / 128, 128, 0, s>>>(
                e->rows.as<float>(), H.principal ? e->proj_s.as<float>() : nullptr, e->starts.as<int>(), H.P,
                kSampleStride, ns, sh->work.as<unsigned long long>());
            FRNN_CHECK(e, cudaGetLastError(), "work sample launch");
            e->launches++;
            FRNN_CHECK(e, cudaMemcpyAsync(sh->h_work, sh->work.p, (size_t)ns * 8, cudaMemcpyDeviceToHost, s),
                       "work sample readback");
            FRNN_CHECK(e, cudaMemcpyAsync(sh->h_stat, e->err_flag.p, sizeof(int), cudaMemcpyDeviceToHost, s),
                       "error flag readback");
            FRNN_CHECK(e, cudaStreamSynchronize(s), "partition sync");
            if (sh->h_stat[0] != 0) {
                cudaMemsetAsync(e->err_flag.p, 0, sizeof(int), s);
                cudaStreamSynchronize(s);
                return fail(e, FRNN_ERR_TIMEOUT, "a bounded device-side wait gave up");
            }
            for (int i = 0; i < ns; ++i) sh->h_wstart[i] = i * kSampleStride;
            if (frnn_shard_partition(sh->h_work, sh->h_wstart, ns, N, parts, H.bounds) != FRNN_OK)
                return fail(e, FRNN_ERR_INVALID_ARG, "partition failed");
        } else {
            H.bounds[0] = 0;
            H.bounds[1] = N;
        }
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
    bool ok = cudaStreamCreateWithFlags(&sh->cs, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&sh->comm_done, cudaEventDisableTiming) == cudaSuccess;
    for (cudaEvent_t& ev : sh->chunk_ev) ok = ok && cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) == cudaSuccess;
    for (cudaEvent_t& ev : sh->ev) ok = ok && cudaEventCreate(&ev) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        frnn_shard_destroy(sh);
        return fail(e, FRNN_ERR_CUDA, "shard stream and events");
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
        if (sh->cs) cudaStreamSynchronize(sh->cs);
        for (DevBuf* b : {&sh->d_hdr, &sh->d_stat, &sh->work, &sh->pts, &sh->st_idx, &sh->st_dist, &sh->res_idx,
                          &sh->res_dist})
            if (b->p) cudaFree(b->p);
        if (sh->h_hdr) cudaFreeHost(sh->h_hdr);
        if (sh->h_stat) cudaFreeHost(sh->h_stat);
        if (sh->h_work) cudaFreeHost(sh->h_work);
        if (sh->h_wstart) cudaFreeHost(sh->h_wstart);
        for (cudaEvent_t ev : sh->ev)
            if (ev) cudaEventDestroy(ev);
        for (cudaEvent_t ev : sh->chunk_ev)
            if (ev) cudaEventDestroy(ev);
        if (sh->comm_done) cudaEventDestroy(sh->comm_done);
        if (sh->cs) cudaStreamDestroy(sh->cs);
    }
    delete sh;
    return FRNN_OK;
}

int frnn_shard_set_timeout(frnn_shard* sh, double seconds) {
    if (!sh || !(seconds > 0.0)) return FRNN_ERR_INVALID_ARG;
    sh->timeout_s = seconds;
    return FRNN_OK;
}

int frnn_shard_set_option(frnn_shard* sh, int option, int64_t value) {
    if (!sh) return FRNN_ERR_INVALID_ARG;
    switch (option) {
        case FRNN_SHARD_OPT_CHUNKS:
            if (value < 1 || value > kMaxChunks) return fail(sh->e, FRNN_ERR_INVALID_ARG, "chunks must be in [1, 8]");
            sh->chunks = (int)value;
            return FRNN_OK;
        case FRNN_SHARD_OPT_COMM_PRIORITY: {
            if (value != 0 && value != 1) return fail(sh->e, FRNN_ERR_INVALID_ARG, "priority must be 0 or 1");
            if ((int)value == sh->comm_priority) return FRNN_OK;
            DeviceGuard g(sh->e->device);
            int lo = 0, hi = 0;
            cudaStream_t ns = nullptr;
            if (cudaDeviceGetStreamPriorityRange(&lo, &hi) != cudaSuccess ||
                cudaStreamCreateWithPriority(&ns, cudaStreamNonBlocking, value ? hi : lo) != cudaSuccess) {
                cudaGetLastError();
                return fail(sh->e, FRNN_ERR_CUDA, "communication stream");
            }
            cudaStreamSynchronize(sh->cs);
            cudaStreamDestroy(sh->cs);
            sh->cs = ns;
            sh->comm_priority = (int)value;
            return FRNN_OK;
        }
        default:
            return fail(sh->e, FRNN_ERR_INVALID_ARG, "unknown shard option");
    }
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

    // 4 and 5. this rank's slice, chunk by chunk; every finished chunk goes to
    // the root on the communication stream while the next is searched, and
    // the root scatters each arrived chunk
    const float r2 = radius * radius;
    const int* scatter_ids = path == FRNN_PATH_GRID ? e->ids.as<int>() : nullptr;
    if (path == FRNN_PATH_BRUTE_TC && rows > 0) {
        st = tc_prepare(e, pts, N, dim, H.tc);
        if (st != FRNN_OK) return st;
    }
    int cb[kMaxChunks + 1];
    const int m = chunk_bounds(b0, b1, path, sh->chunks, cb);
    sh_begin(sh, SH_SEARCH);
    if (is_root && sh->e->timing) cudaEventRecord(sh->ev[2 * SH_GATHER], sh->cs);
    for (int c = 0; c < m; ++c) {
        const int q0 = cb[c], q1 = cb[c + 1], n_c = q1 - q0;
        const size_t off = (size_t)K * (q0 - b0);  // chunk c's [K, n_c] block in this rank's output
        int* oi = e->out_idx.as<int>() + off;
        float* od = e->out_dist.as<float>() + off;
        if (n_c > 0) {
            if (path == FRNN_PATH_GRID)
                st = search_built(e, P, H.principal != 0, K, r2, q0, q1, false, oi, od);
            else if (path == FRNN_PATH_BRUTE_TC)
                st = tc_query_tiles(e, pts, N, dim, K, radius, oi, od, q0 / 128, (q1 + 127) / 128);
            else {
                FRNN_CHECK(e, launch_bruteforce(pts, N, dim, K, r2, q0, q1, oi, od, n_c, s), "bruteforce launch");
                e->launches++;
            }
            if (st != FRNN_OK) return st;
        }
        FRNN_CHECK(e, cudaEventRecord(sh->chunk_ev[c], s), "chunk event");
        FRNN_CHECK(e, cudaStreamWaitEvent(sh->cs, sh->chunk_ev[c], 0), "chunk wait");
        if (is_root) {
            // chunk c of every other rank's slice, then this rank's own
            SH_NCCL(sh, api->GroupStart(), "group start");
            for (int r = 0; r < parts; ++r) {
                int rc[kMaxChunks + 1];
                const int mr = chunk_bounds(H.bounds[r], H.bounds[r + 1], path, sh->chunks, rc);
                if (r == root || c >= mr || rc[c + 1] == rc[c]) continue;
                const size_t o = (size_t)K * rc[c], cnt = (size_t)K * (rc[c + 1] - rc[c]);
                SH_NCCL(sh, api->Recv(sh->st_idx.as<int>() + o, cnt, ncclInt32, r, sh->comm, sh->cs), "idx receive");
                SH_NCCL(sh, api->Recv(sh->st_dist.as<float>() + o, cnt, ncclFloat32, r, sh->comm, sh->cs),
                        "dist receive");
                sh->gather_bytes += (long long)cnt * 8;
            }
            SH_NCCL(sh, api->GroupEnd(), "group end");
            for (int r = 0; r < parts; ++r) {
                int rc[kMaxChunks + 1];
                const int mr = chunk_bounds(H.bounds[r], H.bounds[r + 1], path, sh->chunks, rc);
                if (c >= mr) continue;
                const int n_rc = rc[c + 1] - rc[c];
                const int* si = r == root ? oi : sh->st_idx.as<int>() + (size_t)K * rc[c];
                const float* sd = r == root ? od : sh->st_dist.as<float>() + (size_t)K * rc[c];
                FRNN_CHECK(e, launch_shard_scatter(si, sd, rc[c], n_rc, K, scatter_ids, N, sh->res_idx.as<int>(),
                                                   sh->res_dist.as<float>(), sh->cs),
                           "scatter launch");
                if (n_rc > 0) e->launches++;
            }
        } else if (n_c > 0) {
            const size_t cnt = (size_t)K * n_c;
            SH_NCCL(sh, api->GroupStart(), "group start");
            SH_NCCL(sh, api->Send(oi, cnt, ncclInt32, root, sh->comm, sh->cs), "idx send");
            SH_NCCL(sh, api->Send(od, cnt, ncclFloat32, root, sh->comm, sh->cs), "dist send");
            SH_NCCL(sh, api->GroupEnd(), "group end");
            sh->gather_bytes += (long long)cnt * 8;
        }
    }
    if (is_root) {
        // chunks of other slices beyond this rank's own chunk count
        int mmax = m;
        for (int r = 0; r < parts; ++r) {
            int rc[kMaxChunks + 1];
            mmax = std::max(mmax, chunk_bounds(H.bounds[r], H.bounds[r + 1], path, sh->chunks, rc));
        }
        for (int c = m; c < mmax; ++c) {
            SH_NCCL(sh, api->GroupStart(), "group start");
            for (int r = 0; r < parts; ++r) {
                int rc[kMaxChunks + 1];
                const int mr = chunk_bounds(H.bounds[r], H.bounds[r + 1], path, sh->chunks, rc);
                if (r == root || c >= mr || rc[c + 1] == rc[c]) continue;
                const size_t o = (size_t)K * rc[c], cnt = (size_t)K * (rc[c + 1] - rc[c]);
                SH_NCCL(sh, api->Recv(sh->st_idx.as<int>() + o, cnt, ncclInt32, r, sh->comm, sh->cs), "idx receive");
                SH_NCCL(sh, api->Recv(sh->st_dist.as<float>() + o, cnt, ncclFloat32, r, sh->comm, sh->cs),
                        "dist receive");
                sh->gather_bytes += (long long)cnt * 8;
            }
            SH_NCCL(sh, api->GroupEnd(), "group end");
            for (int r = 0; r < parts; ++r) {
                int rc[kMaxChunks + 1];
                const int mr = chunk_bounds(H.bounds[r], H.bounds[r + 1], path, sh->chunks, rc);
                if (r == root || c >= mr) continue;
                FRNN_CHECK(e, launch_shard_scatter(sh->st_idx.as<int>() + (size_t)K * rc[c],
                                                   sh->st_dist.as<float>() + (size_t)K * rc[c], rc[c],
                                                   rc[c + 1] - rc[c], K, scatter_ids, N, sh->res_idx.as<int>(),
                                                   sh->res_dist.as<float>(), sh->cs),
                           "scatter launch");
                e->launches++;
            }
        }
    }
    sh_end(sh, SH_SEARCH);
    if (is_root && sh->e->timing) {
        cudaEventRecord(sh->ev[2 * SH_GATHER + 1], sh->cs);
        sh->ev_used[SH_GATHER] = true;
    }
    // the engine stream waits for the communication stream's work
    FRNN_CHECK(e, cudaEventRecord(sh->comm_done, sh->cs), "comm event");
    FRNN_CHECK(e, cudaStreamWaitEvent(s, sh->comm_done, 0), "comm wait");
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
