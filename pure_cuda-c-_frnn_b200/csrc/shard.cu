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
//      scale.  Rank r owns the queries of one range of ORIGINAL indices, so
//      its results are one contiguous column block of the [K, N] output.  On
//      the grid path the ranges are cut so that every rank gets the same
//      estimated work: the candidates of every 64th cell-sorted query (the
//      point count of its 3^g shell, what a search scans) are summed into
//      4,096 buckets of original index, and frnn_shard_partition cuts them;
//   2. header broadcast (plan, sizes, ranges, the root's status and the IPC
//      handles of its result buffers), then an all-reduce of every rank's
//      status, so that a rank that cannot take part makes every rank return
//      the same error instead of waiting;
//   3. data broadcast in one NCCL group: the cell-sorted rows, their ids, the
//      cell starts (and the sorted projected coordinates of a principal-axis
//      grid); on the brute-force paths the cloud itself (every rank then
//      prepares its own fp16 tiles from it);
//   4. every rank searches its queries in cell order (the grid path lists
//      their sorted positions with a scan), writing rows in original order;
//      on the tensor-core path the ranks share the symmetric filter (each
//      unordered pair of tiles once): rank r filters its query blocks
//      against the tiles at or above them, keeping every passing pair, from
//      either side, in its own lists; after a barrier each rank pulls the
//      entries the other ranks listed for its queries (plain loads from
//      their lists, mapped through CUDA IPC) and re-ranks its own queries;
//   5. each rank's block goes straight into the root's result buffers with
//      a 2-D copy over NVLink on a copy engine (the root's buffers are mapped
//      through CUDA IPC); no SM takes part in the gather, so with several
//      chunks per rank the copy of one chunk overlaps the search of the
//      next.  A final all-reduce on every rank's stream, after its copies,
//      tells the root that every block has landed.
//
// Every wait on the host is bounded (FRNN_ERR_TIMEOUT after the shard's
// timeout; the communicator is then aborted and the shard unusable); an NCCL
// error reported by the communicator ends the call with FRNN_ERR_COMM.
// Apart from the symmetric filter's pull (loads only), no kernel here touches
// another GPU's memory; the gather's writes to the root are copy-engine
// copies.
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
    int tc_sym;          // the tensor-core filter is shared symmetrically
    cudaIpcMemHandle_t res_idx, res_dist;  // the root's result buffers
    int bounds[kMaxShardRanks + 1];  // rank r owns original query indices [bounds[r], bounds[r+1])
};
static_assert(std::is_trivially_copyable<ShardHeader>::value, "sent as bytes");

// stages timed when the engine's timing is on: the root's plan and build, the
// header and status exchange, the data broadcast, the rank's search (engine
// stream), its copies into the root's buffers (communication stream)
enum ShardStage { SH_BUILD = 0, SH_HEADER, SH_BCAST, SH_SEARCH, SH_GATHER, SH_STAGES };

// Chunks of a rank's range: each is searched, then copied to the root while
// the next one is searched.  Chunks hold at least kChunkMin queries.
constexpr int kMaxChunks = 8;
constexpr int kChunkMin = 65536;
// Every kSampleStride-th cell-sorted query samples the search work, summed
// into kWorkBuckets ranges of original index.
constexpr int kSampleStride = 64;
constexpr int kWorkBuckets = 4096;

// Chunk c of the range [b0, b1) is [cb[c], cb[c+1]); on the tensor-core path
// every cut is a multiple of 128 (whole query tiles).
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
    DevBuf d_hdr, d_stat, work, pts, res_idx, res_dist;
    // the grid path's per-rank query lists: original -> sorted position, the
    // range's flags and their prefix, the sorted positions of each chunk
    DevBuf inv, flags, fpos, fstatus, qlist;
    unsigned fepoch = 0;
    ShardHeader* h_hdr = nullptr;   // pinned
    int* h_stat = nullptr;          // pinned, 16 ints
    uint64_t* h_work = nullptr;     // pinned, kWorkBuckets
    int* h_wstart = nullptr;        // pinned, kWorkBuckets
    cudaStream_t cs = nullptr;      // communication stream (the copies to the root)
    int chunks = 1;                 // FRNN_SHARD_OPT_CHUNKS
    int comm_priority = 0;          // FRNN_SHARD_OPT_COMM_PRIORITY
    cudaEvent_t chunk_ev[kMaxChunks] = {}, comm_done = nullptr;
    cudaEvent_t ev[2 * SH_STAGES] = {};
    bool ev_used[SH_STAGES] = {};
    // the root's result buffers as mapped on this rank (other ranks)
    cudaIpcMemHandle_t open_h_idx{}, open_h_dist{};
    int* peer_idx = nullptr;
    float* peer_dist = nullptr;
    // the symmetric tensor-core filter (FRNN_SHARD_OPT_TC_SYMMETRIC): every
    // rank's candidate lists and counters, exchanged as IPC handles (slot r
    // of the exchange buffer is rank r's) and mapped here
    int tc_sym = 1;
    DevBuf d_handles;
    unsigned char* h_handles = nullptr;  // pinned
    cudaIpcMemHandle_t open_lists[kTcMaxPeers]{}, open_counts[kTcMaxPeers]{};
    int* peer_lists[kTcMaxPeers] = {};
    int* peer_counts[kTcMaxPeers] = {};
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

void sh_begin(frnn_shard* sh, int st, cudaStream_t s) {
    if (sh->e->timing) cudaEventRecord(sh->ev[2 * st], s);
}
void sh_end(frnn_shard* sh, int st, cudaStream_t s) {
    if (sh->e->timing) {
        cudaEventRecord(sh->ev[2 * st + 1], s);
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

// The work of the cell-sorted queries, sampled: for sorted position
// i * stride, the points in its cell's 3^g shell (the x-merged rows a grid
// search walks) plus a fixed charge per row, for the stride queries from
// there, added to the bucket of the sample's original index.
__global__ void sample_work_kernel(const float* __restrict__ rows, const float* __restrict__ proj_s,
                                   const int* __restrict__ starts, const int* __restrict__ ids, GridPlan P,
                                   int stride, int nsamples, unsigned long long* __restrict__ bucket_work) {
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
    const long long q = __ldg(&ids[sq]);
    if ((unsigned long long)q >= (unsigned long long)P.n) return;  // only after a scan gave up
    const int b = (int)(q * kWorkBuckets / P.n);
    atomicAdd(&bucket_work[b], (total + 8ull * nrows) * (unsigned long long)min((long long)stride, (long long)P.n - sq));
}

// inv[ids[sq]] = sq: each query's sorted position
__global__ void inv_kernel(const int* __restrict__ ids, int n, int* __restrict__ inv) {
    const int sq = blockIdx.x * blockDim.x + threadIdx.x;
    if (sq >= n) return;
    const int q = __ldg(&ids[sq]);
    if ((unsigned)q < (unsigned)n) inv[q] = sq;
}

// flags[sq] = 1 when the query at sorted position sq has an original index in [lo, hi)
__global__ void range_flags_kernel(const int* __restrict__ ids, int n, int lo, int hi, int* __restrict__ flags) {
    const int sq = blockIdx.x * blockDim.x + threadIdx.x;
    if (sq >= n) return;
    const int q = __ldg(&ids[sq]);
    flags[sq] = (q >= lo && q < hi) ? 1 : 0;
}

// qlist[pos[sq]] = sq for every flagged sq (pos: exclusive prefix of flags;
// at most cap entries)
__global__ void compact_kernel(const int* __restrict__ flags, const int* __restrict__ pos, int n, int cap,
                               int* __restrict__ qlist) {
    const int sq = blockIdx.x * blockDim.x + threadIdx.x;
    if (sq >= n || !__ldg(&flags[sq])) return;
    const int p = __ldg(&pos[sq]);
    if ((unsigned)p < (unsigned)cap) qlist[p] = sq;
}

// Step 1 on the root: plan, build and the owners' ranges into h_hdr.
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
    for (int r = 0; r <= parts; ++r) H.bounds[r] = (int)((long long)N * r / parts);
    if (H.path == FRNN_PATH_GRID) {
        cudaStream_t s = e->stream;
        int st = build_points(e, d_pts, H.P, H.principal ? e->proj_u.as<float>() : nullptr, false);
        if (st != FRNN_OK) return st;
        if (parts > 1) {
            const int ns = (N + kSampleStride - 1) / kSampleStride;
            FRNN_GROW(e, sh->work, (size_t)kWorkBuckets * 8);
            FRNN_CHECK(e, cudaMemsetAsync(sh->work.p, 0, (size_t)kWorkBuckets * 8, s), "memset work");
            sample_work_kernel<<<(ns + 127) / 128, 128, 0, s>>>(
                e->rows.as<float>(), H.principal ? e->proj_s.as<float>() : nullptr, e->starts.as<int>(),
                e->ids.as<int>(), H.P, kSampleStride, ns, sh->work.as<unsigned long long>());
            FRNN_CHECK(e, cudaGetLastError(), "work sample launch");
            e->launches++;
            FRNN_CHECK(e, cudaMemcpyAsync(sh->h_work, sh->work.p, (size_t)kWorkBuckets * 8, cudaMemcpyDeviceToHost, s),
                       "work readback");
            FRNN_CHECK(e, cudaMemcpyAsync(sh->h_stat, e->err_flag.p, sizeof(int), cudaMemcpyDeviceToHost, s),
                       "error flag readback");
            FRNN_CHECK(e, cudaStreamSynchronize(s), "partition sync");
            if (sh->h_stat[0] != 0) {
                cudaMemsetAsync(e->err_flag.p, 0, sizeof(int), s);
                cudaStreamSynchronize(s);
                return fail(e, FRNN_ERR_TIMEOUT, "a bounded device-side wait gave up");
            }
            for (int b = 0; b < kWorkBuckets; ++b) sh->h_wstart[b] = (int)((long long)N * b / kWorkBuckets);
            if (frnn_shard_partition(sh->h_work, sh->h_wstart, kWorkBuckets, N, parts, H.bounds) != FRNN_OK)
                return fail(e, FRNN_ERR_INVALID_ARG, "partition failed");
        }
    } else if (H.path == FRNN_PATH_BRUTE_TC) {
        H.tc_sym = sh->tc_sym && e->tc_symmetric && parts > 1 && parts <= kTcMaxPeers ? 1 : 0;
        if (H.tc_sym) {
            frnn_shard_tc_partition(N, parts, H.bounds);
        } else {
            // whole 128-query tiles; every query costs the same
            const int ntq = (N + 127) / 128;
            for (int r = 0; r <= parts; ++r) H.bounds[r] = std::min(N, (int)((long long)ntq * r / parts) * 128);
        }
    }
    // the results land in these buffers, on this GPU and (mapped) on the others
    FRNN_GROW(e, sh->res_idx, (size_t)N * K * 4);
    FRNN_GROW(e, sh->res_dist, (size_t)N * K * 4);
    if (parts > 1) {
        FRNN_CHECK(e, cudaIpcGetMemHandle(&H.res_idx, sh->res_idx.p), "result handle");
        FRNN_CHECK(e, cudaIpcGetMemHandle(&H.res_dist, sh->res_dist.p), "result handle");
    }
    return FRNN_OK;
}

// The root's result buffers on this (non-root) rank, mapped through IPC; the
// mapping is renewed when the root reallocated them.
int map_root_results(frnn_shard* sh, const ShardHeader& H) {
    if (sh->peer_idx && !std::memcmp(&sh->open_h_idx, &H.res_idx, sizeof(H.res_idx)) &&
        !std::memcmp(&sh->open_h_dist, &H.res_dist, sizeof(H.res_dist)))
        return FRNN_OK;
    if (sh->peer_idx) cudaIpcCloseMemHandle(sh->peer_idx);
    if (sh->peer_dist) cudaIpcCloseMemHandle(sh->peer_dist);
    sh->peer_idx = nullptr;
    sh->peer_dist = nullptr;
    void* pi = nullptr;
    void* pd = nullptr;
    FRNN_CHECK(sh->e, cudaIpcOpenMemHandle(&pi, H.res_idx, cudaIpcMemLazyEnablePeerAccess), "map root results");
    cudaError_t err = cudaIpcOpenMemHandle(&pd, H.res_dist, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) {
        cudaIpcCloseMemHandle(pi);
        return cuda_fail(sh->e, err, "map root results");
    }
    sh->peer_idx = static_cast<int*>(pi);
    sh->peer_dist = static_cast<float*>(pd);
    sh->open_h_idx = H.res_idx;
    sh->open_h_dist = H.res_dist;
    return FRNN_OK;
}

// The sorted positions of the queries with original index in [lo, hi), in
// increasing order, to qlist (hi - lo entries): flags, a scan, a compaction.
int range_queries(frnn_shard* sh, const int* ids, int N, int lo, int hi, int* qlist) {
    frnn_engine* e = sh->e;
    cudaStream_t s = e->stream;
    const long long tiles = scan_tiles(N);
    FRNN_GROW(e, sh->flags, (size_t)N * 4);
    FRNN_GROW(e, sh->fpos, ((size_t)N + 1) * 4);
    const size_t before = sh->fstatus.bytes;
    FRNN_GROW(e, sh->fstatus, (size_t)tiles * 8 + 16);
    // status words carry the scan's epoch; new memory could hold words of the
    // same epoch, so it is cleared first (as for the engine's own scan)
    if (sh->fstatus.bytes != before) FRNN_CHECK(e, cudaMemsetAsync(sh->fstatus.p, 0, sh->fstatus.bytes, s), "memset");
    sh->fepoch = (sh->fepoch + 1) & 0x3fffffffu;
    if (sh->fepoch == 0) {
        FRNN_CHECK(e, cudaMemsetAsync(sh->fstatus.p, 0, sh->fstatus.bytes, s), "memset");
        sh->fepoch = 1;
    }
    int* ticket = reinterpret_cast<int*>(static_cast<char*>(sh->fstatus.p) + (size_t)tiles * 8);
    FRNN_CHECK(e, cudaMemsetAsync(ticket, 0, 4, s), "memset ticket");
    range_flags_kernel<<<(N + 255) / 256, 256, 0, s>>>(ids, N, lo, hi, sh->flags.as<int>());
    FRNN_CHECK(e, cudaGetLastError(), "flags launch");
    FRNN_CHECK(e, launch_scan(sh->flags.as<int>(), sh->fpos.as<int>(), N, sh->fstatus.as<unsigned long long>(), ticket,
                              sh->fepoch, e->err_flag.as<int>(), s),
               "range scan launch");
    compact_kernel<<<(N + 255) / 256, 256, 0, s>>>(sh->flags.as<int>(), sh->fpos.as<int>(), N, hi - lo, qlist);
    FRNN_CHECK(e, cudaGetLastError(), "compact launch");
    e->launches += 3;
    return FRNN_OK;
}

// The symmetric filter's set-up, on every rank: its candidate lists (all N
// points: pairs seen from any point it owns may come from other ranks) and
// counters, zeroed; every rank's IPC handles of both, exchanged with one
// all-reduce (MAX over bytes, every rank filling its own slot) and mapped;
// then an all-reduce of the ranks' status, so that every rank stops together
// when one cannot take part.
int tc_sym_setup(frnn_shard* sh, const ShardHeader& H, int cap) {
    frnn_engine* e = sh->e;
    cudaStream_t s = e->stream;
    const NcclApi* api = nccl_api();
    const size_t slot = 2 * sizeof(cudaIpcMemHandle_t), nbytes = slot * (size_t)sh->nranks;
    int local = FRNN_OK;
    if ((local = grow(e, e->lists, (size_t)H.N * cap * 4, "lists")) == FRNN_OK &&
        (local = grow(e, e->list_counts, (size_t)H.N * 4, "list_counts")) == FRNN_OK &&
        (local = grow(e, e->overflow, (size_t)H.N * 4, "overflow")) == FRNN_OK &&
        (local = grow(e, e->n_overflow, 16, "n_overflow")) == FRNN_OK)
        local = grow(e, sh->d_handles, slot * kTcMaxPeers, "handles");
    std::memset(sh->h_handles, 0, slot * kTcMaxPeers);
    if (local == FRNN_OK) {
        cudaIpcMemHandle_t* mine = reinterpret_cast<cudaIpcMemHandle_t*>(sh->h_handles + slot * sh->rank);
        if (cudaMemsetAsync(e->list_counts.p, 0, (size_t)H.N * 4, s) != cudaSuccess ||
            cudaMemsetAsync(e->n_overflow.p, 0, 4, s) != cudaSuccess ||
            cudaIpcGetMemHandle(&mine[0], e->lists.p) != cudaSuccess ||
            cudaIpcGetMemHandle(&mine[1], e->list_counts.p) != cudaSuccess)
            local = cuda_fail(e, cudaGetLastError(), "symmetric filter set-up");
    }
    if (sh->d_handles.p == nullptr) return local;  // cannot take part in the exchange at all
    FRNN_CHECK(e, cudaMemcpyAsync(sh->d_handles.p, sh->h_handles, nbytes, cudaMemcpyHostToDevice, s), "handles upload");
    SH_NCCL(sh, api->AllReduce(sh->d_handles.p, sh->d_handles.p, nbytes, ncclUint8, ncclMax, sh->comm, s),
            "handle exchange");
    FRNN_CHECK(e, cudaMemcpyAsync(sh->h_handles, sh->d_handles.p, nbytes, cudaMemcpyDeviceToHost, s),
               "handles readback");
    int st = wait_stream(sh, "handle exchange");
    if (st != FRNN_OK) return st;
    for (int r = 0; r < sh->nranks && local == FRNN_OK; ++r) {
        if (r == sh->rank) continue;
        const cudaIpcMemHandle_t* h = reinterpret_cast<const cudaIpcMemHandle_t*>(sh->h_handles + slot * r);
        for (int b = 0; b < 2 && local == FRNN_OK; ++b) {
            cudaIpcMemHandle_t& open = b ? sh->open_counts[r] : sh->open_lists[r];
            int*& ptr = b ? sh->peer_counts[r] : sh->peer_lists[r];
            if (ptr && !std::memcmp(&open, &h[b], sizeof(open))) continue;
            if (ptr) cudaIpcCloseMemHandle(ptr);
            ptr = nullptr;
            void* p = nullptr;
            const cudaError_t err = cudaIpcOpenMemHandle(&p, h[b], cudaIpcMemLazyEnablePeerAccess);
            if (err != cudaSuccess) {
                local = cuda_fail(e, err, "map another rank's candidate lists");
                break;
            }
            ptr = static_cast<int*>(p);
            open = h[b];
        }
    }
    sh->h_stat[3] = local;
    FRNN_CHECK(e, cudaMemcpyAsync(sh->d_stat.p, sh->h_stat + 3, sizeof(int), cudaMemcpyHostToDevice, s),
               "status upload");
    SH_NCCL(sh, api->AllReduce(sh->d_stat.p, sh->d_stat.p, 1, ncclInt32, ncclMax, sh->comm, s), "status all-reduce");
    FRNN_CHECK(e, cudaMemcpyAsync(sh->h_stat + 4, sh->d_stat.p, sizeof(int), cudaMemcpyDeviceToHost, s),
               "status readback");
    st = wait_stream(sh, "symmetric filter set-up");
    if (st != FRNN_OK) return st;
    if (sh->h_stat[4] != FRNN_OK) {
        if (local == FRNN_OK) fail(e, sh->h_stat[4], "another rank could not set up the symmetric filter");
        return sh->h_stat[4];
    }
    return FRNN_OK;
}

// This rank's part of the symmetric filter over its query blocks, a barrier
// (one all-reduce: every rank's filter has finished), then its own queries
// [lo, hi): the other ranks' entries for them pulled in, the overflow list,
// the exact re-rank and the SIMT brute force for overflowing lists.  Every
// rank runs it, also one with no queries.
int tc_sym_range(frnn_shard* sh, const ShardHeader& H, const float* pts, int lo, int hi, int cap, int* oi,
                 float* od) {
    frnn_engine* e = sh->e;
    cudaStream_t s = e->stream;
    const NcclApi* api = nccl_api();
    const int N = H.N, K = H.K, dim = H.dim, rows = hi - lo;
    const float r2 = H.radius * H.radius;
    TcPeers peers;
    peers.n = sh->nranks;
    for (int r = 0; r < sh->nranks; ++r) {
        peers.counts[r] = r == sh->rank ? e->list_counts.as<int>() : sh->peer_counts[r];
        peers.lists[r] = r == sh->rank ? e->lists.as<int>() : sh->peer_lists[r];
    }
    if (rows > 0) {
        stage_begin(e, ST_TC_FILTER);
        FRNN_CHECK(e, launch_tc_filter(e->tc_tiles.as<uint8_t>(), e->tc_qa.as<float>(), e->tc_pb.as<float>(), N, dim,
                                       cap, e->lists.as<int>(), e->list_counts.as<int>(), e->overflow.as<int>(),
                                       e->n_overflow.as<int>(), e->err_flag.as<int>(), lo / 128, (hi + 127) / 128, s,
                                       nullptr, N, -1, true, true),
                   "filter launch");
        stage_end(e, ST_TC_FILTER);
        e->launches++;
    }
    SH_NCCL(sh, api->AllReduce(sh->d_stat.p, sh->d_stat.p, 1, ncclInt32, ncclMax, sh->comm, s), "filter barrier");
    if (rows <= 0) return FRNN_OK;
    FRNN_CHECK(e, launch_tc_pull(peers, sh->rank, e->list_counts.as<int>(), e->lists.as<int>(), lo, hi, cap, s),
               "pull launch");
    FRNN_CHECK(e, launch_tc_sym_overflow(e->list_counts.as<int>(), lo, hi, cap, e->overflow.as<int>(),
                                         e->n_overflow.as<int>(), s),
               "overflow launch");
    stage_begin(e, ST_TC_RERANK);
    FRNN_CHECK(e, launch_tc_rerank(e->tc_rows.as<float>(), dim, e->lists.as<int>(), e->list_counts.as<int>(), cap, N,
                                   K, r2, oi, od, lo, hi, s),
               "rerank launch");
    stage_end(e, ST_TC_RERANK);
    e->launches += 3;
    int* h_nov = sh->h_stat + 5;
    FRNN_CHECK(e, cudaMemcpyAsync(h_nov, e->n_overflow.p, sizeof(int), cudaMemcpyDeviceToHost, s),
               "overflow count readback");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "overflow count sync");
    if (*h_nov > 0) {
        stage_begin(e, ST_BRUTE);
        FRNN_CHECK(e, launch_bruteforce(pts, N, dim, K, r2, 0, *h_nov, oi, od, rows, s, e->overflow.as<int>(), lo),
                   "overflow brute force launch");
        stage_end(e, ST_BRUTE);
        e->launches++;
    }
    return FRNN_OK;
}

// Search the queries with original index in [lo, hi) (this rank's chunk),
// results row q - lo of out[k*(hi-lo) + row].
int search_range(frnn_shard* sh, const ShardHeader& H, const float* pts, int lo, int hi, int* oi, float* od) {
    frnn_engine* e = sh->e;
    cudaStream_t s = e->stream;
    const int N = H.N, K = H.K, dim = H.dim, rows = hi - lo;
    const float r2 = H.radius * H.radius;
    if (rows <= 0) return FRNN_OK;
    if (H.path == FRNN_PATH_BRUTE_TC)
        return tc_query_tiles(e, pts, N, dim, K, H.radius, oi, od, lo / 128, (hi + 127) / 128);
    if (H.path == FRNN_PATH_BRUTE) {
        FRNN_CHECK(e, launch_bruteforce(pts, N, dim, K, r2, lo, hi, oi, od, rows, s), "bruteforce launch");
        e->launches++;
        return FRNN_OK;
    }
    // grid: the range's sorted positions, then the search in cell order with
    // rows written in original order
    const GridPlan& P = H.P;
    const float* proj_s = H.principal ? e->proj_s.as<float>() : nullptr;
    const int* ids = e->ids.as<int>();
    int* qlist = sh->qlist.as<int>();
    int st = range_queries(sh, ids, N, lo, hi, qlist);
    if (st != FRNN_OK) return st;
    if (uses_lists(e, P, K, H.principal != 0)) {
        const int cap = K <= 16 ? 64 : 128;
        FRNN_GROW(e, e->lists, (size_t)N * cap * 8);
        FRNN_GROW(e, e->list_counts, (size_t)N * 4);
        FRNN_GROW(e, e->overflow, (size_t)N * 4);
        FRNN_GROW(e, e->n_overflow, 16);
        FRNN_CHECK(e, cudaMemsetAsync(e->n_overflow.p, 0, 4, s), "memset overflow count");
        const bool d3 = P.dim == 3 && P.g == 3 && !H.principal;
        // engine stages as in a single-GPU search (with several chunks the
        // last chunk's times remain)
        stage_begin(e, ST_COLLECT);
        if (d3)
            FRNN_CHECK(e, launch_collect_d3(e->rows.as<float>(), e->starts.as<int>(), P, r2, cap,
                                            e->lists.as<unsigned long long>(), e->list_counts.as<int>(),
                                            e->overflow.as<int>(), e->n_overflow.as<int>(), 0, rows, s, nullptr, qlist),
                       "collect launch");
        else
            FRNN_CHECK(e, launch_collect_nd(e->rows.as<float>(), ids, e->starts.as<int>(), P, r2, cap,
                                            e->lists.as<unsigned long long>(), e->list_counts.as<int>(),
                                            e->overflow.as<int>(), e->n_overflow.as<int>(), 0, rows, s, nullptr,
                                            proj_s, qlist),
                       "collect launch");
        stage_end(e, ST_COLLECT);
        stage_begin(e, ST_EMIT);
        // output row q - lo reads sorted position inv[q]
        FRNN_CHECK(e, launch_emit_lists(e->lists.as<unsigned long long>(), e->list_counts.as<int>(),
                                        sh->inv.as<int>() + lo, 0, rows, K, cap, r2, oi, od, s, N),
                   "emit launch");
        FRNN_CHECK(e, launch_grid_search(e->rows.as<float>(), ids, e->starts.as<int>(), P, K, r2, 0, N, oi, od, rows,
                                         ids, s, e->overflow.as<int>(), e->n_overflow.as<int>(), lo, proj_s),
                   "overflow search launch");
        stage_end(e, ST_EMIT);
        e->launches += 3;
        return FRNN_OK;
    }
    stage_begin(e, ST_SEARCH);
    FRNN_CHECK(e, launch_grid_search(e->rows.as<float>(), ids, e->starts.as<int>(), P, K, r2, 0, rows, oi, od, rows,
                                     ids, s, qlist, nullptr, lo, proj_s),
               "grid search launch");
    stage_end(e, ST_SEARCH);
    e->launches++;
    return FRNN_OK;
}

}  // namespace

extern "C" {

// Owners' ranges for the symmetric tensor-core filter: query block b filters
// the tiles t >= b, so block b costs T - b tiles, and its re-rank about
// kRerankTiles more (B200, cfg5: 15.5 ms of re-rank for 7,813 blocks against
// 177 ms of filter for 30.5M tiles); ranges are cut at even blocks (the
// filter's CTAs take blocks in pairs) so that every rank gets an equal share.
int frnn_shard_tc_partition(int N, int nparts, int* bounds) {
    if (!bounds || N < 0 || nparts < 1 || nparts > kMaxShardRanks) return FRNN_ERR_INVALID_ARG;
    constexpr double kRerankTiles = 0.35;
    const long long T = ((long long)N + 127) / 128, pairs = (T + 1) / 2;
    auto pair_work = [&](long long j) {
        return (long double)((T - 2 * j) + (2 * j + 1 < T ? T - 2 * j - 1 + kRerankTiles : 0.0)) + kRerankTiles;
    };
    long double total = 0.0L;
    for (long long j = 0; j < pairs; ++j) total += pair_work(j);
    bounds[0] = 0;
    long long j = 0;
    long double before = 0.0L;
    for (int r = 1; r < nparts; ++r) {
        const long double target = total * r / nparts;
        while (j < pairs && before + pair_work(j) <= target) before += pair_work(j++);
        if (j < pairs && target - before > 0.5L * pair_work(j)) before += pair_work(j++);
        bounds[r] = (int)std::min<long long>(N, j * 256);
    }
    bounds[nparts] = N;
    return FRNN_OK;
}

int frnn_shard_partition(const uint64_t* tile_work, const int* tile_start, int64_t tiles, int N, int nparts,
                         int* bounds) {
    if (!tile_work || !tile_start || !bounds || tiles < 1 || N < 0 || nparts < 1) return FRNN_ERR_INVALID_ARG;
    unsigned long long total = 0;
    for (int64_t t = 0; t < tiles; ++t) total += tile_work[t];
    bounds[0] = 0;
    bounds[nparts] = N;
    // boundary r sits at the tile edge nearest to the r/nparts quantile of the
    // cumulative work
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
        cudaMallocHost(&sh->h_stat, 64) != cudaSuccess ||
        cudaMallocHost(&sh->h_work, (size_t)kWorkBuckets * 8) != cudaSuccess ||
        cudaMallocHost(&sh->h_wstart, (size_t)kWorkBuckets * 4) != cudaSuccess ||
        cudaMallocHost(&sh->h_handles, 2 * sizeof(cudaIpcMemHandle_t) * kTcMaxPeers) != cudaSuccess) {
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
        if (sh->cs) cudaStreamSynchronize(sh->cs);
        const NcclApi* api = nccl_api();
        if (sh->comm && api) api->CommDestroy(sh->comm);
        if (sh->peer_idx) cudaIpcCloseMemHandle(sh->peer_idx);
        if (sh->peer_dist) cudaIpcCloseMemHandle(sh->peer_dist);
        for (int r = 0; r < kTcMaxPeers; ++r) {
            if (sh->peer_lists[r]) cudaIpcCloseMemHandle(sh->peer_lists[r]);
            if (sh->peer_counts[r]) cudaIpcCloseMemHandle(sh->peer_counts[r]);
        }
        for (DevBuf* b : {&sh->d_handles, &sh->d_hdr, &sh->d_stat, &sh->work, &sh->pts, &sh->res_idx, &sh->res_dist, &sh->inv,
                          &sh->flags, &sh->fpos, &sh->fstatus, &sh->qlist})
            if (b->p) cudaFree(b->p);
        if (sh->h_hdr) cudaFreeHost(sh->h_hdr);
        if (sh->h_stat) cudaFreeHost(sh->h_stat);
        if (sh->h_work) cudaFreeHost(sh->h_work);
        if (sh->h_wstart) cudaFreeHost(sh->h_wstart);
        if (sh->h_handles) cudaFreeHost(sh->h_handles);
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
        case FRNN_SHARD_OPT_TC_SYMMETRIC:
            if (value != 0 && value != 1) return fail(sh->e, FRNN_ERR_INVALID_ARG, "tc symmetric must be 0 or 1");
            sh->tc_sym = (int)value;
            return FRNN_OK;
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

    // 1. root: plan, build, owners' ranges
    ShardHeader& H = *sh->h_hdr;
    if (is_root) {
        std::memset(&H, 0, sizeof(H));
        H.N = N;
        H.dim = dim;
        H.K = K;
        H.radius = radius;
        H.nparts = parts;
        sh_begin(sh, SH_BUILD, s);
        H.status = local == FRNN_OK ? root_plan(sh, d_points_soa, N, dim, K, radius) : local;
        sh_end(sh, SH_BUILD, s);
        FRNN_CHECK(e, cudaMemcpyAsync(sh->d_hdr.p, &H, sizeof(H), cudaMemcpyHostToDevice, s), "header upload");
    }
    // 2. header, then every rank's status
    sh_begin(sh, SH_HEADER, s);
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
    const int lo = H.bounds[sh->rank], hi = H.bounds[sh->rank + 1], rows = hi - lo;
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
    if (local == FRNN_OK && path == FRNN_PATH_GRID) {
        if ((local = grow(e, sh->inv, (size_t)N * 4, "inv")) == FRNN_OK)
            local = grow(e, sh->qlist, (size_t)std::max(rows, 1) * 4, "qlist");
    }
    if (local == FRNN_OK && !is_root) local = map_root_results(sh, H);
    sh->h_stat[0] = local;
    FRNN_CHECK(e, cudaMemcpyAsync(sh->d_stat.p, sh->h_stat, sizeof(int), cudaMemcpyHostToDevice, s),
               "status upload");
    SH_NCCL(sh, api->AllReduce(sh->d_stat.p, sh->d_stat.p, 1, ncclInt32, ncclMax, sh->comm, s), "status all-reduce");
    FRNN_CHECK(e, cudaMemcpyAsync(sh->h_stat + 1, sh->d_stat.p, sizeof(int), cudaMemcpyDeviceToHost, s),
               "status readback");
    st = wait_stream(sh, "status all-reduce");
    if (st != FRNN_OK) return st;
    sh_end(sh, SH_HEADER, s);
    if (sh->h_stat[1] != FRNN_OK) {
        if (local == FRNN_OK) fail(e, sh->h_stat[1], "another rank could not take part in the sharded search");
        return sh->h_stat[1];
    }

    // 3. the data every rank searches
    sh_begin(sh, SH_BCAST, s);
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
    sh_end(sh, SH_BCAST, s);

    // 4 and 5. this rank's queries, chunk by chunk; each finished chunk is
    // copied into the root's result block on the communication stream (a copy
    // engine over NVLink) while the next chunk is searched
    const bool tc_sym = path == FRNN_PATH_BRUTE_TC && H.tc_sym;
    const int tc_cap = tc_list_cap(K);
    if (path == FRNN_PATH_BRUTE_TC && rows > 0) {
        st = tc_prepare(e, pts, N, dim, H.tc);
        if (st != FRNN_OK) return st;
    }
    if (tc_sym) {
        st = tc_sym_setup(sh, H, tc_cap);
        if (st != FRNN_OK) return st;
    }
    if (path == FRNN_PATH_GRID && rows > 0) {
        inv_kernel<<<(N + 255) / 256, 256, 0, s>>>(e->ids.as<int>(), N, sh->inv.as<int>());
        FRNN_CHECK(e, cudaGetLastError(), "inv launch");
        e->launches++;
    }
    int* dst_idx = is_root ? sh->res_idx.as<int>() : sh->peer_idx;
    float* dst_dist = is_root ? sh->res_dist.as<float>() : sh->peer_dist;
    int cb[kMaxChunks + 1];
    // the symmetric filter runs in one piece, on every rank (it holds barriers)
    const int m = tc_sym ? 1 : chunk_bounds(lo, hi, path, sh->chunks, cb);
    if (tc_sym) {
        cb[0] = lo;
        cb[1] = hi;
    }
    sh_begin(sh, SH_SEARCH, s);
    sh_begin(sh, SH_GATHER, sh->cs);
    for (int c = 0; c < m && (rows > 0 || tc_sym); ++c) {
        const int c0 = cb[c], c1 = cb[c + 1], n_c = c1 - c0;
        if (n_c <= 0 && !tc_sym) continue;
        const size_t off = (size_t)K * (c0 - lo);  // chunk c's [K, n_c] block in this rank's output
        int* oi = e->out_idx.as<int>() + off;
        float* od = e->out_dist.as<float>() + off;
        st = tc_sym ? tc_sym_range(sh, H, pts, c0, c1, tc_cap, oi, od) : search_range(sh, H, pts, c0, c1, oi, od);
        if (st != FRNN_OK) return st;
        if (n_c <= 0) continue;
        FRNN_CHECK(e, cudaEventRecord(sh->chunk_ev[c], s), "chunk event");
        FRNN_CHECK(e, cudaStreamWaitEvent(sh->cs, sh->chunk_ev[c], 0), "chunk wait");
        // [K, n_c] -> columns [c0, c1) of the root's [K, N] results
        FRNN_CHECK(e, cudaMemcpy2DAsync(dst_idx + c0, (size_t)N * 4, oi, (size_t)n_c * 4, (size_t)n_c * 4, (size_t)K,
                                        cudaMemcpyDeviceToDevice, sh->cs),
                   "result copy");
        FRNN_CHECK(e, cudaMemcpy2DAsync(dst_dist + c0, (size_t)N * 4, od, (size_t)n_c * 4, (size_t)n_c * 4, (size_t)K,
                                        cudaMemcpyDeviceToDevice, sh->cs),
                   "result copy");
        if (!is_root) sh->gather_bytes += (long long)n_c * K * 8;
    }
    sh_end(sh, SH_SEARCH, s);
    sh_end(sh, SH_GATHER, sh->cs);
    // every rank's copies precede its part of one last all-reduce, so the
    // root's all-reduce completes only when every block has landed
    FRNN_CHECK(e, cudaEventRecord(sh->comm_done, sh->cs), "comm event");
    FRNN_CHECK(e, cudaStreamWaitEvent(s, sh->comm_done, 0), "comm wait");
    SH_NCCL(sh, api->AllReduce(sh->d_stat.p, sh->d_stat.p, 1, ncclInt32, ncclMax, sh->comm, s), "completion");
    if (is_root)
        for (int r = 0; r < parts; ++r)
            if (r != root) sh->gather_bytes += (long long)(H.bounds[r + 1] - H.bounds[r]) * K * 8;
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
