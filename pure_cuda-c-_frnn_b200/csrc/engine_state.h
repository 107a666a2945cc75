// engine_state.h -- the engine object and the helpers its .cu files share.
// Internal to the library (the public ABI is include/frnn_b200.h).
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "frnn_b200.h"
#include "frnn_device.cuh"

namespace frnn {
namespace eng {

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    template <class T>
    T* as() const { return static_cast<T*>(p); }
};

constexpr int kBoxMaxBlocks = 1024;
// bbox, hash, scan, scatter, search, unpermute, brute force, collect, emit,
// tensor-core prep, tensor-core filter, exact re-rank
#define FRNN_STAGES 12

}  // namespace eng
}  // namespace frnn

struct frnn_engine {
    int device = 0;
    int max_points = 0;
    int sms = 148;
    cudaStream_t stream = 0;
    int forced_path = FRNN_PATH_AUTO;
    unsigned epoch = 0;
    long long direct_output_max_bytes = 48LL << 20;

    frnn::eng::DevBuf box_partial, box_ticket, box_out;
    frnn::eng::DevBuf counts, starts, scan_status, scan_ticket, err_flag;
    frnn::eng::DevBuf cellrank, rows, ids, inv;
    frnn::eng::DevBuf lists, list_counts, overflow, n_overflow;
    frnn::eng::DevBuf tmp_idx, tmp_dist, out_idx, out_dist;
    frnn::eng::DevBuf in_stage, in_soa, out_rm_idx, out_rm_dist;
    frnn::eng::DevBuf tc_box, tc_center, tc_tiles, tc_rows, tc_qa, tc_pb;
    frnn::eng::DevBuf part_ids;          // original query index of each row of a part search
    // principal-axis grid: moments, axes, projected coordinates, estimate
    frnn::eng::DevBuf pca_partial, pca_moments, pca_mu, pca_pm, proj_box_partial, proj_ticket, proj_out;
    frnn::eng::DevBuf proj_u, proj_s, pca_smp, pca_h, pca_counts;
    // a separate query set: its grid (same plan as the points), projected
    // coordinates and tensor-core tiles
    frnn::eng::DevBuf q_counts, q_starts, q_cellrank, q_rows, q_ids, q_inv, q_proj_u, q_proj_s, q_proj_partial,
        q_proj_out, q_box_out;
    frnn::eng::DevBuf q_tiles, q_rows32, q_qa, q_pb;
    void* h_pca = nullptr;    // pinned, 32 KiB
    int grid_axes_mode = 0;   // FRNN_OPT_GRID_AXES
    int list_search = 0;      // FRNN_OPT_LIST_SEARCH
    int test_stall = 0;       // FRNN_OPT_TEST_STALL (tests of the timeout path)
    int device_plan = 1;      // FRNN_OPT_DEVICE_PLAN
    int tc_symmetric = 1;     // FRNN_OPT_TC_SYMMETRIC
    // device-planned grids: the plan (written by the bounding-box kernel) and
    // its pinned host copy
    frnn::eng::DevBuf dplan;
    void* h_plan = nullptr;   // pinned, one GridPlan
    // a point set kept for frnn_query_grid: on the grid path its sorted rows,
    // ids, cell starts (and projected coordinates) stay in the point buffers
    struct {
        bool valid = false;
        const float* pts = nullptr;
        int N = 0, dim = 0, path = 0;
        float radius = 0.0f;
        bool principal = false;
        double proj_delta = 0.0;
        frnn::GridPlan P{};
    } built;
    int last_principal = 0;   // the last grid was on principal axes
    // rounding bounds of the points' / last query set's projected coordinates
    double proj_delta = 0.0, q_proj_delta = 0.0;
    int last_part_rows = -1;  // rows of the last part search (-1: last search was whole)
    // what the overflow list of the last search holds: 0 nothing (no list
    // search ran), 1 the points' sorted positions (original index = ids[]),
    // 2 query indices, 3 a query set's sorted positions (index = q_ids[])
    int last_overflow_map = 0;
    frnn::eng::DevBuf ovf_ids;
    float* h_box = nullptr;   // pinned, 9 floats
    float* h_tc = nullptr;    // pinned, 512 floats: per-dimension box + flag, then the centre
    int* h_err = nullptr;     // pinned

    int last_N = -1, last_K = -1;
    int last_path = 0, last_g = 0;
    long long last_cells = 0;
    std::string last_error;

    // per-stage device timing (frnn_set_timing); stage s spans events
    // ev[2s] .. ev[2s+1] on the engine stream
    bool timing = false;
    cudaEvent_t ev[2 * FRNN_STAGES] = {};
    bool stage_used[FRNN_STAGES] = {};
    long long launches = 0;
};

namespace frnn {
namespace eng {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// Record msg as the engine's last error and return status.
int fail(frnn_engine* e, int status, const std::string& msg);
// A failed CUDA call: FRNN_ERR_OOM for allocation failures, else FRNN_ERR_CUDA.
int cuda_fail(frnn_engine* e, cudaError_t err, const char* what);
// Grow b to at least `bytes` (contents are not kept).
int grow(frnn_engine* e, DevBuf& b, size_t bytes, const char* what);

#define FRNN_CHECK(e, call, what)                                   \
    do {                                                            \
        cudaError_t err__ = (call);                                 \
        if (err__ != cudaSuccess) return frnn::eng::cuda_fail(e, err__, what); \
    } while (0)

#define FRNN_GROW(e, buf, bytes)                                    \
    do {                                                            \
        int st__ = frnn::eng::grow(e, buf, bytes, #buf);            \
        if (st__ != FRNN_OK) return st__;                           \
    } while (0)

enum Stage {
    ST_BBOX = 0, ST_HASH, ST_SCAN, ST_SCATTER, ST_SEARCH, ST_UNPERMUTE, ST_BRUTE, ST_COLLECT, ST_EMIT,
    ST_TC_PREP, ST_TC_FILTER, ST_TC_RERANK
};
void stage_begin(frnn_engine* e, int st);
void stage_end(frnn_engine* e, int st);

// ---- pieces of a self-search (engine.cu), shared with the sharded search ----

// Argument checks of a search entry point (status, with the last error set).
int check_search_args(frnn_engine* e, const void* pts, int N, int dim, int K, float radius);
int check_device_ptr(frnn_engine* e, const void* p);
// The dispatcher's path for a self-search of N points in dim dimensions
// (before any grid is planned): FRNN_PATH_GRID, _BRUTE or _BRUTE_TC.
int self_search_path(const frnn_engine* e, int N, int dim);
// Grid path: bounding box (read back), plan, principal axes when they pay; the
// projected coordinates are then in e->proj_u.  *path becomes
// FRNN_PATH_BRUTE when no useful grid exists.
int plan_grid_search(frnn_engine* e, const float* d_pts, int N, int dim, float radius, int* path,
                     frnn::GridPlan& P, bool* principal);
// Whether a grid search with K neighbours uses candidate lists (collect + emit).
bool uses_lists(const frnn_engine* e, const frnn::GridPlan& P, int K, bool principal);
// Cell histogram, prefix scan and counting-sort scatter of the P.n points into
// e->counts / starts / rows / ids (inv when with_inv, proj_s when proj).
int build_points(frnn_engine* e, const float* d_pts, const frnn::GridPlan& P, const float* proj,
                 bool with_inv);
// Search the built points' sorted positions [q0, q1).  whole: every query,
// out[k*N + q] in original order (needs inv when lists are used); otherwise
// row j = sorted position q0 + j of out[k*(q1-q0) + j].
// Pd (optional): the plan as the GPU made it (run_grid_dplan); P then
// carries only what the host knows before the box (n, dim, g, row).
int search_built(frnn_engine* e, const frnn::GridPlan& P, bool principal, int K, float r2, int q0, int q1,
                 bool whole, int* out_idx, float* out_dist, const frnn::GridPlan* Pd = nullptr);

// Tensor-core brute force: the host-side plan (centre, scale, thresholds)
// and the device work for query tiles [qb_begin, qb_end).
struct TcPlan {
    bool ok = false;
    float scale = 1.0f, one_minus_alpha = 1.0f, eta_c = 0.0f, rc = 0.0f;
    float center[kMaxD] = {};
};
int tc_plan(frnn_engine* e, const float* d_pts, int N, int dim, float radius, TcPlan* tp,
            const float* d_q = nullptr, int M = 0);
int tc_search(frnn_engine* e, const float* d_pts, int N, int dim, int K, float radius, const TcPlan& tp,
              int* out_idx, float* out_dist, int qb_begin, int qb_end, const float* d_q = nullptr, int M = 0);
// tc_search in two steps: the tiles and rows of every point (and query) once,
// then any number of query-tile ranges.
int tc_prepare(frnn_engine* e, const float* d_pts, int N, int dim, const TcPlan& tp, const float* d_q = nullptr,
               int M = 0);
int tc_query_tiles(frnn_engine* e, const float* d_pts, int N, int dim, int K, float radius, int* out_idx,
                   float* out_dist, int qb_begin, int qb_end, const float* d_q = nullptr, int M = 0);

}  // namespace eng
}  // namespace frnn
