// frnn_internal.h -- kernel launchers shared between the engine's .cu files.
// Not part of the public ABI (that is include/frnn_b200.h).
#pragma once

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include "frnn_device.cuh"

namespace frnn {

// grid_build.cu
int bbox_blocks(int n, int sms);
// plan_out (optional): the grid planned on the device from the box
// (plan_grid with dim, radius and at most max_cells cells); a plan with
// cells = 0 means no grid (pre_r2 = 1: the data hold NaN or Inf)
cudaError_t launch_bbox(const float* pts, int n, int g, float* partial, unsigned int* ticket,
                        float* out, int blocks, cudaStream_t s, GridPlan* plan_out = nullptr,
                        int dim = 0, float radius = 0.0f, long long max_cells = 0);
// proj (optional): the grid axes are proj[i*kProjStride + d] instead of the
// leading coordinates of pts.  Pd (optional, every launcher below): the plan
// made on the device, read by the kernel in place of P (the host's P then
// only needs n, dim, g and row); a device plan with cells = 0 makes the
// kernel do nothing.
cudaError_t launch_hash_count(const float* pts, const GridPlan& P, int* counts, int2* cellrank,
                              cudaStream_t s, const float* proj = nullptr, const GridPlan* Pd = nullptr);
long long scan_tiles(long long cells);
// withhold >= 0 makes that tile keep its status to itself, so the bounded
// look-back of the next tile gives up (tests of the timeout path only).
// With Pd, `cells` is the largest table the device plan may have and the
// kernel scans Pd->cells of them.
cudaError_t launch_scan(const int* counts, int* starts, long long cells,
                        unsigned long long* status, int* ticket, unsigned epoch, int* err,
                        cudaStream_t s, int withhold = -1, const GridPlan* Pd = nullptr);
// counts[0, Pd->cells) = 0 for a plan made on the device (max_cells: the
// largest table it may have, which sizes the launch); zero0 / zero1
// (optional): two more words set to 0
cudaError_t launch_clear_counts(int* counts, long long max_cells, const GridPlan* Pd, int sms,
                                cudaStream_t s, int* zero0 = nullptr, int* zero1 = nullptr);
// inv (optional): inv[original index] = sorted position; proj (optional, D > 3):
// projected coordinates copied to proj_sorted in cell order
cudaError_t launch_scatter(const float* pts, const GridPlan& P, const int2* cellrank,
                           const int* starts, float* rows, int* ids, cudaStream_t s,
                           int* inv = nullptr, const float* proj = nullptr,
                           float* proj_sorted = nullptr, const GridPlan* Pd = nullptr);

// grid_search.cu
// Searches sorted query positions [q0, q1).  Results for sorted position sq go
// to row (sq - q0) of the outputs: out[k*ostride + (sq - q0)], or, when
// scatter_ids is non-null, straight to out[k*ostride + scatter_ids[sq] -
// row_base] (row_base 0 unless given).
// qlist (optional): the searched sorted positions are qlist[q0..q1) instead
// of q0..q1; qcount (optional, device): only the first *qcount of them.
// row_base (>= 0): without scatter_ids, sorted position sq goes to row
// sq - row_base instead of sq - q0 (for query lists).  proj (optional): the
// grid axes are the sorted projected coordinates proj[sq*kProjStride + d].
// qrows / qproj (optional): a separate query set's rows and projected
// coordinates in the same grid's cell order (sq indexes them).
cudaError_t launch_grid_search(const float* rows, const int* ids, const int* starts,
                               const GridPlan& P, int K, float r2, int q0, int q1, int* oidx,
                               float* odist, long long ostride, const int* scatter_ids,
                               cudaStream_t s, const int* qlist = nullptr,
                               const int* qcount = nullptr, long long row_base = -1,
                               const float* proj = nullptr, const float* qrows = nullptr,
                               const float* qproj = nullptr, const GridPlan* Pd = nullptr);

// grid_collect.cu -- D = 3 two-kernel search (K <= 32).
constexpr int kCollectRowPad = 8;

// collect: for sorted queries sq in [q0, q1), every in-radius key goes to
// lists[sq*cap + j]; counts[sq] = number found; queries with more than cap are
// appended to overflow[0..*n_overflow).  qrows (optional): a separate query
// set's rows in the grid's cell order.  qlist (optional): the searched sorted
// positions are qlist[q0..q1) instead of q0..q1.  rows must be readable
// kCollectRowPad rows past P.n (the kernel loads whole 8-row passes and masks
// the excess).
cudaError_t launch_collect_d3(const float* rows, const int* starts, const GridPlan& P, float r2,
                              int cap, unsigned long long* lists, int* counts, int* overflow,
                              int* n_overflow, int q0, int q1, cudaStream_t s,
                              const float* qrows = nullptr, const int* qlist = nullptr,
                              const GridPlan* Pd = nullptr);
// collect for D != 3 (any grid the planner makes, K-independent): the same
// lists as launch_collect_d3 from one thread per query over its 3^g shell;
// qproj: the queries' projected coordinates on a principal-axis grid (the
// points' own sorted projections for a self-search).
cudaError_t launch_collect_nd(const float* rows, const int* ids, const int* starts, const GridPlan& P,
                              float r2, int cap, unsigned long long* lists, int* counts, int* overflow,
                              int* n_overflow, int q0, int q1, cudaStream_t s, const float* qrows = nullptr,
                              const float* qproj = nullptr, const int* qlist = nullptr,
                              const GridPlan* Pd = nullptr);
// emit: for output rows q < n -- sorted position map[q] (map = inv: rows in
// original order), or q0 + q without map -- whose count is at most cap, the K
// smallest keys ascending to out[k*n + q], padded (-1, r2).  map_range: the
// number of sorted positions map's entries index (default n).
cudaError_t launch_emit_lists(const unsigned long long* lists, const int* counts, const int* map,
                              int q0, int n, int K, int cap, float r2, int* oidx, float* odist,
                              cudaStream_t s, int map_range = -1, const GridPlan* Pd = nullptr);
// out[k*N + ids[sq]] = in[k*N + sq]
cudaError_t launch_unpermute(const int* in_idx, const float* in_dist, const int* ids, int n,
                             int K, int* out_idx, float* out_dist, cudaStream_t s,
                             const GridPlan* Pd = nullptr);

// bruteforce.cu
// Queries [q0, q1) of the SoA cloud against all n points; results of query q
// go to out[k*ostride + (q - q0)].  With qlist (device), the queries are
// qlist[q0..q1) instead and query q's results go to out[k*ostride + q - row_base].
// qpts (optional): the queries are a separate SoA set of qn points.
cudaError_t launch_bruteforce(const float* pts, int n, int dim, int K, float r2, int q0, int q1,
                              int* oidx, float* odist, long long ostride, cudaStream_t s,
                              const int* qlist = nullptr, int row_base = 0,
                              const float* qpts = nullptr, int qn = 0);

// grid_pca.cu -- principal axes for the grid (5 <= dim <= 32).
int pca_slots(int dim);            // dim sums + dim*(dim+1)/2 products
// sums over `samples` strided points of x - x0 and the upper triangle of
// (x - x0)(x - x0)^T (x0 = point 0) into out[pca_slots(dim)] (double), then
// x0 itself in out[pca_slots(dim) + d], via blocks x slots partials;
// deterministic
cudaError_t launch_pca_moments(const float* pts, int n, int dim, int samples, int blocks, double* partial,
                               double* out, cudaStream_t s);
int pca_project_slots();           // 2 * kMaxGridAxes + 2
// proj[i*kProjStride + k] = sum_d pm[k*dim + d] (x_d - mu_d), k < axes;
// out[2k], out[2k+1] = min, max of axis k; out[2*kMaxGridAxes] = max |x - mu|^2;
// out[2*kMaxGridAxes + 1] = 1 if any coordinate is NaN or Inf
cudaError_t launch_pca_project(const float* pts, int n, int dim, int axes, const float* mu, const float* pm,
                               float* proj, float* partial, unsigned int* ticket, float* out, int blocks,
                               cudaStream_t s);
// counts[q*16 + b*8 + g-1] for nq sample queries over m sample points: points
// within h[b*8 + g-1] of the query on each of the first g axes of basis b
// (0 leading coordinates, 1 principal axes); smp is m x 16 floats of scratch
cudaError_t launch_pca_estimate(const float* pts, int n, int dim, const float* proj, int m, int nq, float* smp,
                                const float* h, int* counts, cudaStream_t s);

// bf_tc.cu -- brute force with a tcgen05 distance filter, 33 <= dim <= 128.

// The ranks of a sharded symmetric filter: every rank's candidate lists and
// counters (this rank's own buffers, the others' mapped through CUDA IPC).
constexpr int kTcMaxPeers = 8;
struct TcPeers {
    int n = 0;  // ranks
    const int* counts[kTcMaxPeers] = {};
    const int* lists[kTcMaxPeers] = {};
};
int tc_kc(int dim);                 // 64-dimension slabs per row (1 or 2)
size_t tc_tile_bytes(int dim);      // bytes of one 128-row fp16 tile
int tc_row_floats(int dim);         // floats per fp32 row (dim rounded up to 4)
int tc_list_cap(int K);             // candidate list capacity per query
// box[2d], box[2d+1] = min, max of dimension d; *nonfinite |= any NaN/Inf
cudaError_t launch_tc_box(const float* pts, int n, int dim, float* box, int* nonfinite, cudaStream_t s);
// fp16 tiles (ceil(n/128) tiles), fp32 rows, threshold terms qa / pb (padded
// to whole tiles with +inf); the query blocks searched are [qb_begin, qb_end)
cudaError_t launch_tc_prep(const float* pts, int n, int dim, const float* center, float scale,
                           float one_minus_alpha, float eta_c, float rc, uint8_t* tiles, float* rows32,
                           float* qa, float* pb, cudaStream_t s);
// counts[q] = candidates of query q (all q < n); the first cap of them in
// lists[q*cap ..]; queries with more go to overflow[0..*n_overflow)
// qtiles (optional): a separate query set of m points (its own tiles; qa then
// holds its terms), searched against the n points of tiles / pb
// skip_tile >= 0: the producer never copies that point tile, so the MMA
// thread's bounded wait for it gives up (tests of the timeout path only)
// sym (a self-search, no qtiles): each unordered pair of tiles is filtered
// once and every passing pair goes to both lists; counts must be zero on
// entry.  Without sym_part the query tiles must be all of them, and the
// overflow list is made at the end; with sym_part (a sharded search) the
// query tiles are this rank's range, the pairs seen from other ranks' points
// stay in this rank's lists for those ranks to pull (launch_tc_pull), and
// launch_tc_sym_overflow makes the list after the pull.
cudaError_t launch_tc_filter(const uint8_t* tiles, const float* qa, const float* pb, int n, int dim,
                             int cap, int* lists, int* counts, int* overflow, int* n_overflow, int* err,
                             int qb_begin, int qb_end, cudaStream_t s, const uint8_t* qtiles = nullptr,
                             int m = 0, int skip_tile = -1, bool sym = false, bool sym_part = false);
// After every rank's symmetric filter: the entries the other ranks listed for
// this rank's queries [q0, q1), appended to their own lists
cudaError_t launch_tc_pull(const TcPeers& peers, int self, int* counts, int* lists, int q0, int q1, int cap,
                           cudaStream_t s);
// overflow[0..*n_overflow) = the queries q in [q0, q1) with counts[q] > cap
cudaError_t launch_tc_sym_overflow(const int* counts, int q0, int q1, int cap, int* overflow, int* n_overflow,
                                   cudaStream_t s);
// exact results for the queries q in [q0, q1) with counts[q] <= cap, to row
// q - q0 of out[k*(q1-q0) + row]
// qrows32 (optional): the separate query set's fp32 rows (n = its size)
cudaError_t launch_tc_rerank(const float* rows32, int dim, const int* lists, const int* counts, int cap,
                             int n, int K, float r2, int* oidx, float* odist, int q0, int q1,
                             cudaStream_t s, const float* qrows32 = nullptr);

}  // namespace frnn
