// engine.cu -- host engine, dispatcher and the C ABI of include/frnn_b200.h.
//
// Replaces the reference's FRNNEngine (python_interface/frnn_engine.{h,cu}).
// Differences by design:
//   * scratch is allocated lazily from the sizes of each call and kept across
//     calls (the reference allocates 32-dim / 128-slot buffers up front and
//     overflows them for D > 32, frnn_engine.cu:26-27);
//   * all work runs on one stream (the legacy default stream unless the
//     caller sets another) with no device-wide synchronisation;
//   * the dispatcher (frnn_engine.cu:215-246 in the reference) decides from
//     N, D, K, r and the bounding box of the grid axes; no path drops points;
//   * every CUDA call is checked and reported through the status codes.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>

#include "frnn_b200.h"
#include "frnn_device.cuh"
#include "frnn_internal.h"
#include "grid_plan.cuh"
#include "engine_state.h"

using namespace frnn;

namespace frnn {
namespace eng {

// Brute force is taken when the all-pairs work is small enough that the grid
// build would dominate (the reference's own small-input rule is
// N^2*D*ceil(K/8) <= 2e6, frnn_engine.cu:215-219; a B200 finishes far larger
// all-pairs problems in the time of one grid build).
constexpr double kBruteSmallWork = 4.0e8;   // N*N*D below this -> brute force
// D > 32 goes to brute force; from this many points on, with the tcgen05
// distance filter (measured on B200 at D = 128, K = 128: 0.22 ms against the
// SIMT kernel's 29 ms at N = 4096; below ~1K points the filter's prep and two
// host round trips are most of its time).
constexpr int kTcMinPoints = 1024;



int fail(frnn_engine* e, int status, const std::string& msg) {
    if (e) e->last_error = msg;
    return status;
}

int cuda_fail(frnn_engine* e, cudaError_t err, const char* what) {
    std::string m = std::string(what) + ": " + cudaGetErrorString(err);
    cudaGetLastError();  // clear a sticky launch error so the engine stays usable
    return fail(e, err == cudaErrorMemoryAllocation ? FRNN_ERR_OOM : FRNN_ERR_CUDA, m);
}

int grow(frnn_engine* e, DevBuf& b, size_t bytes, const char* what) {
    if (bytes == 0) bytes = 16;
    if (b.bytes >= bytes) return FRNN_OK;
    if (b.p) cudaFree(b.p);
    b.p = nullptr;
    b.bytes = 0;
    // round up to limit regrowth
    size_t want = bytes + bytes / 8;
    want = (want + 255) & ~size_t(255);
    cudaError_t err = cudaMalloc(&b.p, want);
    if (err != cudaSuccess) {
        cudaGetLastError();
        b.p = nullptr;
        return fail(e, FRNN_ERR_OOM, std::string("cudaMalloc failed for ") + what + " (" +
                                         std::to_string(want) + " bytes)");
    }
    b.bytes = want;
    return FRNN_OK;
}

// The scan's look-back status words carry the epoch of the search that wrote
// them, and every engine counts epochs from 1: a status buffer that reuses
// memory another engine (or anything else) wrote could hold words that look
// current.  So a newly allocated buffer is cleared before its first scan.
int grow_scan_status(frnn_engine* e, size_t bytes) {
    const size_t before = e->scan_status.bytes;
    FRNN_GROW(e, e->scan_status, bytes);
    if (e->scan_status.bytes != before)  // reallocated (grow never shrinks)
        FRNN_CHECK(e, cudaMemsetAsync(e->scan_status.p, 0, e->scan_status.bytes, e->stream), "memset status");
    return FRNN_OK;
}

void stage_begin(frnn_engine* e, int st) {
    if (e->timing) cudaEventRecord(e->ev[2 * st], e->stream);
}
void stage_end(frnn_engine* e, int st) {
    if (e->timing) {
        cudaEventRecord(e->ev[2 * st + 1], e->stream);
        e->stage_used[st] = true;
    }
}

void free_buf(DevBuf& b) {
    if (b.p) cudaFree(b.p);
    b.p = nullptr;
    b.bytes = 0;
}

int check_search_args(frnn_engine* e, const void* pts, int N, int dim, int K, float radius) {
    if (!e) return FRNN_ERR_INVALID_ARG;
    if (!pts) return fail(e, FRNN_ERR_INVALID_ARG, "points pointer is null");
    if (N <= 0) return fail(e, FRNN_ERR_INVALID_ARG, "N must be positive");
    if (N > e->max_points)
        return fail(e, FRNN_ERR_INVALID_ARG,
                    "N=" + std::to_string(N) + " exceeds max_points=" + std::to_string(e->max_points));
    if (dim < 1 || dim > kMaxD) return fail(e, FRNN_ERR_INVALID_ARG, "dim must be in [1, 128]");
    if (K < 1 || K > kMaxK) return fail(e, FRNN_ERR_INVALID_ARG, "K must be in [1, 128]");
    if (!(radius > 0.0f) || !std::isfinite(radius) || !std::isfinite(radius * radius) ||
        !(radius * radius > 0.0f))
        return fail(e, FRNN_ERR_INVALID_ARG, "radius must be finite and positive");
    return FRNN_OK;
}

int check_device_ptr(frnn_engine* e, const void* p) {
    cudaPointerAttributes a{};
    cudaError_t err = cudaPointerGetAttributes(&a, p);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(e, FRNN_ERR_INVALID_ARG, "points pointer is not CUDA memory");
    }
    if (a.type == cudaMemoryTypeDevice && a.device != e->device)
        return fail(e, FRNN_ERR_INVALID_ARG, "points pointer lives on another device");
    if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged)
        return fail(e, FRNN_ERR_INVALID_ARG, "points pointer is not device memory");
    return FRNN_OK;
}

// ---- transposes for the host paths --------------------------------------------

// out[c*rows + r] = in[r*cols + c]  (in: rows x cols row-major)
__global__ void transpose32_kernel(const unsigned* __restrict__ in, unsigned* __restrict__ out,
                                   int rows, int cols) {
    __shared__ unsigned t[32][33];
    // 1-D grid over 32x32 tiles (either extent may exceed the 65535 limit of gridDim.y)
    const long long tiles_c = (cols + 31) / 32;
    const int c0 = (int)(blockIdx.x % tiles_c) * 32, r0 = (int)(blockIdx.x / tiles_c) * 32;
    for (int i = threadIdx.y; i < 32; i += 8) {
        int r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) t[i][threadIdx.x] = in[(long long)r * cols + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        int c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) out[(long long)c * rows + r] = t[threadIdx.x][i];
    }
}

// out[i] = starts[c] for the largest cell c with starts[c] <= t[i]: a target
// position rounded down to the first point of its cell (the order of points
// inside a cell depends on atomic ranks and changes between builds; the cell
// starts do not).
__global__ void cell_floor_kernel(const int* __restrict__ starts, long long cells, int t0, int t1,
                                  int* __restrict__ out) {
    const int i = threadIdx.x;
    if (i > 1) return;
    const int t = i == 0 ? t0 : t1;
    long long lo = 0, hi = cells;  // starts[0] = 0 <= t; find the last c with starts[c] <= t
    while (hi - lo > 1) {
        const long long mid = (lo + hi) / 2;
        if (starts[mid] <= t) lo = mid;
        else hi = mid;
    }
    out[i] = starts[lo];
}

cudaError_t launch_cell_floor(const int* starts, long long cells, int t0, int t1, int* out, cudaStream_t s) {
    cell_floor_kernel<<<1, 32, 0, s>>>(starts, cells, t0, t1, out);
    return cudaGetLastError();
}

__global__ void iota_kernel(int* __restrict__ out, int base, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = base + i;
}

// out[j] = original query index of overflow entry j < min(*n, max_out)
__global__ void overflow_ids_kernel(const int* __restrict__ ovf, const int* __restrict__ n,
                                    const int* __restrict__ map, int max_out, int* __restrict__ out) {
    const int cnt = min(*n, max_out);
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < cnt; j += gridDim.x * blockDim.x)
        out[j] = map ? map[ovf[j]] : ovf[j];
}

cudaError_t launch_iota(int* out, int base, int n, cudaStream_t s) {
    iota_kernel<<<(n + 255) / 256, 256, 0, s>>>(out, base, n);
    return cudaGetLastError();
}

cudaError_t launch_transpose(const void* in, void* out, int rows, int cols, cudaStream_t s) {
    const long long tiles = (long long)((cols + 31) / 32) * ((rows + 31) / 32);
    dim3 grid((unsigned)tiles), block(32, 8);
    transpose32_kernel<<<grid, block, 0, s>>>(static_cast<const unsigned*>(in),
                                              static_cast<unsigned*>(out), rows, cols);
    return cudaGetLastError();
}

// ---- planning -------------------------------------------------------------------

int grid_axes_for(int dim) { return dim <= 4 ? dim : 4; }

// Build the grid plan from the box of the grid axes (plan_grid): false when a
// grid is useless or cannot be formed.  The dense cell table may hold
// `cells_per_point` cells per point (at least 2^22): 12 bytes of build traffic
// per cell, and sparse clouds such as Gaussian mixtures leave most cells
// empty, while coarser cells would multiply the candidates of every query.
long long cell_budget(int N, long long cells_per_point) {
    return std::min<long long>(std::max<long long>(1LL << 22, cells_per_point * N), (1LL << 31) - 2);
}

bool make_plan_axes(const float* box, int g, int N, int dim, float radius, double extra, GridPlan& P,
                    long long cells_per_point = 32) {
    return plan_grid(box, g, N, dim, radius, extra, cell_budget(N, cells_per_point), P);
}

bool make_plan(const float* box, int N, int dim, float radius, GridPlan& P) {
    return make_plan_axes(box, grid_axes_for(dim), N, dim, radius, 0.0, P);
}

constexpr long long kPrincipalCellsPerPoint = 128;

// Per-coordinate rounding bound of projected coordinates computed in fp32:
// (D + 2) 2^-24 |x - mu| (one fixed summation order over D terms), for the
// largest |x - mu| of a point set (max_sq = its square).
double projection_delta(int dim, double max_sq) {
    return (dim + 2) * std::ldexp(std::sqrt(std::max(0.0, max_sq)) * 1.001, -24);
}

// Screening bound of projected squared distances on a principal-axis grid.
// A pair the fp32 chain accepts (d2 < fl(r*r)) is within r (1 + 2^-16) in the
// full dimension -- the chain's relative rounding is below (D + 3) 2^-25 --
// and so in projection (orthonormal axes never lengthen a distance; the fp32
// axes are orthonormal to about 2^-20).  Computed projections differ from
// exact ones by at most delta_q + delta_p per coordinate, so the computed
// projected distance stays below r (1 + 2^-16) + (delta_q + delta_p) sqrt(g);
// the factor (1 + 2^-16)^2 covers the fp32 evaluation of the screened
// distance itself.
float screen_r2(float radius, int g, double delta_sum) {
    const double e = std::ldexp(1.0, -16);
    const double rr = ((double)radius * (1.0 + e) + delta_sum * std::sqrt((double)g)) * (1.0 + e);
    float f = (float)(rr * rr);
    if ((double)f < rr * rr) f = std::nextafter(f, INFINITY);
    return f;
}

// Eigen-decomposition of a symmetric n x n matrix (row-major, destroyed) by
// cyclic Jacobi rotations in double: w[i] eigenvalues, column i of V (row-major
// n x n) the eigenvector of w[i].
void jacobi_eigen(int n, double* A, double* V, double* w) {
    for (int i = 0; i < n * n; ++i) V[i] = 0.0;
    for (int i = 0; i < n; ++i) V[i * n + i] = 1.0;
    for (int sweep = 0; sweep < 100; ++sweep) {
        double off = 0.0, diag = 0.0;
        for (int p = 0; p < n; ++p) {
            diag += A[p * n + p] * A[p * n + p];
            for (int q = p + 1; q < n; ++q) off += A[p * n + q] * A[p * n + q];
        }
        if (off <= 1e-30 * diag || off == 0.0) break;
        for (int p = 0; p < n; ++p) {
            for (int q = p + 1; q < n; ++q) {
                const double apq = A[p * n + q];
                if (apq == 0.0) continue;
                const double theta = (A[q * n + q] - A[p * n + p]) / (2.0 * apq);
                const double t = (theta >= 0 ? 1.0 : -1.0) / (std::fabs(theta) + std::sqrt(theta * theta + 1.0));
                const double c = 1.0 / std::sqrt(t * t + 1.0), sn = t * c;
                for (int k = 0; k < n; ++k) {
                    const double akp = A[k * n + p], akq = A[k * n + q];
                    A[k * n + p] = c * akp - sn * akq;
                    A[k * n + q] = sn * akp + c * akq;
                }
                for (int k = 0; k < n; ++k) {
                    const double apk = A[p * n + k], aqk = A[q * n + k];
                    A[p * n + k] = c * apk - sn * aqk;
                    A[q * n + k] = sn * apk + c * aqk;
                }
                for (int k = 0; k < n; ++k) {
                    const double vkp = V[k * n + p], vkq = V[k * n + q];
                    V[k * n + p] = c * vkp - sn * vkq;
                    V[k * n + q] = sn * vkp + c * vkq;
                }
            }
        }
    }
    for (int i = 0; i < n; ++i) w[i] = A[i * n + i];
}

// ---- principal axes ---------------------------------------------------------------

// For 5 <= D <= 32 on the grid path: the sample moments give the principal
// axes; every point is projected on the top min(D, 6) of them; a sampled
// shell count estimates the candidates per query of the leading-coordinate
// grid (`first`, if valid) and of principal-axis grids on g = 2..6 axes; the
// cheapest is kept.  On return *principal says whether P now holds a
// principal-axis plan (the projected coordinates are then in e->proj_u).
int plan_principal(frnn_engine* e, const float* d_pts, int N, int dim, float radius, bool first_ok,
                   GridPlan& P, bool* principal) {
    cudaStream_t s = e->stream;
    *principal = false;
    const int slots = pca_slots(dim);
    const int samples = std::min(N, 65536);
    const int mblocks = std::max(1, std::min(256, samples / 256));
    FRNN_GROW(e, e->pca_partial, (size_t)mblocks * slots * 8);
    FRNN_GROW(e, e->pca_moments, (size_t)(slots + dim) * 8);
    FRNN_CHECK(e, launch_pca_moments(d_pts, N, dim, samples, mblocks, e->pca_partial.as<double>(),
                                     e->pca_moments.as<double>(), s),
               "moments launch");
    double* hm = static_cast<double*>(e->h_pca);
    FRNN_CHECK(e, cudaMemcpyAsync(hm, e->pca_moments.p, (size_t)(slots + dim) * 8, cudaMemcpyDeviceToHost, s),
               "moments readback");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "moments sync");
    e->launches += 2;

    // covariance of the sample (about x0, then about the mean)
    double mean[kMaxPcaDim], C[kMaxPcaDim * kMaxPcaDim], V[kMaxPcaDim * kMaxPcaDim], w[kMaxPcaDim];
    for (int d = 0; d < dim; ++d) mean[d] = hm[d] / samples;
    int k = dim;
    for (int a = 0; a < dim; ++a)
        for (int b = a; b < dim; ++b, ++k) {
            const double c = hm[k] / samples - mean[a] * mean[b];
            C[a * dim + b] = c;
            C[b * dim + a] = c;
        }
    jacobi_eigen(dim, C, V, w);
    int order[kMaxPcaDim];
    for (int i = 0; i < dim; ++i) order[i] = i;
    std::stable_sort(order, order + dim, [&](int x, int y) { return w[x] > w[y]; });
    const int axes = std::min(dim, kMaxGridAxes);
    // host staging after the moments: mu (dim floats), pm (axes x dim floats)
    float* hmu = reinterpret_cast<float*>(static_cast<char*>(e->h_pca) + 8192);
    float* hpm = hmu + kMaxPcaDim;
    for (int d = 0; d < dim; ++d) hmu[d] = (float)(hm[slots + d] + mean[d]);  // x0 + sample mean
    for (int a = 0; a < axes; ++a) {
        const int c = order[a];
        int big = 0;
        for (int d = 1; d < dim; ++d)
            if (std::fabs(V[d * dim + c]) > std::fabs(V[big * dim + c])) big = d;
        const double sg = V[big * dim + c] < 0 ? -1.0 : 1.0;
        for (int d = 0; d < dim; ++d) hpm[a * dim + d] = (float)(sg * V[d * dim + c]);
    }
    FRNN_GROW(e, e->pca_mu, (size_t)kMaxPcaDim * 4);
    FRNN_GROW(e, e->pca_pm, (size_t)kMaxGridAxes * kMaxPcaDim * 4);
    FRNN_CHECK(e, cudaMemcpyAsync(e->pca_mu.p, hmu, (size_t)dim * 4, cudaMemcpyHostToDevice, s), "mu upload");
    FRNN_CHECK(e, cudaMemcpyAsync(e->pca_pm.p, hpm, (size_t)axes * dim * 4, cudaMemcpyHostToDevice, s),
               "axes upload");

    // projection and its bounding box
    const int pblocks = std::min(bbox_blocks(N, e->sms), kBoxMaxBlocks);
    const int pslots = pca_project_slots();
    FRNN_GROW(e, e->proj_u, (size_t)N * kProjStride * 4);
    FRNN_GROW(e, e->proj_box_partial, (size_t)pblocks * pslots * 4);
    if (!e->proj_ticket.p) {
        FRNN_GROW(e, e->proj_ticket, 16);
        FRNN_CHECK(e, cudaMemsetAsync(e->proj_ticket.p, 0, 16, s), "memset ticket");
    }
    FRNN_GROW(e, e->proj_out, 64 * 4);
    FRNN_CHECK(e, launch_pca_project(d_pts, N, dim, axes, e->pca_mu.as<float>(), e->pca_pm.as<float>(),
                                     e->proj_u.as<float>(), e->proj_box_partial.as<float>(),
                                     e->proj_ticket.as<unsigned>(), e->proj_out.as<float>(), pblocks, s),
               "project launch");
    float* hbox = hpm + kMaxGridAxes * kMaxPcaDim;
    FRNN_CHECK(e, cudaMemcpyAsync(hbox, e->proj_out.p, (size_t)pslots * 4, cudaMemcpyDeviceToHost, s),
               "projected box readback");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "projected box sync");
    e->launches++;
    if (hbox[pslots - 1] != 0.0f) return fail(e, FRNN_ERR_INVALID_ARG, "points contain NaN or Inf coordinates");

    // Rounding bound of a projected coordinate: (D + 2) 2^-24 |x - mu|; a pair
    // within r differs by at most r (1 + 2^-20) + 2 delta on every axis.
    const double nmax = std::sqrt(std::max(0.0, (double)hbox[pslots - 2])) * 1.001;
    const double extra = 2.0 * (dim + 2) * std::ldexp(nmax, -24) + (double)radius * std::ldexp(1.0, -20);
    GridPlan cand[kMaxGridAxes + 1];
    bool ok[kMaxGridAxes + 1] = {};
    // principal-axis grids serve D > 4 clouds, whose search costs far more
    // than the build: a finer table (up to 128 cells per point) is worth it
    for (int g = 2; g <= axes; ++g)
        ok[g] = make_plan_axes(hbox, g, N, dim, radius, extra, cand[g], kPrincipalCellsPerPoint);

    // sampled shell counts
    const int m = std::min(N, 16384), nq = std::min(m, 256);
    float* hh = hbox + 16;
    for (int t = 0; t < 16; ++t) hh[t] = -1.0f;
    if (first_ok) hh[P.g - 1] = 1.5f * P.cell;
    for (int g = 2; g <= axes; ++g)
        if (ok[g]) hh[8 + g - 1] = 1.5f * cand[g].cell;
    FRNN_GROW(e, e->pca_h, 16 * 4);
    FRNN_GROW(e, e->pca_smp, (size_t)m * 16 * 4);
    FRNN_GROW(e, e->pca_counts, (size_t)nq * 16 * 4);
    FRNN_CHECK(e, cudaMemcpyAsync(e->pca_h.p, hh, 16 * 4, cudaMemcpyHostToDevice, s), "estimate upload");
    FRNN_CHECK(e, launch_pca_estimate(d_pts, N, dim, e->proj_u.as<float>(), m, nq, e->pca_smp.as<float>(),
                                      e->pca_h.as<float>(), e->pca_counts.as<int>(), s),
               "estimate launch");
    int* hc = reinterpret_cast<int*>(static_cast<char*>(e->h_pca) + 16384);
    FRNN_CHECK(e, cudaMemcpyAsync(hc, e->pca_counts.p, (size_t)nq * 16 * 4, cudaMemcpyDeviceToHost, s),
               "estimate readback");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "estimate sync");
    e->launches += 2;
    // cost per query: candidates plus a fixed charge per shell row (3^(g-1))
    auto cost = [&](int col, int g) {
        double c = 0.0;
        for (int q = 0; q < nq; ++q) c += hc[q * 16 + col];
        return c / nq * ((double)N / m) + 8.0 * std::pow(3.0, g - 1);
    };
    int best_g = 0;
    double best = INFINITY;
    for (int g = 2; g <= axes; ++g)
        if (ok[g] && cost(8 + g - 1, g) < best) best = cost(8 + g - 1, g), best_g = g;
    if (best_g == 0) return FRNN_OK;
    // principal axes replace the leading coordinates (the reference's grid)
    // only when clearly cheaper, unless they are forced
    if (e->grid_axes_mode != FRNN_GRID_AXES_PRINCIPAL && first_ok && !(1.25 * best < cost(P.g - 1, P.g)))
        return FRNN_OK;
    P = cand[best_g];
    e->proj_delta = projection_delta(dim, (double)hbox[pslots - 2]);
    P.pre_r2 = screen_r2(radius, P.g, 2.0 * e->proj_delta);
    *principal = true;
    return FRNN_OK;
}

// ---- the search core ------------------------------------------------------------

// Whole search (part == false): results for every query in original order,
// out[k*N + q].  Part search: the queries at sorted positions [s0, s1) only,
// row j = sorted position s0 + j of out[k*(s1-s0) + j].
// proj: the points' projected coordinates when P is a principal-axis grid.
// Whether a grid search with D != 3 and K <= 32 takes the list search
// (collect + emit) rather than the warp-cooperative kernel.  AUTO: rows of at
// most 12 floats (B200, 12 clouds: the list search is 1.2-3x faster for
// D <= 12 on every grid but one dense five-dimensional mixture, and 1.3-1.6x
// slower at D = 16 and 24 on six principal axes, where the cooperative
// kernel's shared candidate loads pay).
bool list_search_nd(const frnn_engine* e, const GridPlan& P) {
    if (e->list_search == FRNN_LIST_SEARCH_ALWAYS) return true;
    if (e->list_search == FRNN_LIST_SEARCH_NEVER) return false;
    return P.row <= 12;
}

// Whether a grid search over plan P with K neighbours takes the list search
// (collect + emit): D = 3 on its own coordinates always, other D as
// list_search_nd decides; K <= 32 only.
bool uses_lists(const frnn_engine* e, const GridPlan& P, int K, bool principal) {
    const bool d3 = P.dim == 3 && P.g == 3 && !principal;
    return K <= 32 && (d3 || list_search_nd(e, P));
}

int build_points(frnn_engine* e, const float* d_pts, const GridPlan& P, const float* proj, bool with_inv) {
    cudaStream_t s = e->stream;
    const int N = P.n;
    FRNN_GROW(e, e->counts, (size_t)P.cells * 4);
    FRNN_GROW(e, e->starts, ((size_t)P.cells + 1) * 4);
    const long long tiles = scan_tiles(P.cells);
    {
        const int st = grow_scan_status(e, (size_t)tiles * 8);
        if (st != FRNN_OK) return st;
    }
    FRNN_GROW(e, e->cellrank, (size_t)N * 8);
    // padded: the D = 3 collect kernel reads whole 8-row passes
    FRNN_GROW(e, e->rows, ((size_t)N + kCollectRowPad) * P.row * 4);
    FRNN_GROW(e, e->ids, (size_t)N * 4);

    FRNN_CHECK(e, cudaMemsetAsync(e->counts.p, 0, (size_t)P.cells * 4, s), "memset counts");
    FRNN_CHECK(e, cudaMemsetAsync(e->scan_ticket.p, 0, 4, s), "memset scan ticket");
    stage_begin(e, ST_HASH);
    FRNN_CHECK(e, launch_hash_count(d_pts, P, e->counts.as<int>(), e->cellrank.as<int2>(), s, proj),
               "hash_count launch");
    stage_end(e, ST_HASH);
    e->launches++;
    e->epoch = (e->epoch + 1) & 0x3fffffffu;
    if (e->epoch == 0) {
        // status words of every earlier epoch must read as "not ready"
        FRNN_CHECK(e, cudaMemsetAsync(e->scan_status.p, 0, e->scan_status.bytes, s), "memset status");
        e->epoch = 1;
    }
    stage_begin(e, ST_SCAN);
    FRNN_CHECK(e, launch_scan(e->counts.as<int>(), e->starts.as<int>(), P.cells,
                              e->scan_status.as<unsigned long long>(), e->scan_ticket.as<int>(),
                              e->epoch, e->err_flag.as<int>(), s,
                              e->test_stall == FRNN_TEST_STALL_SCAN ? 1 : -1),
               "scan launch");
    stage_end(e, ST_SCAN);
    if (with_inv) FRNN_GROW(e, e->inv, (size_t)N * 4);
    if (proj) FRNN_GROW(e, e->proj_s, (size_t)N * kProjStride * 4);
    stage_begin(e, ST_SCATTER);
    FRNN_CHECK(e, launch_scatter(d_pts, P, e->cellrank.as<int2>(), e->starts.as<int>(),
                                 e->rows.as<float>(), e->ids.as<int>(), s,
                                 with_inv ? e->inv.as<int>() : nullptr, proj,
                                 proj ? e->proj_s.as<float>() : nullptr),
               "scatter launch");
    stage_end(e, ST_SCATTER);
    e->launches += 2;
    return FRNN_OK;
}

int search_built(frnn_engine* e, const GridPlan& P, bool principal, int K, float r2, int q0, int q1,
                 bool whole, int* out_idx, float* out_dist, const GridPlan* Pd) {
    cudaStream_t s = e->stream;
    const int N = P.n;
    const float* proj_s = principal ? e->proj_s.as<float>() : nullptr;
    const bool d3 = P.dim == 3 && P.g == 3 && !principal;
    const int rows = q1 - q0;
    if (uses_lists(e, P, K, principal)) {
        // collect every in-radius key per query, then sort and emit (whole:
        // original query order through inv, no unpermute; slice: sorted
        // order); queries whose list overflows are searched again by the
        // cooperative kernel.
        const int cap = K <= 16 ? 64 : 128;
        FRNN_GROW(e, e->lists, (size_t)N * cap * 8);
        FRNN_GROW(e, e->list_counts, (size_t)N * 4);
        FRNN_GROW(e, e->overflow, (size_t)N * 4);
        FRNN_GROW(e, e->n_overflow, 16);
        // (a device-planned search zeroed it with its count table)
        if (!Pd) FRNN_CHECK(e, cudaMemsetAsync(e->n_overflow.p, 0, 4, s), "memset overflow count");
        e->last_overflow_map = whole ? 1 : 0;
        stage_begin(e, ST_COLLECT);
        if (d3)
            FRNN_CHECK(e, launch_collect_d3(e->rows.as<float>(), e->starts.as<int>(), P, r2, cap,
                                            e->lists.as<unsigned long long>(), e->list_counts.as<int>(),
                                            e->overflow.as<int>(), e->n_overflow.as<int>(), q0, q1, s, nullptr,
                                            nullptr, Pd),
                       "collect launch");
        else
            FRNN_CHECK(e, launch_collect_nd(e->rows.as<float>(), e->ids.as<int>(), e->starts.as<int>(), P, r2,
                                            cap, e->lists.as<unsigned long long>(), e->list_counts.as<int>(),
                                            e->overflow.as<int>(), e->n_overflow.as<int>(), q0, q1, s, nullptr,
                                            proj_s, nullptr, Pd),
                       "collect launch");
        stage_end(e, ST_COLLECT);
        stage_begin(e, ST_EMIT);
        FRNN_CHECK(e, launch_emit_lists(e->lists.as<unsigned long long>(), e->list_counts.as<int>(),
                                        whole ? e->inv.as<int>() : nullptr, q0, rows, K, cap, r2,
                                        out_idx, out_dist, s, -1, Pd),
                   "emit launch");
        FRNN_CHECK(e, launch_grid_search(e->rows.as<float>(), e->ids.as<int>(), e->starts.as<int>(),
                                         P, K, r2, 0, N, out_idx, out_dist, rows,
                                         whole ? e->ids.as<int>() : nullptr, s, e->overflow.as<int>(),
                                         e->n_overflow.as<int>(), q0, proj_s, nullptr, nullptr, Pd),
                   "overflow search launch");
        stage_end(e, ST_EMIT);
        e->launches += 3;
        return FRNN_OK;
    }
    // Small result sets: write straight to the original query ids (the
    // scattered stores stay in L2).  Large ones: write in cell order, then
    // unpermute one output row at a time.
    const long long out_bytes = (long long)N * K * 8;
    if (!whole) {
        stage_begin(e, ST_SEARCH);
        FRNN_CHECK(e, launch_grid_search(e->rows.as<float>(), e->ids.as<int>(), e->starts.as<int>(), P, K,
                                         r2, q0, q1, out_idx, out_dist, rows, nullptr, s, nullptr,
                                         nullptr, -1, proj_s, nullptr, nullptr, Pd),
                   "grid search launch");
        stage_end(e, ST_SEARCH);
        e->launches++;
    } else if (out_bytes <= e->direct_output_max_bytes || P.dim > 3) {
        // D > 3 always writes directly (B200, cfg3: 2.30 against 2.38 ms with
        // the unpermute pass; cfg4 equal)
        stage_begin(e, ST_SEARCH);
        FRNN_CHECK(e, launch_grid_search(e->rows.as<float>(), e->ids.as<int>(), e->starts.as<int>(), P, K,
                                         r2, 0, N, out_idx, out_dist, N, e->ids.as<int>(), s, nullptr,
                                         nullptr, -1, proj_s, nullptr, nullptr, Pd),
                   "grid search launch");
        stage_end(e, ST_SEARCH);
        e->launches++;
    } else {
        FRNN_GROW(e, e->tmp_idx, (size_t)N * K * 4);
        FRNN_GROW(e, e->tmp_dist, (size_t)N * K * 4);
        stage_begin(e, ST_SEARCH);
        FRNN_CHECK(e, launch_grid_search(e->rows.as<float>(), e->ids.as<int>(), e->starts.as<int>(), P, K,
                                         r2, 0, N, e->tmp_idx.as<int>(), e->tmp_dist.as<float>(), N,
                                         nullptr, s, nullptr, nullptr, -1, proj_s, nullptr, nullptr, Pd),
                   "grid search launch");
        stage_end(e, ST_SEARCH);
        stage_begin(e, ST_UNPERMUTE);
        FRNN_CHECK(e, launch_unpermute(e->tmp_idx.as<int>(), e->tmp_dist.as<float>(), e->ids.as<int>(),
                                       N, K, out_idx, out_dist, s, Pd),
                   "unpermute launch");
        stage_end(e, ST_UNPERMUTE);
        e->launches += 2;
    }
    return FRNN_OK;
}

// Whole search (part == false): results for every query in original order,
// out[k*N + q].  Part search: the queries at sorted positions [s0, s1) only,
// rounded to cell starts, row j = sorted position s0 + j of
// out[k*(s1-s0) + j].  proj: the points' projected coordinates when P is a
// principal-axis grid.
int run_grid(frnn_engine* e, const float* d_pts, int N, int dim, int K, float r2,
             const GridPlan& P, int* out_idx, float* out_dist, bool part, int& s0, int& s1,
             const float* proj) {
    cudaStream_t s = e->stream;
    const bool principal = proj != nullptr;
    int st = build_points(e, d_pts, P, proj, !part && uses_lists(e, P, K, principal));
    if (st != FRNN_OK) return st;
    if (part) {
        // part boundaries move to cell boundaries, so that parts searched by
        // separate builds cover every query exactly once
        int* h = reinterpret_cast<int*>(e->h_tc);
        FRNN_CHECK(e, launch_cell_floor(e->starts.as<int>(), P.cells, s0, s1, e->scan_ticket.as<int>() + 1, s),
                   "cell floor launch");
        FRNN_CHECK(e, cudaMemcpyAsync(h, e->scan_ticket.as<int>() + 1, 2 * sizeof(int), cudaMemcpyDeviceToHost, s),
                   "part bounds readback");
        FRNN_CHECK(e, cudaStreamSynchronize(s), "part bounds sync");
        s0 = s0 >= N ? N : h[0];
        s1 = s1 >= N ? N : h[1];
    }
    return search_built(e, P, principal, K, r2, part ? s0 : 0, part ? s1 : N, !part, out_idx, out_dist);
}

// Whether a self-search takes run_grid_dplan: whole, blocking, on the grid,
// D <= 4 (the grid axes are the coordinates, so the host needs nothing from
// the box to choose the kernels).
bool uses_device_plan(const frnn_engine* e, int path, int dim, bool blocking, bool part) {
    return e->device_plan && path == FRNN_PATH_GRID && dim <= 4 && blocking && !part;
}

// A whole self-search on the grid with D <= 4, planned on the device: the
// bounding-box kernel's last block plans the grid (plan_grid, the same code
// and arithmetic as the host planner) into e->dplan, and every later kernel
// reads that plan, so box, build and search run back to back with no host
// round trip.  What the host must size before the plan exists is sized for
// the largest plan the cell budget allows: the cell tables and the scan's
// tiles (those past the plan's table return at once); a kernel zeroes the
// plan's own count table in place of the host path's memset.  The plan is
// copied to e->h_plan with the search; after the caller's sync,
// h_plan->cells == 0 means that no grid was built (finish_dplan).
int run_grid_dplan(frnn_engine* e, const float* d_pts, int N, int dim, int K, float radius, int* out_idx,
                   float* out_dist) {
    cudaStream_t s = e->stream;
    const int g = grid_axes_for(dim);
    const long long budget = cell_budget(N, 32);
    GridPlan P{};  // what the host knows: the kernels read the rest from Pd
    P.g = g;
    P.n = N;
    P.dim = dim;
    P.row = plan_row_floats(dim);
    P.cells = budget;
    const bool lists = uses_lists(e, P, K, false);
    FRNN_GROW(e, e->counts, (size_t)budget * 4);
    FRNN_GROW(e, e->starts, ((size_t)budget + 1) * 4);
    {
        const int st = grow_scan_status(e, (size_t)scan_tiles(budget) * 8);
        if (st != FRNN_OK) return st;
    }
    FRNN_GROW(e, e->dplan, sizeof(GridPlan));
    FRNN_GROW(e, e->n_overflow, 16);
    FRNN_GROW(e, e->cellrank, (size_t)N * 8);
    FRNN_GROW(e, e->rows, ((size_t)N + kCollectRowPad) * P.row * 4);
    FRNN_GROW(e, e->ids, (size_t)N * 4);
    if (lists) FRNN_GROW(e, e->inv, (size_t)N * 4);
    GridPlan* Pd = e->dplan.as<GridPlan>();

    const int blocks = std::min(bbox_blocks(N, e->sms), kBoxMaxBlocks);
    stage_begin(e, ST_BBOX);
    FRNN_CHECK(e, launch_bbox(d_pts, N, g, e->box_partial.as<float>(), e->box_ticket.as<unsigned>(),
                              e->box_out.as<float>(), blocks, s, Pd, dim, radius, budget),
               "bbox launch");
    stage_end(e, ST_BBOX);
    // the count table, the scan's ticket and the overflow count, in one kernel
    FRNN_CHECK(e, launch_clear_counts(e->counts.as<int>(), budget, Pd, e->sms, s, e->scan_ticket.as<int>(),
                                      e->n_overflow.as<int>()),
               "clear counts launch");
    stage_begin(e, ST_HASH);
    FRNN_CHECK(e, launch_hash_count(d_pts, P, e->counts.as<int>(), e->cellrank.as<int2>(), s, nullptr, Pd),
               "hash_count launch");
    stage_end(e, ST_HASH);
    e->epoch = (e->epoch + 1) & 0x3fffffffu;
    if (e->epoch == 0) {
        FRNN_CHECK(e, cudaMemsetAsync(e->scan_status.p, 0, e->scan_status.bytes, s), "memset status");
        e->epoch = 1;
    }
    stage_begin(e, ST_SCAN);
    FRNN_CHECK(e, launch_scan(e->counts.as<int>(), e->starts.as<int>(), budget,
                              e->scan_status.as<unsigned long long>(), e->scan_ticket.as<int>(), e->epoch,
                              e->err_flag.as<int>(), s, e->test_stall == FRNN_TEST_STALL_SCAN ? 1 : -1, Pd),
               "scan launch");
    stage_end(e, ST_SCAN);
    stage_begin(e, ST_SCATTER);
    FRNN_CHECK(e, launch_scatter(d_pts, P, e->cellrank.as<int2>(), e->starts.as<int>(), e->rows.as<float>(),
                                 e->ids.as<int>(), s, lists ? e->inv.as<int>() : nullptr, nullptr, nullptr, Pd),
               "scatter launch");
    stage_end(e, ST_SCATTER);
    e->launches += 5;
    const int st = search_built(e, P, false, K, radius * radius, 0, N, true, out_idx, out_dist, Pd);
    if (st != FRNN_OK) return st;
    FRNN_CHECK(e, cudaMemcpyAsync(e->h_plan, Pd, sizeof(GridPlan), cudaMemcpyDeviceToHost, s), "plan readback");
    return FRNN_OK;
}

// After the sync that ends a device-planned search: the plan it used, or,
// when the GPU found no grid, an error for non-finite data or *brute = true
// (the caller then searches by brute force; every grid kernel returned at
// once).
int finish_dplan(frnn_engine* e, GridPlan* P, bool* brute) {
    *brute = false;
    *P = *static_cast<const GridPlan*>(e->h_plan);
    if (P->cells == 0) {
        if (P->pre_r2 != 0.0f) return fail(e, FRNN_ERR_INVALID_ARG, "points contain NaN or Inf coordinates");
        *brute = true;
    }
    return FRNN_OK;
}

// Brute force with the tcgen05 distance filter (bf_tc.cu), in two halves.
//
// tc_plan: the per-dimension box of the points (and of a separate query set
// d_q of M points), read back to the host, gives the centre and power-of-two
// scale of the fp16 tiles and the filter's threshold constants.  tp->ok is
// false (nothing else launched) when the data do not suit the filter --
// non-finite coordinates, or a radius whose scaled square is not a finite
// fp32 -- and the caller runs the SIMT brute force instead.
int tc_plan(frnn_engine* e, const float* d_pts, int N, int dim, float radius, TcPlan* tp,
            const float* d_q, int M) {
    cudaStream_t s = e->stream;
    tp->ok = false;
    const bool sep = d_q != nullptr;
    const float r2 = radius * radius;
    FRNN_GROW(e, e->tc_box, 1024 * sizeof(float) + 16);
    int* nonfinite = reinterpret_cast<int*>(e->tc_box.as<float>() + 1024);
    stage_begin(e, ST_BBOX);
    FRNN_CHECK(e, cudaMemsetAsync(nonfinite, 0, sizeof(int), s), "memset non-finite flag");
    FRNN_CHECK(e, launch_tc_box(d_pts, N, dim, e->tc_box.as<float>(), nonfinite, s), "box launch");
    e->launches += 3;
    if (sep) {
        FRNN_CHECK(e, launch_tc_box(d_q, M, dim, e->tc_box.as<float>() + 512, nonfinite, s), "box launch");
        e->launches += 3;
    }
    stage_end(e, ST_BBOX);
    float* hq = static_cast<float*>(e->h_pca) + 6144;  // the query set's box
    FRNN_CHECK(e, cudaMemcpyAsync(e->h_tc, e->tc_box.p, 2 * dim * sizeof(float), cudaMemcpyDeviceToHost, s),
               "box readback");
    if (sep)
        FRNN_CHECK(e, cudaMemcpyAsync(hq, e->tc_box.as<float>() + 512, 2 * dim * sizeof(float),
                                      cudaMemcpyDeviceToHost, s),
                   "query box readback");
    FRNN_CHECK(e, cudaMemcpyAsync(e->h_tc + 2 * kMaxK, nonfinite, sizeof(int), cudaMemcpyDeviceToHost, s),
               "flag readback");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "box sync");
    int flag = 0;
    std::memcpy(&flag, e->h_tc + 2 * kMaxK, sizeof(int));
    if (flag != 0) return FRNN_OK;

    // centre = per-dimension midpoint of the box of points (and queries);
    // scale = 2^(14 - e) with max|x - c| < 2^e, so every scaled coordinate
    // stays below 2^14 in magnitude (fp16 max 65504)
    double hmax = 0.0;
    for (int d = 0; d < dim; ++d) {
        double lo = e->h_tc[2 * d], hi = e->h_tc[2 * d + 1];
        if (sep) {
            lo = std::min(lo, (double)hq[2 * d]);
            hi = std::max(hi, (double)hq[2 * d + 1]);
        }
        tp->center[d] = (float)(0.5 * (lo + hi));
        hmax = std::max(hmax, std::max(hi - (double)tp->center[d], (double)tp->center[d] - lo));
    }
    int ex = 0;
    if (hmax > 0.0) std::frexp(hmax * (1.0 + 1e-6), &ex);
    const int sexp = std::max(-120, std::min(120, 14 - ex));
    const double scale = hmax > 0.0 ? std::ldexp(1.0, sexp) : 1.0;
    const double eta = std::ldexp(1.0, -25);
    const double rcd = (double)r2 * scale * scale * (1.0 + std::ldexp(1.0, -15)) + 4.0 * dim * eta * eta;
    float rc = (float)rcd;
    if ((double)rc < rcd) rc = std::nextafter(rc, INFINITY);
    if (!std::isfinite(rc)) return FRNN_OK;
    tp->scale = (float)scale;
    tp->rc = rc;
    tp->one_minus_alpha = 1.0f - std::ldexp(1.0f, -8);
    tp->eta_c = (float)(4.0 * eta * std::sqrt((double)dim));
    tp->ok = true;
    return FRNN_OK;
}

// tc_prepare: fp16 tiles, fp32 rows and threshold terms of the points (and of
// the separate query set) with the plan's centre and scale.
int tc_prepare(frnn_engine* e, const float* d_pts, int N, int dim, const TcPlan& tp, const float* d_q, int M) {
    cudaStream_t s = e->stream;
    const bool sep = d_q != nullptr;
    const int ntiles = (N + 127) / 128, qtiles = (M + 127) / 128;
    const int dp = tc_row_floats(dim);
    FRNN_GROW(e, e->tc_center, (size_t)dim * 4);
    FRNN_GROW(e, e->tc_tiles, (size_t)ntiles * tc_tile_bytes(dim));
    FRNN_GROW(e, e->tc_rows, (size_t)N * dp * 4);
    FRNN_GROW(e, e->tc_qa, (size_t)ntiles * 128 * 4);
    FRNN_GROW(e, e->tc_pb, (size_t)ntiles * 128 * 4);
    // the centre goes through pinned staging (the caller's plan may be on the stack)
    float* hcenter = e->h_tc + 2 * kMaxK + 4;
    std::memcpy(hcenter, tp.center, (size_t)dim * 4);
    stage_begin(e, ST_TC_PREP);
    FRNN_CHECK(e, cudaMemcpyAsync(e->tc_center.p, hcenter, (size_t)dim * 4, cudaMemcpyHostToDevice, s),
               "centre upload");
    FRNN_CHECK(e, launch_tc_prep(d_pts, N, dim, e->tc_center.as<float>(), tp.scale, tp.one_minus_alpha,
                                 tp.eta_c, tp.rc, e->tc_tiles.as<uint8_t>(), e->tc_rows.as<float>(),
                                 e->tc_qa.as<float>(), e->tc_pb.as<float>(), s),
               "prep launch");
    e->launches++;
    if (sep) {
        // the queries' tiles, rows and query-side terms (point-side terms unused)
        FRNN_GROW(e, e->q_tiles, (size_t)qtiles * tc_tile_bytes(dim));
        FRNN_GROW(e, e->q_rows32, (size_t)M * dp * 4);
        FRNN_GROW(e, e->q_qa, (size_t)qtiles * 128 * 4);
        FRNN_GROW(e, e->q_pb, (size_t)qtiles * 128 * 4);
        FRNN_CHECK(e, launch_tc_prep(d_q, M, dim, e->tc_center.as<float>(), tp.scale, tp.one_minus_alpha,
                                     tp.eta_c, tp.rc, e->q_tiles.as<uint8_t>(), e->q_rows32.as<float>(),
                                     e->q_qa.as<float>(), e->q_pb.as<float>(), s),
                   "query prep launch");
        e->launches++;
    }
    stage_end(e, ST_TC_PREP);
    return FRNN_OK;
}

// tc_query_tiles: after tc_prepare, the tensor-core filter over query tiles
// [qb_begin, qb_end), the exact fp32 re-rank, and the SIMT brute force for
// queries whose candidate list overflowed.  Queries [qb_begin*128,
// min(Q, qb_end*128)), results to rows q - qb_begin*128 of out[k*rows + row].
int tc_query_tiles(frnn_engine* e, const float* d_pts, int N, int dim, int K, float radius, int* out_idx,
                   float* out_dist, int qb_begin, int qb_end, const float* d_q, int M) {
    cudaStream_t s = e->stream;
    const bool sep = d_q != nullptr;
    const int Q = sep ? M : N;
    const float r2 = radius * radius;
    const int cap = tc_list_cap(K);
    FRNN_GROW(e, e->lists, (size_t)Q * cap * 4);
    FRNN_GROW(e, e->list_counts, (size_t)Q * 4);
    FRNN_GROW(e, e->overflow, (size_t)Q * 4);
    FRNN_GROW(e, e->n_overflow, 16);
    const float* qa = sep ? e->q_qa.as<float>() : e->tc_qa.as<float>();
    const int q0 = qb_begin * 128, q1 = std::min(Q, qb_end * 128), rows = q1 - q0;
    FRNN_CHECK(e, cudaMemsetAsync(e->n_overflow.p, 0, 4, s), "memset overflow count");
    e->last_overflow_map = 2;
    // a whole self-search filters each unordered pair of tiles once (half the
    // MMAs); its candidate counts are global counters, zeroed here
    const bool sym = !sep && e->tc_symmetric && qb_begin == 0 && qb_end == (N + 127) / 128;
    if (sym) FRNN_CHECK(e, cudaMemsetAsync(e->list_counts.p, 0, (size_t)Q * 4, s), "memset candidate counts");
    stage_begin(e, ST_TC_FILTER);
    FRNN_CHECK(e, launch_tc_filter(e->tc_tiles.as<uint8_t>(), qa, e->tc_pb.as<float>(), N, dim, cap,
                                   e->lists.as<int>(), e->list_counts.as<int>(), e->overflow.as<int>(),
                                   e->n_overflow.as<int>(), e->err_flag.as<int>(), qb_begin, qb_end, s,
                                   sep ? e->q_tiles.as<uint8_t>() : nullptr, Q,
                                   e->test_stall == FRNN_TEST_STALL_TC_FILTER ? 1 : -1, sym),
               "filter launch");
    stage_end(e, ST_TC_FILTER);
    stage_begin(e, ST_TC_RERANK);
    FRNN_CHECK(e, launch_tc_rerank(e->tc_rows.as<float>(), dim, e->lists.as<int>(), e->list_counts.as<int>(),
                                   cap, Q, K, r2, out_idx, out_dist, q0, q1, s,
                                   sep ? e->q_rows32.as<float>() : nullptr),
               "rerank launch");
    stage_end(e, ST_TC_RERANK);
    e->launches += 2;
    // queries with more candidates than their list holds: SIMT brute force
    int* h_nov = reinterpret_cast<int*>(e->h_tc + 2 * kMaxK + 1);
    FRNN_CHECK(e, cudaMemcpyAsync(h_nov, e->n_overflow.p, sizeof(int), cudaMemcpyDeviceToHost, s),
               "overflow count readback");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "overflow count sync");
    if (*h_nov > 0) {
        stage_begin(e, ST_BRUTE);
        FRNN_CHECK(e, launch_bruteforce(d_pts, N, dim, K, r2, 0, *h_nov, out_idx, out_dist, rows, s,
                                        e->overflow.as<int>(), q0, d_q, M),
                   "overflow brute force launch");
        stage_end(e, ST_BRUTE);
        e->launches++;
    }
    return FRNN_OK;
}

int tc_search(frnn_engine* e, const float* d_pts, int N, int dim, int K, float radius, const TcPlan& tp,
              int* out_idx, float* out_dist, int qb_begin, int qb_end, const float* d_q, int M) {
    int st = tc_prepare(e, d_pts, N, dim, tp, d_q, M);
    if (st != FRNN_OK) return st;
    return tc_query_tiles(e, d_pts, N, dim, K, radius, out_idx, out_dist, qb_begin, qb_end, d_q, M);
}

// Both halves; *done = false when the filter does not suit the data (the
// caller then runs the SIMT brute force).
int run_brute_tc(frnn_engine* e, const float* d_pts, int N, int dim, int K, float radius,
                 int* out_idx, float* out_dist, int qb_begin, int qb_end, bool* done,
                 const float* d_q = nullptr, int M = 0) {
    *done = false;
    TcPlan tp;
    int st = tc_plan(e, d_pts, N, dim, radius, &tp, d_q, M);
    if (st != FRNN_OK || !tp.ok) return st;
    st = tc_search(e, d_pts, N, dim, K, radius, tp, out_idx, out_dist, qb_begin, qb_end, d_q, M);
    if (st != FRNN_OK) return st;
    *done = true;
    return FRNN_OK;
}

// Cell histogram, prefix scan and counting-sort scatter of one point set
// (points or queries) on plan P; the scan's status words and ticket are shared.
int sort_into_cells(frnn_engine* e, const float* pts, const GridPlan& P, const float* proj, DevBuf& counts,
                    DevBuf& starts, DevBuf& cellrank, DevBuf& rows, DevBuf& ids, DevBuf* inv,
                    DevBuf* proj_s) {
    cudaStream_t s = e->stream;
    const int n = P.n;
    FRNN_GROW(e, counts, (size_t)P.cells * 4);
    FRNN_GROW(e, starts, ((size_t)P.cells + 1) * 4);
    {
        const int st = grow_scan_status(e, (size_t)scan_tiles(P.cells) * 8);
        if (st != FRNN_OK) return st;
    }
    FRNN_GROW(e, cellrank, (size_t)n * 8);
    // padded: the D = 3 collect kernel reads whole 8-row passes
    FRNN_GROW(e, rows, ((size_t)n + kCollectRowPad) * P.row * 4);
    FRNN_GROW(e, ids, (size_t)n * 4);
    if (inv) FRNN_GROW(e, *inv, (size_t)n * 4);
    if (proj) FRNN_GROW(e, *proj_s, (size_t)n * kProjStride * 4);
    FRNN_CHECK(e, cudaMemsetAsync(counts.p, 0, (size_t)P.cells * 4, s), "memset counts");
    FRNN_CHECK(e, cudaMemsetAsync(e->scan_ticket.p, 0, 4, s), "memset scan ticket");
    FRNN_CHECK(e, launch_hash_count(pts, P, counts.as<int>(), cellrank.as<int2>(), s, proj), "hash_count launch");
    e->epoch = (e->epoch + 1) & 0x3fffffffu;
    if (e->epoch == 0) {
        FRNN_CHECK(e, cudaMemsetAsync(e->scan_status.p, 0, e->scan_status.bytes, s), "memset status");
        e->epoch = 1;
    }
    FRNN_CHECK(e, launch_scan(counts.as<int>(), starts.as<int>(), P.cells, e->scan_status.as<unsigned long long>(),
                              e->scan_ticket.as<int>(), e->epoch, e->err_flag.as<int>(), s,
                              e->test_stall == FRNN_TEST_STALL_SCAN ? 1 : -1),
               "scan launch");
    FRNN_CHECK(e, launch_scatter(pts, P, cellrank.as<int2>(), starts.as<int>(), rows.as<float>(), ids.as<int>(), s,
                                 inv ? inv->as<int>() : nullptr, proj, proj ? proj_s->as<float>() : nullptr),
               "scatter launch");
    e->launches += 3;
    return FRNN_OK;
}

// Grid search of a separate query set against the points: the queries are
// sorted into the points' grid (the same plan) so that neighbouring queries
// read the same candidate rows; results out[k*M + q] in query order.
// The second half: the points are already sorted into P's cells (rows, ids,
// starts, and their projected coordinates when proj_p).
int search_sorted_queries(frnn_engine* e, const float* d_q, int M, int K, float r2, const GridPlan& P,
                          bool proj_p, const float* proj_q, int* out_idx, float* out_dist) {
    cudaStream_t s = e->stream;
    GridPlan Pq = P;
    Pq.n = M;
    stage_begin(e, ST_HASH);
    int st = sort_into_cells(e, d_q, Pq, proj_q, e->q_counts, e->q_starts, e->q_cellrank, e->q_rows, e->q_ids,
                             &e->q_inv, &e->q_proj_s);
    if (st != FRNN_OK) return st;
    stage_end(e, ST_HASH);
    const float* proj_s = proj_p ? e->proj_s.as<float>() : nullptr;
    const float* qproj_s = proj_q ? e->q_proj_s.as<float>() : nullptr;
    const bool d3 = P.dim == 3 && P.g == 3 && !proj_p;
    if (K <= 32 && (d3 || list_search_nd(e, P))) {
        const int cap = K <= 16 ? 64 : 128;
        FRNN_GROW(e, e->lists, (size_t)M * cap * 8);
        FRNN_GROW(e, e->list_counts, (size_t)M * 4);
        FRNN_GROW(e, e->overflow, (size_t)M * 4);
        FRNN_GROW(e, e->n_overflow, 16);
        FRNN_CHECK(e, cudaMemsetAsync(e->n_overflow.p, 0, 4, s), "memset overflow count");
        e->last_overflow_map = 3;
        stage_begin(e, ST_COLLECT);
        if (d3)
            FRNN_CHECK(e, launch_collect_d3(e->rows.as<float>(), e->starts.as<int>(), P, r2, cap,
                                            e->lists.as<unsigned long long>(), e->list_counts.as<int>(),
                                            e->overflow.as<int>(), e->n_overflow.as<int>(), 0, M, s,
                                            e->q_rows.as<float>()),
                       "collect launch");
        else
            FRNN_CHECK(e, launch_collect_nd(e->rows.as<float>(), e->ids.as<int>(), e->starts.as<int>(), P, r2,
                                            cap, e->lists.as<unsigned long long>(), e->list_counts.as<int>(),
                                            e->overflow.as<int>(), e->n_overflow.as<int>(), 0, M, s,
                                            e->q_rows.as<float>(), qproj_s),
                       "collect launch");
        stage_end(e, ST_COLLECT);
        stage_begin(e, ST_EMIT);
        FRNN_CHECK(e, launch_emit_lists(e->lists.as<unsigned long long>(), e->list_counts.as<int>(),
                                        e->q_inv.as<int>(), 0, M, K, cap, r2, out_idx, out_dist, s),
                   "emit launch");
        FRNN_CHECK(e, launch_grid_search(e->rows.as<float>(), e->ids.as<int>(), e->starts.as<int>(), P, K, r2, 0,
                                         M, out_idx, out_dist, M, e->q_ids.as<int>(), s, e->overflow.as<int>(),
                                         e->n_overflow.as<int>(), -1, proj_s, e->q_rows.as<float>(), qproj_s),
                   "overflow search launch");
        stage_end(e, ST_EMIT);
        e->launches += 3;
        return FRNN_OK;
    }
    stage_begin(e, ST_SEARCH);
    if ((long long)M * K * 8 <= e->direct_output_max_bytes) {
        FRNN_CHECK(e, launch_grid_search(e->rows.as<float>(), e->ids.as<int>(), e->starts.as<int>(), P, K, r2, 0,
                                         M, out_idx, out_dist, M, e->q_ids.as<int>(), s, nullptr, nullptr, -1,
                                         proj_s, e->q_rows.as<float>(), qproj_s),
                   "grid search launch");
        stage_end(e, ST_SEARCH);
        e->launches++;
        return FRNN_OK;
    }
    FRNN_GROW(e, e->tmp_idx, (size_t)M * K * 4);
    FRNN_GROW(e, e->tmp_dist, (size_t)M * K * 4);
    FRNN_CHECK(e, launch_grid_search(e->rows.as<float>(), e->ids.as<int>(), e->starts.as<int>(), P, K, r2, 0, M,
                                     e->tmp_idx.as<int>(), e->tmp_dist.as<float>(), M, nullptr, s, nullptr,
                                     nullptr, -1, proj_s, e->q_rows.as<float>(), qproj_s),
               "grid search launch");
    stage_end(e, ST_SEARCH);
    stage_begin(e, ST_UNPERMUTE);
    FRNN_CHECK(e, launch_unpermute(e->tmp_idx.as<int>(), e->tmp_dist.as<float>(), e->q_ids.as<int>(), M, K,
                                   out_idx, out_dist, s),
               "unpermute launch");
    stage_end(e, ST_UNPERMUTE);
    e->launches += 2;
    return FRNN_OK;
}

int run_grid_queries(frnn_engine* e, const float* d_pts, int N, const float* d_q, int M, int dim, int K,
                     float r2, const GridPlan& P, const float* proj_p, const float* proj_q, int* out_idx,
                     float* out_dist) {
    stage_begin(e, ST_SCATTER);
    int st = sort_into_cells(e, d_pts, P, proj_p, e->counts, e->starts, e->cellrank, e->rows, e->ids, nullptr,
                             &e->proj_s);
    if (st != FRNN_OK) return st;
    stage_end(e, ST_SCATTER);
    return search_sorted_queries(e, d_q, M, K, r2, P, proj_p != nullptr, proj_q, out_idx, out_dist);
}

// Checks a query set for NaN/Inf (the grid's leading coordinates; all of them
// through the projection when the grid is on principal axes) and projects it
// on the principal axes planned for the points.
int prepare_queries(frnn_engine* e, const float* d_q, int M, int dim, bool principal) {
    cudaStream_t s = e->stream;
    const int g = grid_axes_for(dim);
    const int blocks = std::min(bbox_blocks(M, e->sms), kBoxMaxBlocks);
    FRNN_GROW(e, e->q_box_out, 64);
    FRNN_CHECK(e, launch_bbox(d_q, M, g, e->box_partial.as<float>(), e->box_ticket.as<unsigned>(),
                              e->q_box_out.as<float>(), blocks, s),
               "query bbox launch");
    e->launches++;
    float* hqb = static_cast<float*>(e->h_pca) + 6144;
    FRNN_CHECK(e, cudaMemcpyAsync(hqb, e->q_box_out.p, 9 * sizeof(float), cudaMemcpyDeviceToHost, s),
               "query bbox readback");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "query bbox sync");
    if (hqb[8] != 0.0f) return fail(e, FRNN_ERR_INVALID_ARG, "queries contain NaN or Inf coordinates");
    if (!principal) return FRNN_OK;
    const int axes = std::min(dim, kMaxGridAxes);
    const int pslots = pca_project_slots();
    FRNN_GROW(e, e->q_proj_u, (size_t)M * kProjStride * 4);
    FRNN_GROW(e, e->q_proj_partial, (size_t)blocks * pslots * 4);
    FRNN_GROW(e, e->q_proj_out, 64 * 4);
    FRNN_CHECK(e, launch_pca_project(d_q, M, dim, axes, e->pca_mu.as<float>(), e->pca_pm.as<float>(),
                                     e->q_proj_u.as<float>(), e->q_proj_partial.as<float>(),
                                     e->proj_ticket.as<unsigned>(), e->q_proj_out.as<float>(), blocks, s),
               "query project launch");
    e->launches++;
    float* hqp = static_cast<float*>(e->h_pca) + 6400;
    FRNN_CHECK(e, cudaMemcpyAsync(hqp, e->q_proj_out.p, (size_t)pslots * 4, cudaMemcpyDeviceToHost, s),
               "query projection readback");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "query projection sync");
    if (hqp[pslots - 1] != 0.0f) return fail(e, FRNN_ERR_INVALID_ARG, "queries contain NaN or Inf coordinates");
    e->q_proj_delta = projection_delta(dim, (double)hqp[pslots - 2]);
    return FRNN_OK;
}

// Blocking end of a search: the bounded device waits' error flag.
int finish_search(frnn_engine* e) {
    cudaStream_t s = e->stream;
    FRNN_CHECK(e, cudaMemcpyAsync(e->h_err, e->err_flag.p, sizeof(int), cudaMemcpyDeviceToHost, s),
               "error flag readback");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "search sync");
    if (*e->h_err != 0) {
        cudaMemsetAsync(e->err_flag.p, 0, sizeof(int), s);
        cudaStreamSynchronize(s);
        return fail(e, FRNN_ERR_TIMEOUT, "a bounded device-side wait gave up");
    }
    return FRNN_OK;
}

// A separate query set (M points, SoA) against the N points: the same paths
// and arithmetic as the self-query; results out[k*M + q].
int search_queries_core(frnn_engine* e, const float* d_pts, int N, const float* d_q, int M, int dim, int K,
                        float radius) {
    cudaStream_t s = e->stream;
    const float r2 = radius * radius;
    FRNN_GROW(e, e->out_idx, (size_t)M * K * 4);
    FRNN_GROW(e, e->out_dist, (size_t)M * K * 4);
    int* out_idx = e->out_idx.as<int>();
    float* out_dist = e->out_dist.as<float>();
    e->last_N = -1;
    e->last_part_rows = -1;
    e->built.valid = false;  // the point buffers are about to be overwritten
    e->last_overflow_map = 0;
    for (int i = 0; i < FRNN_STAGES; ++i) e->stage_used[i] = false;
    int path = e->forced_path;
    if (path == FRNN_PATH_AUTO) {
        const double work = (double)N * (double)M * dim;
        if (dim > 32) path = N >= kTcMinPoints ? FRNN_PATH_BRUTE_TC : FRNN_PATH_BRUTE;
        else if (work <= kBruteSmallWork) path = FRNN_PATH_BRUTE;
        else path = FRNN_PATH_GRID;
    }
    if (path == FRNN_PATH_GRID && dim > 32) path = FRNN_PATH_BRUTE;

    GridPlan P{};
    bool grid_ok = false, principal = false;
    if (path == FRNN_PATH_GRID) {
        const int g = grid_axes_for(dim);
        const int blocks = std::min(bbox_blocks(std::max(N, M), e->sms), kBoxMaxBlocks);
        FRNN_GROW(e, e->q_box_out, 64);
        stage_begin(e, ST_BBOX);
        FRNN_CHECK(e, launch_bbox(d_pts, N, g, e->box_partial.as<float>(), e->box_ticket.as<unsigned>(),
                                  e->box_out.as<float>(), blocks, s),
                   "bbox launch");
        FRNN_CHECK(e, launch_bbox(d_q, M, g, e->box_partial.as<float>(), e->box_ticket.as<unsigned>(),
                                  e->q_box_out.as<float>(), blocks, s),
                   "query bbox launch");
        stage_end(e, ST_BBOX);
        e->launches += 2;
        float* hqb = static_cast<float*>(e->h_pca) + 6144;
        FRNN_CHECK(e, cudaMemcpyAsync(e->h_box, e->box_out.p, 9 * sizeof(float), cudaMemcpyDeviceToHost, s),
                   "bbox readback");
        FRNN_CHECK(e, cudaMemcpyAsync(hqb, e->q_box_out.p, 9 * sizeof(float), cudaMemcpyDeviceToHost, s),
                   "query bbox readback");
        FRNN_CHECK(e, cudaStreamSynchronize(s), "bbox sync");
        if (e->h_box[8] != 0.0f || hqb[8] != 0.0f)
            return fail(e, FRNN_ERR_INVALID_ARG, "points or queries contain NaN or Inf coordinates");
        // the grid covers the points; queries outside it clamp to the edge
        // cells, whose shells still hold every point within r of them
        grid_ok = make_plan(e->h_box, N, dim, radius, P);
        if (dim > 4 && dim <= kMaxPcaDim && e->grid_axes_mode != FRNN_GRID_AXES_LEADING) {
            int st = plan_principal(e, d_pts, N, dim, radius, grid_ok, P, &principal);
            if (st != FRNN_OK) return st;
            grid_ok |= principal;
        }
        if (!grid_ok) path = FRNN_PATH_BRUTE;
    }
    if (path == FRNN_PATH_GRID && principal) {
        // the queries' projected coordinates on the same axes
        const int axes = std::min(dim, kMaxGridAxes);
        const int pblocks = std::min(bbox_blocks(M, e->sms), kBoxMaxBlocks);
        const int pslots = pca_project_slots();
        FRNN_GROW(e, e->q_proj_u, (size_t)M * kProjStride * 4);
        FRNN_GROW(e, e->q_proj_partial, (size_t)pblocks * pslots * 4);
        FRNN_GROW(e, e->q_proj_out, 64 * 4);
        FRNN_CHECK(e, launch_pca_project(d_q, M, dim, axes, e->pca_mu.as<float>(), e->pca_pm.as<float>(),
                                         e->q_proj_u.as<float>(), e->q_proj_partial.as<float>(),
                                         e->proj_ticket.as<unsigned>(), e->q_proj_out.as<float>(), pblocks, s),
                   "query project launch");
        e->launches++;
        float* hqp = static_cast<float*>(e->h_pca) + 6400;
        FRNN_CHECK(e, cudaMemcpyAsync(hqp, e->q_proj_out.p, (size_t)pslots * 4, cudaMemcpyDeviceToHost, s),
                   "query projection readback");
        FRNN_CHECK(e, cudaStreamSynchronize(s), "query projection sync");
        if (hqp[pslots - 1] != 0.0f)
            return fail(e, FRNN_ERR_INVALID_ARG, "points or queries contain NaN or Inf coordinates");
        // the queries' own projection rounding widens the screening bound
        P.pre_r2 = screen_r2(radius, P.g, e->proj_delta + projection_delta(dim, (double)hqp[pslots - 2]));
    }
    if (path == FRNN_PATH_BRUTE_TC) {
        bool done = false;
        int st = run_brute_tc(e, d_pts, N, dim, K, radius, out_idx, out_dist, 0, (M + 127) / 128, &done, d_q, M);
        if (st != FRNN_OK) return st;
        if (!done) path = FRNN_PATH_BRUTE;
    }
    if (path == FRNN_PATH_GRID) {
        int st = run_grid_queries(e, d_pts, N, d_q, M, dim, K, r2, P, principal ? e->proj_u.as<float>() : nullptr,
                                  principal ? e->q_proj_u.as<float>() : nullptr, out_idx, out_dist);
        if (st != FRNN_OK) return st;
        e->last_g = P.g;
        e->last_cells = P.cells;
    } else {
        e->last_g = 0;
        e->last_cells = 0;
        if (path == FRNN_PATH_BRUTE) {
            stage_begin(e, ST_BRUTE);
            FRNN_CHECK(e, launch_bruteforce(d_pts, N, dim, K, r2, 0, M, out_idx, out_dist, M, s, nullptr, 0, d_q, M),
                       "bruteforce launch");
            stage_end(e, ST_BRUTE);
            e->launches++;
        }
    }
    e->last_path = path;
    e->last_principal = path == FRNN_PATH_GRID && principal;
    FRNN_CHECK(e, cudaMemcpyAsync(e->h_err, e->err_flag.p, sizeof(int), cudaMemcpyDeviceToHost, s),
               "error flag readback");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "search sync");
    if (*e->h_err != 0) {
        cudaMemsetAsync(e->err_flag.p, 0, sizeof(int), s);
        cudaStreamSynchronize(s);
        return fail(e, FRNN_ERR_TIMEOUT, "a bounded device-side wait gave up");
    }
    e->last_N = M;
    e->last_K = K;
    return FRNN_OK;
}

int self_search_path(const frnn_engine* e, int N, int dim) {
    int path = e->forced_path;
    if (path == FRNN_PATH_AUTO) {
        const double work = (double)N * (double)N * dim;
        if (dim > 32) path = N >= kTcMinPoints ? FRNN_PATH_BRUTE_TC : FRNN_PATH_BRUTE;
        else if (work <= kBruteSmallWork) path = FRNN_PATH_BRUTE;
        else path = FRNN_PATH_GRID;
    }
    if (path == FRNN_PATH_GRID && dim > 32) path = FRNN_PATH_BRUTE;
    return path;
}

int plan_grid_search(frnn_engine* e, const float* d_pts, int N, int dim, float radius, int* path, GridPlan& P,
                     bool* principal) {
    cudaStream_t s = e->stream;
    *principal = false;
    const int g = grid_axes_for(dim);
    const int blocks = std::min(bbox_blocks(N, e->sms), kBoxMaxBlocks);
    stage_begin(e, ST_BBOX);
    FRNN_CHECK(e, launch_bbox(d_pts, N, g, e->box_partial.as<float>(), e->box_ticket.as<unsigned>(),
                              e->box_out.as<float>(), blocks, s),
               "bbox launch");
    stage_end(e, ST_BBOX);
    e->launches++;
    FRNN_CHECK(e, cudaMemcpyAsync(e->h_box, e->box_out.p, 9 * sizeof(float), cudaMemcpyDeviceToHost, s),
               "bbox readback");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "bbox sync");
    if (e->h_box[8] != 0.0f) return fail(e, FRNN_ERR_INVALID_ARG, "points contain NaN or Inf coordinates");
    bool grid_ok = make_plan(e->h_box, N, dim, radius, P);
    if (dim > 4 && dim <= kMaxPcaDim && e->grid_axes_mode != FRNN_GRID_AXES_LEADING) {
        int st = plan_principal(e, d_pts, N, dim, radius, grid_ok, P, principal);
        if (st != FRNN_OK) return st;
        grid_ok |= *principal;
    }
    if (!grid_ok) *path = FRNN_PATH_BRUTE;
    return FRNN_OK;
}

// Whole search (nparts == 0): every query, results out[k*N + q].  Part search
// (0 <= part < nparts): the part-th of nparts contiguous slices of the path's
// query order -- cell order on the grid path, input order on brute force,
// whole 128-query tiles on the tensor-core path -- with row j of
// out[k*rows + j] belonging to query part_ids[j].  The slices of all parts
// cover every query exactly once.
int search_core(frnn_engine* e, const float* d_pts, int N, int dim, int K, float radius,
                bool blocking, int part = 0, int nparts = 0) {
    cudaStream_t s = e->stream;
    const float r2 = radius * radius;
    const bool is_part = nparts > 0;
    FRNN_GROW(e, e->out_idx, (size_t)N * K * 4);
    FRNN_GROW(e, e->out_dist, (size_t)N * K * 4);
    int* out_idx = e->out_idx.as<int>();
    float* out_dist = e->out_dist.as<float>();
    e->last_N = -1;
    e->last_part_rows = -1;
    e->built.valid = false;  // the point buffers are about to be overwritten
    e->last_overflow_map = 0;

    for (int i = 0; i < FRNN_STAGES; ++i) e->stage_used[i] = false;
    int path = self_search_path(e, N, dim);

    // this call's slice: [s0, s1) of the query order (tiles [qb0, qb1) on the
    // tensor-core path)
    const int ntq = (N + 127) / 128;
    int qb0 = 0, qb1 = ntq, s0 = 0, s1 = N;
    if (is_part && path == FRNN_PATH_BRUTE_TC) {
        qb0 = (int)((long long)ntq * part / nparts);
        qb1 = (int)((long long)ntq * (part + 1) / nparts);
        s0 = std::min(N, qb0 * 128);
        s1 = std::min(N, qb1 * 128);
    } else if (is_part) {
        s0 = (int)((long long)N * part / nparts);
        s1 = (int)((long long)N * (part + 1) / nparts);
    }
    int rows = s1 - s0;

    GridPlan P{};
    bool principal = false;
    const bool dplan = uses_device_plan(e, path, dim, blocking, is_part);
    if (dplan) {
        int st = run_grid_dplan(e, d_pts, N, dim, K, radius, out_idx, out_dist);
        if (st != FRNN_OK) return st;
        FRNN_CHECK(e, cudaMemcpyAsync(e->h_err, e->err_flag.p, sizeof(int), cudaMemcpyDeviceToHost, s),
                   "error flag readback");
        FRNN_CHECK(e, cudaStreamSynchronize(s), "search sync");
        if (*e->h_err != 0) {
            cudaMemsetAsync(e->err_flag.p, 0, sizeof(int), s);
            cudaStreamSynchronize(s);
            return fail(e, FRNN_ERR_TIMEOUT, "a bounded device-side wait gave up");
        }
        bool brute = false;
        st = finish_dplan(e, &P, &brute);
        if (st != FRNN_OK) return st;
        if (!brute) {
            e->last_g = P.g;
            e->last_cells = P.cells;
        }
        // no useful grid: every grid kernel returned at once; brute force
        // below, then the usual blocking tail
        path = brute ? FRNN_PATH_BRUTE : FRNN_PATH_GRID;
    } else if (path == FRNN_PATH_GRID) {
        int st = plan_grid_search(e, d_pts, N, dim, radius, &path, P, &principal);
        if (st != FRNN_OK) return st;
    }

    if (path == FRNN_PATH_BRUTE_TC) {
        bool done = false;
        int st = run_brute_tc(e, d_pts, N, dim, K, radius, out_idx, out_dist, qb0, qb1, &done);
        if (st != FRNN_OK) return st;
        if (!done) path = FRNN_PATH_BRUTE;
        e->last_g = 0;
        e->last_cells = 0;
    }
    if (path == FRNN_PATH_GRID && !dplan) {
        int st = run_grid(e, d_pts, N, dim, K, r2, P, out_idx, out_dist, is_part, s0, s1,
                          principal ? e->proj_u.as<float>() : nullptr);
        if (st != FRNN_OK) return st;
        rows = s1 - s0;
        e->last_g = P.g;
        e->last_cells = P.cells;
    } else if (path == FRNN_PATH_BRUTE) {
        stage_begin(e, ST_BRUTE);
        FRNN_CHECK(e, launch_bruteforce(d_pts, N, dim, K, r2, s0, s1, out_idx, out_dist, rows, s),
                   "bruteforce launch");
        stage_end(e, ST_BRUTE);
        e->launches++;
        e->last_g = 0;
        e->last_cells = 0;
    }
    if (is_part) {
        FRNN_GROW(e, e->part_ids, (size_t)std::max(rows, 1) * 4);
        if (rows > 0) {
            if (path == FRNN_PATH_GRID)
                FRNN_CHECK(e, cudaMemcpyAsync(e->part_ids.p, e->ids.as<int>() + s0, (size_t)rows * 4,
                                              cudaMemcpyDeviceToDevice, s),
                           "part ids copy");
            else
                FRNN_CHECK(e, launch_iota(e->part_ids.as<int>(), s0, rows, s), "part ids launch");
        }
    }
    e->last_path = path;
    e->last_principal = path == FRNN_PATH_GRID && principal;
    // (a device-planned grid search has had its sync and its error check)
    if (blocking && !(dplan && path == FRNN_PATH_GRID)) {
        FRNN_CHECK(e, cudaMemcpyAsync(e->h_err, e->err_flag.p, sizeof(int), cudaMemcpyDeviceToHost, s),
                   "error flag readback");
        FRNN_CHECK(e, cudaStreamSynchronize(s), "search sync");
        if (*e->h_err != 0) {
            cudaMemsetAsync(e->err_flag.p, 0, sizeof(int), s);
            cudaStreamSynchronize(s);
            return fail(e, FRNN_ERR_TIMEOUT, "a bounded device-side wait gave up");
        }
    }
    if (is_part) {
        e->last_part_rows = rows;
    } else {
        e->last_N = N;
    }
    e->last_K = K;
    return FRNN_OK;
}

}  // namespace eng
}  // namespace frnn

using namespace frnn::eng;

// ---- C ABI ------------------------------------------------------------------------

extern "C" {

const char* frnn_status_string(int status) {
    switch (status) {
        case FRNN_OK: return "ok";
        case FRNN_ERR_INVALID_ARG: return "invalid argument";
        case FRNN_ERR_OOM: return "out of memory";
        case FRNN_ERR_CUDA: return "CUDA error";
        case FRNN_ERR_TIMEOUT: return "device wait timed out";
        case FRNN_ERR_NO_DEVICE: return "no usable CUDA device";
        case FRNN_ERR_STATE: return "invalid call order";
        case FRNN_ERR_COMM: return "collective communication failed";
        default: return "unknown status";
    }
}

const char* frnn_last_error(const frnn_engine* e) { return e ? e->last_error.c_str() : ""; }

int frnn_create(int max_points, int device, frnn_engine** out) {
    if (!out) return FRNN_ERR_INVALID_ARG;
    *out = nullptr;
    if (max_points <= 0) return FRNN_ERR_INVALID_ARG;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return FRNN_ERR_NO_DEVICE;
    }
    if (device < 0 && cudaGetDevice(&device) != cudaSuccess) return FRNN_ERR_NO_DEVICE;
    if (device >= ndev) return FRNN_ERR_INVALID_ARG;
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return FRNN_ERR_NO_DEVICE;
    if (prop.major < 10) return FRNN_ERR_NO_DEVICE;  // kernels are built for sm_100a only
    frnn_engine* e = new frnn_engine();
    e->device = device;
    e->max_points = max_points;
    e->sms = prop.multiProcessorCount;
    DeviceGuard g(device);
    int st = FRNN_OK;
    if ((st = grow(e, e->box_partial, (size_t)kBoxMaxBlocks * 9 * 4, "box_partial")) ||
        (st = grow(e, e->box_ticket, 16, "box_ticket")) || (st = grow(e, e->box_out, 64, "box_out")) ||
        (st = grow(e, e->scan_ticket, 16, "scan_ticket")) || (st = grow(e, e->err_flag, 16, "err_flag"))) {
        frnn_destroy(e);
        return st;
    }
    if (cudaMemset(e->box_ticket.p, 0, e->box_ticket.bytes) != cudaSuccess ||
        cudaMemset(e->err_flag.p, 0, e->err_flag.bytes) != cudaSuccess ||
        cudaMallocHost(&e->h_box, 64) != cudaSuccess || cudaMallocHost(&e->h_err, 64) != cudaSuccess ||
        cudaMallocHost(&e->h_tc, 512 * sizeof(float)) != cudaSuccess ||
        cudaMallocHost(&e->h_pca, 32768) != cudaSuccess ||
        cudaMallocHost(&e->h_plan, sizeof(GridPlan)) != cudaSuccess) {
        cudaGetLastError();
        frnn_destroy(e);
        return FRNN_ERR_OOM;
    }
    *e->h_err = 0;
    *out = e;
    return FRNN_OK;
}

int frnn_destroy(frnn_engine* e) {
    if (!e) return FRNN_OK;
    {
        DeviceGuard g(e->device);
        if (e->stream) cudaStreamSynchronize(e->stream);
        DevBuf* bufs[] = {&e->box_partial, &e->box_ticket, &e->box_out, &e->counts, &e->starts,
                          &e->scan_status, &e->scan_ticket, &e->err_flag, &e->cellrank, &e->rows,
                          &e->ids, &e->inv, &e->lists, &e->list_counts, &e->overflow,
                          &e->n_overflow, &e->tmp_idx, &e->tmp_dist, &e->out_idx, &e->out_dist,
                          &e->in_stage, &e->in_soa, &e->out_rm_idx, &e->out_rm_dist,
                          &e->tc_box, &e->tc_center, &e->tc_tiles, &e->tc_rows, &e->tc_qa,
                          &e->tc_pb, &e->part_ids, &e->pca_partial, &e->pca_moments, &e->pca_mu,
                          &e->pca_pm, &e->proj_box_partial, &e->proj_ticket, &e->proj_out,
                          &e->proj_u, &e->proj_s, &e->pca_smp, &e->pca_h, &e->pca_counts,
                          &e->q_counts, &e->q_starts, &e->q_cellrank, &e->q_rows, &e->q_ids, &e->q_inv,
                          &e->q_proj_u, &e->q_proj_s, &e->q_proj_partial, &e->q_proj_out, &e->q_box_out,
                          &e->q_tiles, &e->q_rows32, &e->q_qa, &e->q_pb, &e->ovf_ids, &e->dplan};
        for (DevBuf* b : bufs) free_buf(*b);
        for (cudaEvent_t& ev : e->ev)
            if (ev) cudaEventDestroy(ev);
        if (e->h_box) cudaFreeHost(e->h_box);
        if (e->h_err) cudaFreeHost(e->h_err);
        if (e->h_tc) cudaFreeHost(e->h_tc);
        if (e->h_pca) cudaFreeHost(e->h_pca);
        if (e->h_plan) cudaFreeHost(e->h_plan);
    }
    delete e;
    return FRNN_OK;
}

int frnn_set_stream(frnn_engine* e, void* stream) {
    if (!e) return FRNN_ERR_INVALID_ARG;
    e->stream = static_cast<cudaStream_t>(stream);
    return FRNN_OK;
}

int frnn_set_path(frnn_engine* e, int path) {
    if (!e) return FRNN_ERR_INVALID_ARG;
    if (path < FRNN_PATH_AUTO || path > FRNN_PATH_BRUTE_TC)
        return fail(e, FRNN_ERR_INVALID_ARG, "unknown path");
    e->forced_path = path;
    return FRNN_OK;
}

int frnn_last_grid_axes(const frnn_engine* e, int* axes) {
    if (!e || !axes) return FRNN_ERR_INVALID_ARG;
    *axes = e->last_principal ? FRNN_GRID_AXES_PRINCIPAL : FRNN_GRID_AXES_LEADING;
    return FRNN_OK;
}

int frnn_set_option(frnn_engine* e, int option, int64_t value) {
    if (!e) return FRNN_ERR_INVALID_ARG;
    switch (option) {
        case FRNN_OPT_DIRECT_OUTPUT_MAX_BYTES:
            if (value < 0) return fail(e, FRNN_ERR_INVALID_ARG, "value must be >= 0");
            e->direct_output_max_bytes = value;
            return FRNN_OK;
        case FRNN_OPT_GRID_AXES:
            if (value < FRNN_GRID_AXES_AUTO || value > FRNN_GRID_AXES_PRINCIPAL)
                return fail(e, FRNN_ERR_INVALID_ARG, "grid axes must be AUTO, LEADING or PRINCIPAL");
            e->grid_axes_mode = (int)value;
            return FRNN_OK;
        case FRNN_OPT_LIST_SEARCH:
            if (value < FRNN_LIST_SEARCH_AUTO || value > FRNN_LIST_SEARCH_NEVER)
                return fail(e, FRNN_ERR_INVALID_ARG, "list search must be AUTO, ALWAYS or NEVER");
            e->list_search = (int)value;
            return FRNN_OK;
        case FRNN_OPT_TEST_STALL:
            if (value < FRNN_TEST_STALL_OFF || value > FRNN_TEST_STALL_TC_FILTER)
                return fail(e, FRNN_ERR_INVALID_ARG, "test stall must be OFF, SCAN or TC_FILTER");
            e->test_stall = (int)value;
            return FRNN_OK;
        case FRNN_OPT_TC_SYMMETRIC:
            if (value < 0 || value > 1) return fail(e, FRNN_ERR_INVALID_ARG, "tc symmetric must be 0 or 1");
            e->tc_symmetric = (int)value;
            return FRNN_OK;
        case FRNN_OPT_DEVICE_PLAN:
            if (value < 0 || value > 1) return fail(e, FRNN_ERR_INVALID_ARG, "device plan must be 0 or 1");
            e->device_plan = (int)value;
            return FRNN_OK;
        default:
            return fail(e, FRNN_ERR_INVALID_ARG, "unknown option");
    }
}

int frnn_last_plan(const frnn_engine* e, int* path, int* grid_dims, int64_t* cells) {
    if (!e) return FRNN_ERR_INVALID_ARG;
    if (path) *path = e->last_path;
    if (grid_dims) *grid_dims = e->last_g;
    if (cells) *cells = e->last_cells;
    return FRNN_OK;
}

static int search_gpu_impl(frnn_engine* e, const float* d_points_soa, int N, int dim, int K,
                           float radius, int** d_idxs, float** d_dists, bool blocking) {
    int st = check_search_args(e, d_points_soa, N, dim, K, radius);
    if (st != FRNN_OK) return st;
    if (!d_idxs || !d_dists) return fail(e, FRNN_ERR_INVALID_ARG, "output pointers are null");
    DeviceGuard g(e->device);
    st = check_device_ptr(e, d_points_soa);
    if (st != FRNN_OK) return st;
    st = search_core(e, d_points_soa, N, dim, K, radius, blocking);
    if (st != FRNN_OK) return st;
    *d_idxs = e->out_idx.as<int>();
    *d_dists = e->out_dist.as<float>();
    return FRNN_OK;
}

int frnn_search_gpu(frnn_engine* e, const float* d_points_soa, int N, int dim, int K, float radius,
                    int** d_idxs, float** d_dists) {
    return search_gpu_impl(e, d_points_soa, N, dim, K, radius, d_idxs, d_dists, true);
}

int frnn_search_gpu_async(frnn_engine* e, const float* d_points_soa, int N, int dim, int K,
                          float radius, int** d_idxs, float** d_dists) {
    return search_gpu_impl(e, d_points_soa, N, dim, K, radius, d_idxs, d_dists, false);
}

int frnn_search_gpu_queries(frnn_engine* e, const float* d_points_soa, int N, const float* d_queries_soa, int M,
                            int dim, int K, float radius, int** d_idxs, float** d_dists) {
    int st = check_search_args(e, d_points_soa, N, dim, K, radius);
    if (st != FRNN_OK) return st;
    if (!d_queries_soa || M < 1) return fail(e, FRNN_ERR_INVALID_ARG, "queries must be a device array of M >= 1 points");
    if (!d_idxs || !d_dists) return fail(e, FRNN_ERR_INVALID_ARG, "output pointers are null");
    DeviceGuard g(e->device);
    st = check_device_ptr(e, d_points_soa);
    if (st != FRNN_OK) return st;
    st = check_device_ptr(e, d_queries_soa);
    if (st != FRNN_OK) return st;
    st = search_queries_core(e, d_points_soa, N, d_queries_soa, M, dim, K, radius);
    if (st != FRNN_OK) return st;
    *d_idxs = e->out_idx.as<int>();
    *d_dists = e->out_dist.as<float>();
    return FRNN_OK;
}

int frnn_build_grid(frnn_engine* e, const float* d_points_soa, int N, int dim, float radius) {
    int st = check_search_args(e, d_points_soa, N, dim, 1, radius);
    if (st != FRNN_OK) return st;
    DeviceGuard g(e->device);
    st = check_device_ptr(e, d_points_soa);
    if (st != FRNN_OK) return st;
    cudaStream_t s = e->stream;
    e->built.valid = false;
    e->last_N = -1;
    e->last_part_rows = -1;
    e->last_overflow_map = 0;
    for (int i = 0; i < FRNN_STAGES; ++i) e->stage_used[i] = false;
    int path = e->forced_path;
    if (path == FRNN_PATH_AUTO)
        path = dim > 32 ? (N >= kTcMinPoints ? FRNN_PATH_BRUTE_TC : FRNN_PATH_BRUTE) : FRNN_PATH_GRID;
    if (path == FRNN_PATH_GRID && dim > 32) path = FRNN_PATH_BRUTE;
    GridPlan P{};
    bool principal = false;
    if (path == FRNN_PATH_GRID) {
        const int blocks = std::min(bbox_blocks(N, e->sms), kBoxMaxBlocks);
        stage_begin(e, ST_BBOX);
        FRNN_CHECK(e, launch_bbox(d_points_soa, N, grid_axes_for(dim), e->box_partial.as<float>(),
                                  e->box_ticket.as<unsigned>(), e->box_out.as<float>(), blocks, s),
                   "bbox launch");
        stage_end(e, ST_BBOX);
        e->launches++;
        FRNN_CHECK(e, cudaMemcpyAsync(e->h_box, e->box_out.p, 9 * sizeof(float), cudaMemcpyDeviceToHost, s),
                   "bbox readback");
        FRNN_CHECK(e, cudaStreamSynchronize(s), "bbox sync");
        if (e->h_box[8] != 0.0f) return fail(e, FRNN_ERR_INVALID_ARG, "points contain NaN or Inf coordinates");
        bool ok = make_plan(e->h_box, N, dim, radius, P);
        if (dim > 4 && dim <= kMaxPcaDim && e->grid_axes_mode != FRNN_GRID_AXES_LEADING) {
            st = plan_principal(e, d_points_soa, N, dim, radius, ok, P, &principal);
            if (st != FRNN_OK) return st;
            ok |= principal;
        }
        if (!ok) {
            path = FRNN_PATH_BRUTE;
        } else {
            stage_begin(e, ST_SCATTER);
            st = sort_into_cells(e, d_points_soa, P, principal ? e->proj_u.as<float>() : nullptr, e->counts,
                                 e->starts, e->cellrank, e->rows, e->ids, nullptr, &e->proj_s);
            if (st != FRNN_OK) return st;
            stage_end(e, ST_SCATTER);
            st = finish_search(e);
            if (st != FRNN_OK) return st;
        }
    }
    e->built.pts = d_points_soa;
    e->built.N = N;
    e->built.dim = dim;
    e->built.radius = radius;
    e->built.path = path;
    e->built.principal = principal;
    e->built.P = P;
    e->built.proj_delta = principal ? e->proj_delta : 0.0;
    e->built.valid = true;
    return FRNN_OK;
}

int frnn_query_grid(frnn_engine* e, const float* d_queries_soa, int M, int K, int** d_idxs, float** d_dists) {
    if (!e) return FRNN_ERR_INVALID_ARG;
    if (!e->built.valid)
        return fail(e, FRNN_ERR_STATE, "no grid: call frnn_build_grid first (any other search discards it)");
    if (K < 1 || K > kMaxK) return fail(e, FRNN_ERR_INVALID_ARG, "K must be in [1, 128]");
    if (!d_queries_soa || M < 1) return fail(e, FRNN_ERR_INVALID_ARG, "queries must be a device array of M >= 1 points");
    if (!d_idxs || !d_dists) return fail(e, FRNN_ERR_INVALID_ARG, "output pointers are null");
    DeviceGuard g(e->device);
    int st = check_device_ptr(e, d_queries_soa);
    if (st != FRNN_OK) return st;
    const auto b = e->built;
    if (b.path != FRNN_PATH_GRID) {
        // brute force keeps nothing between calls: search the kept points
        const int forced = e->forced_path;
        e->forced_path = b.path;
        st = search_queries_core(e, b.pts, b.N, d_queries_soa, M, b.dim, K, b.radius);
        e->forced_path = forced;
        e->built = b;  // the point set stays kept
        if (st != FRNN_OK) return st;
    } else {
        FRNN_GROW(e, e->out_idx, (size_t)M * K * 4);
        FRNN_GROW(e, e->out_dist, (size_t)M * K * 4);
        e->last_N = -1;
        e->last_part_rows = -1;
        e->last_overflow_map = 0;
        for (int i = 0; i < FRNN_STAGES; ++i) e->stage_used[i] = false;
        st = prepare_queries(e, d_queries_soa, M, b.dim, b.principal);
        if (st != FRNN_OK) return st;
        GridPlan Pq = b.P;
        if (b.principal) Pq.pre_r2 = screen_r2(b.radius, Pq.g, b.proj_delta + e->q_proj_delta);
        st = search_sorted_queries(e, d_queries_soa, M, K, b.radius * b.radius, Pq, b.principal,
                                   b.principal ? e->q_proj_u.as<float>() : nullptr, e->out_idx.as<int>(),
                                   e->out_dist.as<float>());
        if (st != FRNN_OK) return st;
        st = finish_search(e);
        if (st != FRNN_OK) return st;
        e->last_path = FRNN_PATH_GRID;
        e->last_principal = b.principal;
        e->last_g = b.P.g;
        e->last_cells = b.P.cells;
        e->last_N = M;
        e->last_K = K;
    }
    *d_idxs = e->out_idx.as<int>();
    *d_dists = e->out_dist.as<float>();
    return FRNN_OK;
}

int frnn_search_gpu_part(frnn_engine* e, const float* d_points_soa, int N, int dim, int K, float radius,
                         int part, int nparts, int* n_rows, int** d_row_ids, int** d_idxs,
                         float** d_dists) {
    int st = check_search_args(e, d_points_soa, N, dim, K, radius);
    if (st != FRNN_OK) return st;
    if (nparts < 1 || part < 0 || part >= nparts)
        return fail(e, FRNN_ERR_INVALID_ARG, "part must be in [0, nparts)");
    if (!n_rows || !d_row_ids || !d_idxs || !d_dists)
        return fail(e, FRNN_ERR_INVALID_ARG, "output pointers are null");
    DeviceGuard g(e->device);
    st = check_device_ptr(e, d_points_soa);
    if (st != FRNN_OK) return st;
    st = search_core(e, d_points_soa, N, dim, K, radius, true, part, nparts);
    if (st != FRNN_OK) return st;
    *n_rows = e->last_part_rows;
    *d_row_ids = e->part_ids.as<int>();
    *d_idxs = e->out_idx.as<int>();
    *d_dists = e->out_dist.as<float>();
    return FRNN_OK;
}

int frnn_search(frnn_engine* e, const float* h_points_aos, int64_t count, int K, float radius,
                int* h_idxs, float* h_dists) {
    if (!e) return FRNN_ERR_INVALID_ARG;
    if (!h_points_aos || !h_idxs || !h_dists) return fail(e, FRNN_ERR_INVALID_ARG, "null pointer");
    const int N = e->max_points;
    if (count <= 0 || count % N != 0)
        return fail(e, FRNN_ERR_INVALID_ARG, "point count must be a positive multiple of max_points");
    const int64_t dim64 = count / N;
    if (dim64 > kMaxD) return fail(e, FRNN_ERR_INVALID_ARG, "dim must be in [1, 128]");
    const int dim = (int)dim64;
    int st = check_search_args(e, h_points_aos, N, dim, K, radius);
    if (st != FRNN_OK) return st;
    DeviceGuard g(e->device);
    cudaStream_t s = e->stream;
    const size_t in_bytes = (size_t)count * 4;
    FRNN_GROW(e, e->in_stage, in_bytes);
    FRNN_GROW(e, e->in_soa, in_bytes);
    FRNN_CHECK(e, cudaMemcpyAsync(e->in_stage.p, h_points_aos, in_bytes, cudaMemcpyHostToDevice, s), "H2D points");
    FRNN_CHECK(e, launch_transpose(e->in_stage.p, e->in_soa.p, N, dim, s), "transpose points");
    e->launches++;
    st = search_core(e, e->in_soa.as<float>(), N, dim, K, radius, false);
    if (st != FRNN_OK) return st;
    const size_t out_n = (size_t)N * K;
    FRNN_GROW(e, e->out_rm_idx, out_n * 4);
    FRNN_GROW(e, e->out_rm_dist, out_n * 4);
    FRNN_CHECK(e, launch_transpose(e->out_idx.p, e->out_rm_idx.p, K, N, s), "transpose idx");
    FRNN_CHECK(e, launch_transpose(e->out_dist.p, e->out_rm_dist.p, K, N, s), "transpose dist");
    e->launches += 2;
    FRNN_CHECK(e, cudaMemcpyAsync(h_idxs, e->out_rm_idx.p, out_n * 4, cudaMemcpyDeviceToHost, s), "D2H idx");
    FRNN_CHECK(e, cudaMemcpyAsync(h_dists, e->out_rm_dist.p, out_n * 4, cudaMemcpyDeviceToHost, s), "D2H dist");
    FRNN_CHECK(e, cudaMemcpyAsync(e->h_err, e->err_flag.p, sizeof(int), cudaMemcpyDeviceToHost, s), "flag");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "search sync");
    if (*e->h_err != 0) {
        cudaMemsetAsync(e->err_flag.p, 0, sizeof(int), s);
        cudaStreamSynchronize(s);
        e->last_N = -1;
        return fail(e, FRNN_ERR_TIMEOUT, "a bounded device-side wait gave up");
    }
    return FRNN_OK;
}

int frnn_search_host_soa(frnn_engine* e, const float* h_points_soa, int N, int dim, int K,
                         float radius, int* h_idxs, float* h_dists) {
    int st = check_search_args(e, h_points_soa, N, dim, K, radius);
    if (st != FRNN_OK) return st;
    if (!h_idxs || !h_dists) return fail(e, FRNN_ERR_INVALID_ARG, "null output pointer");
    DeviceGuard g(e->device);
    cudaStream_t s = e->stream;
    const size_t in_bytes = (size_t)N * dim * 4;
    FRNN_GROW(e, e->in_soa, in_bytes);
    FRNN_CHECK(e, cudaMemcpyAsync(e->in_soa.p, h_points_soa, in_bytes, cudaMemcpyHostToDevice, s), "H2D points");
    st = search_core(e, e->in_soa.as<float>(), N, dim, K, radius, false);
    if (st != FRNN_OK) return st;
    const size_t out_n = (size_t)N * K;
    FRNN_CHECK(e, cudaMemcpyAsync(h_idxs, e->out_idx.p, out_n * 4, cudaMemcpyDeviceToHost, s), "D2H idx");
    FRNN_CHECK(e, cudaMemcpyAsync(h_dists, e->out_dist.p, out_n * 4, cudaMemcpyDeviceToHost, s), "D2H dist");
    FRNN_CHECK(e, cudaMemcpyAsync(e->h_err, e->err_flag.p, sizeof(int), cudaMemcpyDeviceToHost, s), "flag");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "search sync");
    if (*e->h_err != 0) {
        cudaMemsetAsync(e->err_flag.p, 0, sizeof(int), s);
        cudaStreamSynchronize(s);
        e->last_N = -1;
        return fail(e, FRNN_ERR_TIMEOUT, "a bounded device-side wait gave up");
    }
    return FRNN_OK;
}

int frnn_set_timing(frnn_engine* e, int enable) {
    if (!e) return FRNN_ERR_INVALID_ARG;
    DeviceGuard g(e->device);
    if (enable && !e->ev[0]) {
        for (cudaEvent_t& ev : e->ev)
            FRNN_CHECK(e, cudaEventCreate(&ev), "event create");
    }
    e->timing = enable != 0;
    return FRNN_OK;
}

int frnn_last_stage_times(frnn_engine* e, float* ms, int n) {
    if (!e || !ms || n <= 0) return FRNN_ERR_INVALID_ARG;
    DeviceGuard g(e->device);
    for (int i = 0; i < n; ++i) {
        ms[i] = -1.0f;
        if (i < FRNN_STAGES && e->timing && e->stage_used[i]) {
            FRNN_CHECK(e, cudaEventSynchronize(e->ev[2 * i + 1]), "event sync");
            FRNN_CHECK(e, cudaEventElapsedTime(&ms[i], e->ev[2 * i], e->ev[2 * i + 1]), "event time");
        }
    }
    return FRNN_OK;
}

int frnn_launch_count(const frnn_engine* e, int64_t* n) {
    if (!e || !n) return FRNN_ERR_INVALID_ARG;
    *n = e->launches;
    return FRNN_OK;
}

int frnn_last_overflow(frnn_engine* e, int* count, int* h_query_ids, int max_ids) {
    if (!e || !count) return FRNN_ERR_INVALID_ARG;
    if (max_ids < 0 || (max_ids > 0 && !h_query_ids))
        return fail(e, FRNN_ERR_INVALID_ARG, "max_ids must be >= 0 with a buffer for them");
    if (e->last_N < 0) return fail(e, FRNN_ERR_STATE, "no finished whole search to report on");
    *count = 0;
    if (e->last_overflow_map == 0) return FRNN_OK;
    DeviceGuard g(e->device);
    cudaStream_t s = e->stream;
    FRNN_CHECK(e, cudaMemcpyAsync(e->h_err + 1, e->n_overflow.p, sizeof(int), cudaMemcpyDeviceToHost, s),
               "overflow count readback");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "overflow count sync");
    *count = e->h_err[1];
    const int n = std::min(*count, max_ids);
    if (n > 0) {
        const int* map = e->last_overflow_map == 1 ? e->ids.as<int>()
                         : e->last_overflow_map == 3 ? e->q_ids.as<int>() : nullptr;
        FRNN_GROW(e, e->ovf_ids, (size_t)n * 4);
        overflow_ids_kernel<<<std::min((n + 255) / 256, 4 * e->sms), 256, 0, s>>>(
            e->overflow.as<int>(), e->n_overflow.as<int>(), map, n, e->ovf_ids.as<int>());
        FRNN_CHECK(e, cudaGetLastError(), "overflow ids launch");
        FRNN_CHECK(e, cudaMemcpyAsync(h_query_ids, e->ovf_ids.p, (size_t)n * 4, cudaMemcpyDeviceToHost, s),
                   "overflow ids readback");
        FRNN_CHECK(e, cudaStreamSynchronize(s), "overflow ids sync");
    }
    return FRNN_OK;
}

int frnn_get_results(frnn_engine* e, int N, int K, int* h_idxs, float* h_dists) {
    if (!e) return FRNN_ERR_INVALID_ARG;
    if (!h_idxs || !h_dists) return fail(e, FRNN_ERR_INVALID_ARG, "null output pointer");
    if (e->last_N < 0) return fail(e, FRNN_ERR_STATE, "no finished search to read");
    if (N != e->last_N || K < 1 || K > e->last_K)
        return fail(e, FRNN_ERR_INVALID_ARG, "N must equal the last search's N and K must not exceed its K");
    DeviceGuard g(e->device);
    cudaStream_t s = e->stream;
    const size_t n = (size_t)N * K;
    FRNN_CHECK(e, cudaMemcpyAsync(h_idxs, e->out_idx.p, n * 4, cudaMemcpyDeviceToHost, s), "D2H idx");
    FRNN_CHECK(e, cudaMemcpyAsync(h_dists, e->out_dist.p, n * 4, cudaMemcpyDeviceToHost, s), "D2H dist");
    FRNN_CHECK(e, cudaStreamSynchronize(s), "results sync");
    return FRNN_OK;
}

}  // extern "C"
