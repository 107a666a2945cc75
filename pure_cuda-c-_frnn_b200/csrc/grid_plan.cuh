// grid_plan.cuh -- the grid planner shared by every entry point that builds a
// grid (the engine's searches and the allocation-free search).
//
// Replaces the fixed parameters of the reference's GridParams (grid.h:38-52:
// cell = r, res = ceil(1/r) over [0,1]) and its dense-cell cap
// (python_interface/frnn_engine.cu:35,209-212): the grid covers the bounding
// box of the grid axes, the cell edge sits just above r, and a grid that would
// exceed the cell budget is coarsened (never dropped).  Results do not depend
// on the plan: a coarser grid only scans more candidates.
#pragma once

#include <cmath>

#include "frnn_device.cuh"

namespace frnn {

// Floats per cell-sorted row: D = 3 rows carry (x, y, z, index bits); other D
// are padded to a multiple of 4 (to 32 for D in 17..32, one row per warp
// pass in the cooperative kernel).
__host__ __device__ inline int plan_row_floats(int dim) {
    if (dim == 3) return 4;
    int r = (dim + 3) / 4 * 4;
    if (r > 16 && r <= 32) r = 32;
    return r;
}

// Double products and sums rounded one at a time on the host and on the GPU
// alike: device code would otherwise fuse a*b+c into one FMA, and a plan made
// on the GPU (the bounding-box kernel's planner) must equal the host's.
__host__ __device__ inline double plan_mul(double a, double b) {
#ifdef __CUDA_ARCH__
    return __dmul_rn(a, b);
#else
    return a * b;
#endif
}
__host__ __device__ inline double plan_add(double a, double b) {
#ifdef __CUDA_ARCH__
    return __dadd_rn(a, b);
#else
    return a + b;
#endif
}

// Plan a grid on g axes whose bounding box is box[2d], box[2d+1] (d < g).
// `extra` is an absolute allowance added to the cell edge (the rounding bound
// of projected coordinates; 0 for the data's own coordinates).  At most
// `max_cells` dense cells.  Returns false when no useful grid exists (every
// axis would have at most 3 cells, so each query would scan nearly
// everything) or the budget cannot be met.
__host__ __device__ inline bool plan_grid(const float* box, int g, int N, int dim, float radius,
                                          double extra, long long max_cells, GridPlan& P) {
    double ext_max = 0.0, mag = 0.0;
    for (int d = 0; d < g; ++d) {
        const double lo = box[2 * d], hi = box[2 * d + 1];
        ext_max = fmax(ext_max, hi - lo);
        mag = fmax(mag, fmax(fabs(lo), fabs(hi)));
    }
    // Cell edge slightly above r: a point within r of the query then lies in
    // the query's 3^g shell despite float rounding of the cell assignment
    // (|error| of (x - origin) * inv_cell is a few ulps of the cell index).
    const double u = 1.0 / 16777216.0;
    const double slack = plan_mul(plan_mul(8.0, u), plan_add(ext_max / radius, 2.0));
    double cell = plan_add(plan_mul((double)radius, plan_add(1.0 + 1e-5, slack)), extra);
    long long res[kMaxGridAxes];
    long long cells = 1;
    for (int iter = 0; iter < 200; ++iter) {
        cells = 1;
        bool over = false;
        for (int d = 0; d < g; ++d) {
            const double ext = (double)box[2 * d + 1] - (double)box[2 * d];
            res[d] = (long long)floor(ext / cell) + 1;
            if (res[d] > (1LL << 30)) { over = true; break; }
            cells *= res[d];
            if (cells > max_cells) { over = true; break; }
        }
        if (!over) break;
        cell *= 1.25;  // coarser cells keep the 3^g shell exact, only the work grows
    }
    if (cells > max_cells) return false;
    bool useful = false;
    for (int d = 0; d < g; ++d) useful |= res[d] > 3;
    if (!useful) return false;
    P.g = g;
    P.n = N;
    P.dim = dim;
    P.row = plan_row_floats(dim);
    P.cell = (float)cell;
    P.inv_cell = 1.0f / P.cell;
    // Resolutions with the float cell the kernels use: the largest coordinate
    // must map inside the grid.
    long long s = 1;
    for (int d = 0; d < kMaxGridAxes; ++d) {
        if (d < g) {
            P.origin[d] = box[2 * d];
            const int c = (int)floor((double)((box[2 * d + 1] - P.origin[d]) * P.inv_cell));
            if (res[d] < (long long)c + 1) res[d] = (long long)c + 1;
            P.res[d] = (int)res[d];
            P.stride[d] = s;
            s *= res[d];
        } else {
            P.origin[d] = 0.0f;
            P.res[d] = 1;
            P.stride[d] = s;
        }
    }
    P.cells = s;
    if (P.cells > max_cells || P.cells > (1LL << 31) - 2) return false;
    P.eps = (float)(ldexp(1.0, -20) * (mag + ext_max)) + 1e-30f;
    return true;
}

}  // namespace frnn
