// grid_search.cu -- neighbour search over the cell-sorted points.
//
// Replaces the reference's search kernels (frnn/csrc/grid/find_nbrs.cu):
//   FindNbrsAoS3Kernel<CAP>   :400-491  -> grid_search_d3_kernel
//   FindNbrsNDKernel<CAP,DIM> :116-214  -> grid_search_rows_kernel<NV,G> (G = D <= 4)
//   FindNbrsGridDimKernel     :243-353  -> grid_search_rows_kernel<NV,4> (D > 4: grid on
//                                          the first four coordinates, full-D ranking)
//   ScatterToOrigKernel       :505-523  -> unpermute_kernel
//
// Shared structure: one thread per query, queries taken in cell order (so the
// lanes of a warp mostly walk the same cells), each query visiting the 3^G
// cell shell around its own cell.  Because axis 0 varies fastest in the dense
// cell index, the three axis-0 neighbours form one contiguous span, so a query
// issues 3^(G-1) span reads instead of 3^G cell reads.  Cells and spans whose
// box lies beyond the current acceptance threshold are skipped (the
// reference's AABB prune, find_nbrs.cu:179-188, made conservative).
//
// K-selection lives in shared memory (TopK in frnn_device.cuh), one column per
// thread; the reference keeps its heap in local memory.
#include "frnn_device.cuh"
#include "frnn_internal.h"

namespace frnn {
namespace {

constexpr int kSearchThreads = 128;

__global__ void __launch_bounds__(kSearchThreads)
    grid_search_d3_kernel(const float4* __restrict__ rows, const int* __restrict__ starts, GridPlan P,
                          int K, float r2, int q0, int q1, int* __restrict__ oidx,
                          float* __restrict__ odist, long long ostride,
                          const int* __restrict__ scatter_ids) {
    extern __shared__ unsigned long long heap[];
    const int sq = q0 + blockIdx.x * blockDim.x + threadIdx.x;
    if (sq >= q1) return;
    TopK tk;
    tk.init(heap + threadIdx.x, blockDim.x, K, r2);

    const float4 q = __ldg(&rows[sq]);
    const float cs = P.cell, eps = P.eps;
    const int gx = cell_coord(q.x, P.origin[0], P.inv_cell, P.res[0]);
    const int gy = cell_coord(q.y, P.origin[1], P.inv_cell, P.res[1]);
    const int gz = cell_coord(q.z, P.origin[2], P.inv_cell, P.res[2]);

    for (int cz = max(gz - 1, 0); cz <= min(gz + 1, P.res[2] - 1); ++cz) {
        const float bz = axis_gap(q.z, cz, P.origin[2], cs, eps);
        if (bz * kPruneScale > tk.thr_d2()) continue;
        for (int cy = max(gy - 1, 0); cy <= min(gy + 1, P.res[1] - 1); ++cy) {
            const float byz = bz + axis_gap(q.y, cy, P.origin[1], cs, eps);
            if (byz * kPruneScale > tk.thr_d2()) continue;
            int xlo = max(gx - 1, 0), xhi = min(gx + 1, P.res[0] - 1);
            if (xlo < gx && (byz + axis_gap(q.x, xlo, P.origin[0], cs, eps)) * kPruneScale > tk.thr_d2())
                xlo = gx;
            if (xhi > gx && (byz + axis_gap(q.x, xhi, P.origin[0], cs, eps)) * kPruneScale > tk.thr_d2())
                xhi = gx;
            const long long rb = (long long)cz * P.stride[2] + (long long)cy * P.stride[1];
            // spans are clamped to [0, n) so a corrupt start table can never
            // turn into an out-of-bounds read
            const int s = min(max(__ldg(&starts[rb + xlo]), 0), P.n);
            const int e = min(max(__ldg(&starts[rb + xhi + 1]), s), P.n);
            for (int j = s; j < e; ++j) {
                const float4 p = __ldg(&rows[j]);
                const float d2 = dist2_d3(q.x, q.y, q.z, p.x, p.y, p.z);
                const unsigned long long key = make_key(d2, __float_as_int(p.w));
                if (key < tk.thr) tk.push(key);
            }
        }
    }
    const long long orow = scatter_ids ? (long long)__ldg(&scatter_ids[sq]) : (long long)(sq - q0);
    tk.emit(oidx + orow, odist + orow, ostride, r2);
}

template <int G>
struct Pow3 {
    static constexpr int value = 3 * Pow3<G - 1>::value;
};
template <>
struct Pow3<0> {
    static constexpr int value = 1;
};

template <int NV, int G>
__global__ void __launch_bounds__(kSearchThreads)
    grid_search_rows_kernel(const float4* __restrict__ rows, const int* __restrict__ ids,
                            const int* __restrict__ starts, GridPlan P, int K, float r2, int q0,
                            int q1, int* __restrict__ oidx, float* __restrict__ odist,
                            long long ostride, const int* __restrict__ scatter_ids) {
    extern __shared__ unsigned long long heap[];
    const int sq = q0 + blockIdx.x * blockDim.x + threadIdx.x;
    if (sq >= q1) return;
    TopK tk;
    tk.init(heap + threadIdx.x, blockDim.x, K, r2);

    float4 q[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) q[v] = __ldg(&rows[(long long)sq * NV + v]);
    float qc[G];
#pragma unroll
    for (int a = 0; a < G; ++a) {
        const float4& c = q[a >> 2];
        qc[a] = (a & 3) == 0 ? c.x : (a & 3) == 1 ? c.y : (a & 3) == 2 ? c.z : c.w;
    }
    int gc[G];
#pragma unroll
    for (int a = 0; a < G; ++a) gc[a] = cell_coord(qc[a], P.origin[a], P.inv_cell, P.res[a]);
    const float cs = P.cell, eps = P.eps;

    constexpr int kRows = Pow3<G - 1>::value;
    for (int r = 0; r < kRows; ++r) {
        int t = r;
        float b = 0.0f;
        long long rb = 0;
        bool ok = true;
#pragma unroll
        for (int a = 1; a < G; ++a) {
            const int c = gc[a] + (t % 3) - 1;
            t /= 3;
            ok &= (c >= 0) & (c < P.res[a]);
            b += axis_gap(qc[a], c, P.origin[a], cs, eps);
            rb += (long long)c * P.stride[a];
        }
        if (!ok || b * kPruneScale > tk.thr_d2()) continue;
        int xlo = max(gc[0] - 1, 0), xhi = min(gc[0] + 1, P.res[0] - 1);
        if (xlo < gc[0] && (b + axis_gap(qc[0], xlo, P.origin[0], cs, eps)) * kPruneScale > tk.thr_d2())
            xlo = gc[0];
        if (xhi > gc[0] && (b + axis_gap(qc[0], xhi, P.origin[0], cs, eps)) * kPruneScale > tk.thr_d2())
            xhi = gc[0];
        const int s = min(max(__ldg(&starts[rb + xlo]), 0), P.n);
        const int e = min(max(__ldg(&starts[rb + xhi + 1]), s), P.n);
        for (int j = s; j < e; ++j) {
            const float4* pr = rows + (long long)j * NV;
            const float lim = tk.thr_d2();
            float d2 = 0.0f;
            bool alive = true;
            // Chain prefixes never exceed the final value, so stopping once a
            // prefix passes the threshold is exact.  (Predicated rather than a
            // break so the loop unrolls and q[] stays in registers.)
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                if (alive) {
                    const float4 p = __ldg(pr + v);
                    float df = q[v].x - p.x;
                    d2 = __fmaf_rn(df, df, d2);
                    df = q[v].y - p.y;
                    d2 = __fmaf_rn(df, df, d2);
                    df = q[v].z - p.z;
                    d2 = __fmaf_rn(df, df, d2);
                    df = q[v].w - p.w;
                    d2 = __fmaf_rn(df, df, d2);
                    alive = d2 <= lim;
                }
            }
            if (!alive) continue;
            const unsigned long long key = make_key(d2, __ldg(&ids[j]));
            if (key < tk.thr) tk.push(key);
        }
    }
    const long long orow = scatter_ids ? (long long)__ldg(&scatter_ids[sq]) : (long long)(sq - q0);
    tk.emit(oidx + orow, odist + orow, ostride, r2);
}

__global__ void __launch_bounds__(256) unpermute_kernel(const int* __restrict__ in_idx,
                                                        const float* __restrict__ in_dist,
                                                        const int* __restrict__ ids, int n,
                                                        int* __restrict__ out_idx,
                                                        float* __restrict__ out_dist) {
    // blockIdx.y = output row k: blocks of one row run together, so the
    // scattered writes of a row stay inside one L2-resident slab.
    const int sq = blockIdx.x * blockDim.x + threadIdx.x;
    if (sq >= n) return;
    const long long k = blockIdx.y;
    const int o = __ldg(&ids[sq]);
    out_idx[k * n + o] = __ldg(&in_idx[k * n + sq]);
    out_dist[k * n + o] = __ldg(&in_dist[k * n + sq]);
}

template <class Kern>
cudaError_t set_smem(Kern k, size_t smem) {
    if (smem <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

template <int NV, int G>
cudaError_t launch_rows(const float* rows, const int* ids, const int* starts, const GridPlan& P,
                        int K, float r2, int q0, int q1, int* oidx, float* odist,
                        long long ostride, const int* scatter_ids, cudaStream_t s) {
    const size_t smem = (size_t)K * 8 * kSearchThreads;
    cudaError_t err = set_smem(grid_search_rows_kernel<NV, G>, smem);
    if (err != cudaSuccess) return err;
    const int blocks = (q1 - q0 + kSearchThreads - 1) / kSearchThreads;
    grid_search_rows_kernel<NV, G><<<blocks, kSearchThreads, smem, s>>>(
        reinterpret_cast<const float4*>(rows), ids, starts, P, K, r2, q0, q1, oidx, odist, ostride,
        scatter_ids);
    return cudaGetLastError();
}

template <int NV>
cudaError_t launch_rows_g(const float* rows, const int* ids, const int* starts,
                          const GridPlan& P, int K, float r2, int q0, int q1, int* oidx,
                          float* odist, long long ostride, const int* scatter_ids,
                          cudaStream_t s) {
    switch (P.g) {
        case 1: return launch_rows<NV, 1>(rows, ids, starts, P, K, r2, q0, q1, oidx, odist, ostride, scatter_ids, s);
        case 2: return launch_rows<NV, 2>(rows, ids, starts, P, K, r2, q0, q1, oidx, odist, ostride, scatter_ids, s);
        case 3: return launch_rows<NV, 3>(rows, ids, starts, P, K, r2, q0, q1, oidx, odist, ostride, scatter_ids, s);
        case 4: return launch_rows<NV, 4>(rows, ids, starts, P, K, r2, q0, q1, oidx, odist, ostride, scatter_ids, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_grid_search(const float* rows, const int* ids, const int* starts,
                               const GridPlan& P, int K, float r2, int q0, int q1, int* oidx,
                               float* odist, long long ostride, const int* scatter_ids,
                               cudaStream_t s) {
    if (q1 <= q0) return cudaSuccess;
    if (P.dim == 3 && P.g == 3) {
        const size_t smem = (size_t)K * 8 * kSearchThreads;
        cudaError_t err = set_smem(grid_search_d3_kernel, smem);
        if (err != cudaSuccess) return err;
        const int blocks = (q1 - q0 + kSearchThreads - 1) / kSearchThreads;
        grid_search_d3_kernel<<<blocks, kSearchThreads, smem, s>>>(
            reinterpret_cast<const float4*>(rows), starts, P, K, r2, q0, q1, oidx, odist, ostride,
            scatter_ids);
        return cudaGetLastError();
    }
    switch (P.row / 4) {
        case 1: return launch_rows_g<1>(rows, ids, starts, P, K, r2, q0, q1, oidx, odist, ostride, scatter_ids, s);
        case 2: return launch_rows_g<2>(rows, ids, starts, P, K, r2, q0, q1, oidx, odist, ostride, scatter_ids, s);
        case 3: return launch_rows_g<3>(rows, ids, starts, P, K, r2, q0, q1, oidx, odist, ostride, scatter_ids, s);
        case 4: return launch_rows_g<4>(rows, ids, starts, P, K, r2, q0, q1, oidx, odist, ostride, scatter_ids, s);
        case 8: return launch_rows_g<8>(rows, ids, starts, P, K, r2, q0, q1, oidx, odist, ostride, scatter_ids, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_unpermute(const int* in_idx, const float* in_dist, const int* ids, int n,
                             int K, int* out_idx, float* out_dist, cudaStream_t s) {
    dim3 grid((n + 255) / 256, K);
    unpermute_kernel<<<grid, 256, 0, s>>>(in_idx, in_dist, ids, n, out_idx, out_dist);
    return cudaGetLastError();
}

}  // namespace frnn
