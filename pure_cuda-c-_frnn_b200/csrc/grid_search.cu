// grid_search.cu -- neighbour search over the cell-sorted points.
//
// Replaces the reference's search kernels (frnn/csrc/grid/find_nbrs.cu):
//   FindNbrsAoS3Kernel<CAP>   :400-491  -> grid_coop_kernel<1, 3, true>
//   FindNbrsNDKernel<CAP,DIM> :116-214  -> grid_coop_kernel<NV, G, false> (G = D <= 4)
//   FindNbrsGridDimKernel     :243-353  -> grid_coop_kernel<NV, 4, false> (D > 4: grid on
//                                          the first four coordinates, full-D ranking)
//                                          or grid_prj_kernel<NV, G> (D > 4: grid on
//                                          G principal axes, projected screening)
//   ScatterToOrigKernel       :505-523  -> unpermute_kernel
//
// Every query visits the 3^G cell shell around its own cell; because axis 0
// varies fastest in the dense cell index, the three axis-0 neighbours form one
// contiguous span, so a shell is 3^(G-1) spans.  The search itself is the
// warp-cooperative kernel of grid_coop.cuh, or on principal-axis grids the
// pair-queue kernel of grid_prj.cuh.
#include "frnn_device.cuh"
#include "frnn_internal.h"
#include "grid_coop.cuh"
#include "grid_prj.cuh"

namespace frnn {
namespace {

constexpr int kUnpermRows = 1;  // output rows per thread

__global__ void __launch_bounds__(256) unpermute_kernel(const int* __restrict__ in_idx,
                                                        const float* __restrict__ in_dist,
                                                        const int* __restrict__ ids, int n, int K,
                                                        int* __restrict__ out_idx,
                                                        float* __restrict__ out_dist,
                                                        const GridPlan* __restrict__ Pd) {
    // blockIdx.y = a slab of kUnpermRows output rows: blocks of one slab run
    // together, so the scattered writes stay inside an L2-resident region.
    const int sq = blockIdx.x * blockDim.x + threadIdx.x;
    if (sq >= n || (Pd && Pd->cells == 0)) return;
    const int o = __ldg(&ids[sq]);
    // a permutation entry outside [0, n) only exists after a scan gave up
    // (the search then reports FRNN_ERR_TIMEOUT); never write through it
    if ((unsigned)o >= (unsigned)n) return;
    const int k0 = blockIdx.y * kUnpermRows;
    int vi[kUnpermRows];
    float vd[kUnpermRows];
#pragma unroll
    for (int r = 0; r < kUnpermRows; ++r) {
        if (k0 + r < K) {
            vi[r] = __ldg(&in_idx[(long long)(k0 + r) * n + sq]);
            vd[r] = __ldg(&in_dist[(long long)(k0 + r) * n + sq]);
        }
    }
#pragma unroll
    for (int r = 0; r < kUnpermRows; ++r) {
        if (k0 + r < K) {
            out_idx[(long long)(k0 + r) * n + o] = vi[r];
            out_dist[(long long)(k0 + r) * n + o] = vd[r];
        }
    }
}

template <class Kern>
cudaError_t set_smem(Kern k, size_t smem) {
    if (smem <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

struct CoopArgs {
    const float* rows;
    const int* ids;
    const int* starts;
    GridPlan P;
    int K;
    float r2;
    int q0, q1;
    int* oidx;
    float* odist;
    long long ostride;
    const int* scatter_ids;
    const int* qlist;
    const int* qcount;
    long long row_base;
    const float* proj;
    const float* qrows;
    const float* qproj;
    const GridPlan* Pd;
};

template <int NV, int G, bool D3>
cudaError_t launch_coop(const CoopArgs& a, cudaStream_t s) {
    constexpr int GR = coop::kGroup;
    const size_t smem = (size_t)coop::kWarps * coop::warp_bytes<NV, D3, GR>(a.K);
    cudaError_t err = set_smem(coop::grid_coop_kernel<NV, G, D3, GR>, smem);
    if (err != cudaSuccess) return err;
    const int per_block = coop::kWarps * 32;
    const int blocks = (a.q1 - a.q0 + per_block - 1) / per_block;
    coop::grid_coop_kernel<NV, G, D3, GR><<<blocks, coop::kWarps * 32, smem, s>>>(
        reinterpret_cast<const float4*>(a.rows), a.ids, a.starts, a.P, a.K, a.r2, a.q0, a.q1, a.oidx,
        a.odist, a.ostride, a.scatter_ids, a.qlist, a.qcount, a.row_base,
        reinterpret_cast<const float4*>(a.qrows ? a.qrows : a.rows), a.Pd);
    return cudaGetLastError();
}

// Principal-axis grids: the pair-queue kernel (grid_prj.cuh).
template <int NV, int G>
cudaError_t launch_prj(const CoopArgs& a, cudaStream_t s) {
    constexpr int GR = coop::kGroupPrj;
    const size_t smem = (size_t)coop::kWarps * coop::prj_warp_bytes<NV, GR>(a.K);
    cudaError_t err = set_smem(coop::grid_prj_kernel<NV, G, GR>, smem);
    if (err != cudaSuccess) return err;
    const int per_block = coop::kWarps * 32;
    const int blocks = (a.q1 - a.q0 + per_block - 1) / per_block;
    coop::grid_prj_kernel<NV, G, GR><<<blocks, coop::kWarps * 32, smem, s>>>(
        reinterpret_cast<const float4*>(a.rows), a.ids, a.starts, a.P, a.K, a.r2, a.q0, a.q1, a.oidx,
        a.odist, a.ostride, a.scatter_ids, a.qlist, a.qcount, a.row_base,
        reinterpret_cast<const float4*>(a.proj), reinterpret_cast<const float4*>(a.qrows ? a.qrows : a.rows),
        reinterpret_cast<const float4*>(a.qrows ? a.qproj : a.proj));
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_grid_search(const float* rows, const int* ids, const int* starts,
                               const GridPlan& P, int K, float r2, int q0, int q1, int* oidx,
                               float* odist, long long ostride, const int* scatter_ids,
                               cudaStream_t s, const int* qlist, const int* qcount,
                               long long row_base, const float* proj, const float* qrows,
                               const float* qproj, const GridPlan* Pd) {
    if (q1 <= q0) return cudaSuccess;
    // a plan made on the GPU: leading-coordinate grids only (the kernel
    // template follows P.dim and P.g, which the host knows)
    if (Pd && proj) return cudaErrorInvalidValue;
    const CoopArgs a{rows, ids, starts, P, K, r2, q0, q1, oidx, odist, ostride, scatter_ids,
                     qlist, qcount, row_base >= 0 ? row_base : (scatter_ids ? 0LL : (long long)q0), proj, qrows,
                     qproj, Pd};
    if (P.dim == 3 && P.g == 3 && !proj) return launch_coop<1, 3, true>(a, s);
    // (row float4s, grid axes) pairs the planner produces: leading coordinates
    // G = min(D, 4); principal axes (D > 4) G in 2..6
    const int nv = P.row / 4;
    if (nv == 1 && !proj) {
        if (P.g == 1) return launch_coop<1, 1, false>(a, s);
        if (P.g == 2) return launch_coop<1, 2, false>(a, s);
        if (P.g == 4) return launch_coop<1, 4, false>(a, s);
        return cudaErrorInvalidValue;
    }
    // principal axes: candidates are screened on their projected coordinates
    // (P.pre_r2 > 0); leading coordinates: G = 4
#define FRNN_COOP_G(NV)                                                   \
    switch (P.g) {                                                        \
        case 2: return launch_prj<NV, 2>(a, s);                           \
        case 3: return launch_prj<NV, 3>(a, s);                           \
        case 4: return launch_prj<NV, 4>(a, s);                           \
        case 5: return launch_prj<NV, 5>(a, s);                           \
        case 6: return launch_prj<NV, 6>(a, s);                           \
        default: return cudaErrorInvalidValue;                            \
    }
    if (!proj) {
        if (P.g != 4) return cudaErrorInvalidValue;
        switch (nv) {
            case 2: return launch_coop<2, 4, false>(a, s);
            case 3: return launch_coop<3, 4, false>(a, s);
            case 4: return launch_coop<4, 4, false>(a, s);
            case 8: return launch_coop<8, 4, false>(a, s);
            default: return cudaErrorInvalidValue;
        }
    }
    if (!(P.pre_r2 > 0.0f)) return cudaErrorInvalidValue;
    switch (nv) {
        case 2: FRNN_COOP_G(2)
        case 3: FRNN_COOP_G(3)
        case 4: FRNN_COOP_G(4)
        case 8: FRNN_COOP_G(8)
        default: return cudaErrorInvalidValue;
    }
#undef FRNN_COOP_G
}

cudaError_t launch_unpermute(const int* in_idx, const float* in_dist, const int* ids, int n,
                             int K, int* out_idx, float* out_dist, cudaStream_t s, const GridPlan* Pd) {
    dim3 grid((n + 255) / 256, (K + kUnpermRows - 1) / kUnpermRows);
    unpermute_kernel<<<grid, 256, 0, s>>>(in_idx, in_dist, ids, n, K, out_idx, out_dist, Pd);
    return cudaGetLastError();
}

}  // namespace frnn
