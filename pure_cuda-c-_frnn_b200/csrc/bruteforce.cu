// bruteforce.cu -- tiled all-pairs search on the SIMT pipes.
//
// Replaces the reference's TiledBruteforceNDKernel / TiledBruteforce16Kernel
// and their launcher (frnn/csrc/no_grid_frnn/no_grid_frnn.cu:121-326).  One
// thread per query; the block stages a tile of candidates in shared memory and
// every thread scans it.  Differences: the tile is stored dimension-major
// ([d][j]) so the cooperative load is a coalesced SoA read and every lane reads
// the same tile word at the same time (a broadcast); the query and the top-K
// state also live in shared memory, so the kernel has no local-memory arrays;
// distances use the engine's canonical arithmetic (frnn_device.cuh), so brute
// force and grid paths return identical results.
#include "frnn_device.cuh"
#include "frnn_internal.h"

namespace frnn {
namespace {

constexpr int kBfThreads = 128;
constexpr int kBfTileMax = 128;
constexpr size_t kSmemLimit = 227 * 1024;

template <bool D3, int KMAX>
__global__ void __launch_bounds__(kBfThreads)
    bruteforce_kernel(const float* __restrict__ pts, int n, int dim, int K, float r2, int q0, int q1,
                      int* __restrict__ oidx, float* __restrict__ odist, long long ostride,
                      int kBfTile, const int* __restrict__ qlist, int row_base,
                      const float* __restrict__ qpts, int qn) {
    extern __shared__ unsigned long long smem[];
    unsigned long long* heap = smem;                                    // (K+B) x T keys
    float* tile = reinterpret_cast<float*>(heap + (size_t)TopK<KMAX>::slots(K) * kBfThreads);  // dim x kBfTile
    float* qs = tile + (size_t)dim * kBfTile;                          // dim x T
    // slot q0 + i is query q0 + i, or query qlist[q0 + i] with its results at
    // row q - row_base
    const int slot = q0 + blockIdx.x * kBfThreads + threadIdx.x;
    const bool active = slot < q1;
    const int q = active && qlist ? __ldg(&qlist[slot]) : slot;
    TopK<KMAX> tk;
    tk.init(heap + threadIdx.x, kBfThreads, K, r2);
    for (int d = 0; d < dim; ++d)
        qs[d * kBfThreads + threadIdx.x] = active ? __ldg(&qpts[(long long)d * qn + q]) : 0.0f;
    float qx = 0.f, qy = 0.f, qz = 0.f;
    if (D3) { qx = qs[threadIdx.x]; qy = qs[kBfThreads + threadIdx.x]; qz = qs[2 * kBfThreads + threadIdx.x]; }

    for (int j0 = 0; j0 < n; j0 += kBfTile) {
        const int tn = min(kBfTile, n - j0);
        __syncthreads();
        for (int d = 0; d < dim; ++d)
            for (int j = threadIdx.x; j < tn; j += kBfThreads)
                tile[d * kBfTile + j] = __ldg(&pts[(long long)d * n + j0 + j]);
        __syncthreads();
        if (!active) continue;
        for (int j = 0; j < tn; ++j) {
            float d2;
            if (D3) {
                d2 = dist2_d3(qx, qy, qz, tile[j], tile[kBfTile + j], tile[2 * kBfTile + j]);
            } else {
                const float lim = tk.thr_d2();
                d2 = 0.0f;
                int d = 0;
                for (; d < dim; ++d) {
                    const float df = qs[d * kBfThreads + threadIdx.x] - tile[d * kBfTile + j];
                    d2 = __fmaf_rn(df, df, d2);
                    // monotone chain: an exceeded prefix rejects exactly
                    if ((d & 7) == 7 && d2 > lim) break;
                }
                if (d < dim) continue;
            }
            tk.offer(d2, j0 + j);
        }
    }
    if (active) {
        const long long orow = qlist ? q - row_base : q - q0;
        tk.emit(oidx + orow, odist + orow, ostride, r2);
    }
}

template <bool D3, int KMAX>
cudaError_t launch_bf(const float* pts, int n, int dim, int K, float r2, int q0, int q1, int* oidx,
                      float* odist, long long ostride, int tile, size_t smem, int blocks,
                      cudaStream_t s, const int* qlist, int row_base, const float* qpts, int qn) {
    cudaError_t err = cudaFuncSetAttribute(bruteforce_kernel<D3, KMAX>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    bruteforce_kernel<D3, KMAX><<<blocks, kBfThreads, smem, s>>>(pts, n, dim, K, r2, q0, q1, oidx,
                                                                 odist, ostride, tile, qlist, row_base, qpts ? qpts : pts, qpts ? qn : n);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_bruteforce(const float* pts, int n, int dim, int K, float r2, int q0, int q1,
                              int* oidx, float* odist, long long ostride, cudaStream_t s,
                              const int* qlist, int row_base, const float* qpts, int qn) {
    if (q1 <= q0) return cudaSuccess;
    const size_t fixed = (size_t)TopK<128>::slots(K) * 8 * kBfThreads + (size_t)dim * 4 * kBfThreads;
    if (fixed + (size_t)dim * 4 * 8 > kSmemLimit) return cudaErrorInvalidConfiguration;
    int tile = (int)((kSmemLimit - fixed) / ((size_t)dim * 4));
    tile = tile > kBfTileMax ? kBfTileMax : (tile / 8) * 8;
    const size_t smem = fixed + (size_t)dim * 4 * tile;
    const int blocks = (q1 - q0 + kBfThreads - 1) / kBfThreads;
    if (dim == 3) {
        if (K <= 16) return launch_bf<true, 16>(pts, n, dim, K, r2, q0, q1, oidx, odist, ostride, tile, smem, blocks, s, qlist, row_base, qpts, qn);
        if (K <= 32) return launch_bf<true, 32>(pts, n, dim, K, r2, q0, q1, oidx, odist, ostride, tile, smem, blocks, s, qlist, row_base, qpts, qn);
        if (K <= 64) return launch_bf<true, 64>(pts, n, dim, K, r2, q0, q1, oidx, odist, ostride, tile, smem, blocks, s, qlist, row_base, qpts, qn);
        return launch_bf<true, 128>(pts, n, dim, K, r2, q0, q1, oidx, odist, ostride, tile, smem, blocks, s, qlist, row_base, qpts, qn);
    }
    if (K <= 16) return launch_bf<false, 16>(pts, n, dim, K, r2, q0, q1, oidx, odist, ostride, tile, smem, blocks, s, qlist, row_base, qpts, qn);
    if (K <= 32) return launch_bf<false, 32>(pts, n, dim, K, r2, q0, q1, oidx, odist, ostride, tile, smem, blocks, s, qlist, row_base, qpts, qn);
    if (K <= 64) return launch_bf<false, 64>(pts, n, dim, K, r2, q0, q1, oidx, odist, ostride, tile, smem, blocks, s, qlist, row_base, qpts, qn);
    return launch_bf<false, 128>(pts, n, dim, K, r2, q0, q1, oidx, odist, ostride, tile, smem, blocks, s, qlist, row_base, qpts, qn);
}

}  // namespace frnn
