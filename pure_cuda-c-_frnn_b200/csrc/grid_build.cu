// grid_build.cu -- bounding box, cell histogram, prefix scan, counting-sort
// scatter.  Replaces the reference's grid build (frnn/csrc/grid/insert_points.cu:
// CountPointsNDKernel :45-88, CountingSortNDKernel :142-164,
// CountingSortAoS3Kernel :205-226) and its Thrust exclusive scan
// (python_interface/frnn_engine.cu:91-94, :161-164, :233-236).
//
// Differences by design:
//   * the grid covers the data's bounding box, so no point is dropped;
//   * the histogram pass records each point's slot within its cell (the
//     atomicAdd return value), so the scatter needs no second atomic and the
//     cell starts stay intact for the search (the reference re-increments the
//     offsets and reads cell ends, find_nbrs.cu:190-191);
//   * the scan is a single-pass decoupled-lookback scan whose waits are bounded;
//   * sorted points are stored as rows (AoS, D rounded up to 4 floats, 16-byte
//     vector stores); for D = 3 the fourth float carries the original index.
#include <algorithm>

#include "frnn_device.cuh"
#include "frnn_internal.h"
#include "grid_plan.cuh"

namespace frnn {

// ---- bounding box of the grid axes ------------------------------------------

namespace {

constexpr int kBoxThreads = 256;
constexpr int kBoxAxes = 4;                     // leading coordinates boxed (g <= 4)
constexpr int kBoxSlots = 2 * kBoxAxes + 1;     // (min,max) per axis + non-finite flag

// Per-axis min/max of the grid axes, four grid-stride iterations' loads in
// flight per thread.  Each block writes a partial; the last block to finish
// (atomic ticket) folds the partials with all its threads into out[0..8]:
// out[2d] = min, out[2d+1] = max, out[8] = 1 if any coordinate is NaN or Inf.
// With plan_out, that block's thread 0 then plans the grid from the box
// (plan_grid, the host planner's own code) and writes it to *plan_out, so
// no host round trip separates the box from the build; a plan with cells = 0
// means "no grid" (non-finite data, or no useful grid) and every kernel given
// the plan then does nothing.
__global__ void __launch_bounds__(kBoxThreads) bbox_kernel(const float* __restrict__ pts, int n, int g,
                                                           float* __restrict__ partial,
                                                           unsigned int* __restrict__ ticket,
                                                           float* __restrict__ out,
                                                           GridPlan* __restrict__ plan_out, int dim,
                                                           float radius, long long max_cells) {
    float mn[kBoxAxes], mx[kBoxAxes];
    bool bad = false;
#pragma unroll
    for (int d = 0; d < kBoxAxes; ++d) { mn[d] = INFINITY; mx[d] = -INFINITY; }
    const int stride = gridDim.x * blockDim.x;
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n; i += 4 * stride) {
        float v[4][kBoxAxes];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int d = 0; d < kBoxAxes; ++d) v[u][d] = d < g ? __ldg(&pts[(long long)d * n + i + u * stride]) : 0.0f;
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int d = 0; d < kBoxAxes; ++d) {
                if (d < g) {
                    bad |= !isfinite(v[u][d]);
                    mn[d] = fminf(mn[d], v[u][d]);
                    mx[d] = fmaxf(mx[d], v[u][d]);
                }
            }
    }
    for (; i < n; i += stride) {
#pragma unroll
        for (int d = 0; d < kBoxAxes; ++d) {
            if (d < g) {
                float v = __ldg(&pts[(long long)d * n + i]);
                bad |= !isfinite(v);
                mn[d] = fminf(mn[d], v);
                mx[d] = fmaxf(mx[d], v);
            }
        }
    }
    __shared__ float sred[kBoxSlots][kBoxThreads / 32];
    __shared__ float sbox[kBoxSlots];
    __shared__ bool last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int d = 0; d < kBoxAxes; ++d) {
        float a = mn[d], b = mx[d];
        for (int o = 16; o > 0; o >>= 1) {
            a = fminf(a, __shfl_xor_sync(0xffffffffu, a, o));
            b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, o));
        }
        if (lane == 0) { sred[2 * d][warp] = a; sred[2 * d + 1][warp] = b; }
    }
    bool wbad = __any_sync(0xffffffffu, bad);
    if (lane == 0) sred[kBoxSlots - 1][warp] = wbad ? 1.0f : 0.0f;
    __syncthreads();
    if (threadIdx.x < kBoxSlots) {
        int t = threadIdx.x;
        bool is_max = (t & 1) || t == kBoxSlots - 1;
        float acc = sred[t][0];
        for (int w = 1; w < kBoxThreads / 32; ++w)
            acc = is_max ? fmaxf(acc, sred[t][w]) : fminf(acc, sred[t][w]);
        partial[(long long)blockIdx.x * kBoxSlots + t] = acc;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    // every thread folds a strided share of the partials (L2 loads, all in
    // flight together), then the block reduces the shares
    float acc[kBoxSlots];
#pragma unroll
    for (int t = 0; t < kBoxSlots; ++t) acc[t] = ((t & 1) || t == kBoxSlots - 1) ? -INFINITY : INFINITY;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
#pragma unroll
        for (int t = 0; t < kBoxSlots; ++t) {
            const float v = __ldcg(&partial[(long long)b * kBoxSlots + t]);
            acc[t] = ((t & 1) || t == kBoxSlots - 1) ? fmaxf(acc[t], v) : fminf(acc[t], v);
        }
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < kBoxSlots; ++t) {
        float a = acc[t];
        const bool is_max = (t & 1) || t == kBoxSlots - 1;
        for (int o = 16; o > 0; o >>= 1) {
            const float w = __shfl_xor_sync(0xffffffffu, a, o);
            a = is_max ? fmaxf(a, w) : fminf(a, w);
        }
        if (lane == 0) sred[t][warp] = a;
    }
    __syncthreads();
    if (threadIdx.x < kBoxSlots) {
        const int t = threadIdx.x;
        const bool is_max = (t & 1) || t == kBoxSlots - 1;
        float a = sred[t][0];
        for (int w = 1; w < kBoxThreads / 32; ++w) a = is_max ? fmaxf(a, sred[t][w]) : fminf(a, sred[t][w]);
        out[t] = a;
        sbox[t] = a;
    }
    if (threadIdx.x == 0) *ticket = 0u;  // ready for the next launch
    if (plan_out == nullptr) return;
    __syncthreads();
    if (threadIdx.x == 0) {
        GridPlan P{};
        const bool finite = sbox[kBoxSlots - 1] == 0.0f;
        if (!(finite && plan_grid(sbox, g, n, dim, radius, 0.0, max_cells, P))) {
            P = GridPlan{};
            P.g = g;
            P.n = n;
            P.dim = dim;
            P.cells = 0;
            // pre_r2 carries the reason for the host: 1 = non-finite data
            P.pre_r2 = finite ? 0.0f : 1.0f;
        }
        *plan_out = P;
    }
}

// ---- histogram: cell of each point and its slot within the cell ------------

// The grid axes are the leading coordinates of the SoA input, or, with proj,
// the projected coordinates proj[i*kProjStride + d] (principal axes).
__global__ void __launch_bounds__(256) hash_count_kernel(const float* __restrict__ pts, GridPlan Pv,
                                                         int* __restrict__ counts,
                                                         int2* __restrict__ cellrank,
                                                         const float* __restrict__ proj,
                                                         const GridPlan* __restrict__ Pd) {
    const GridPlan P = Pd ? *Pd : Pv;
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= P.n || P.cells == 0) return;
    long long c = 0;
#pragma unroll
    for (int d = 0; d < kMaxGridAxes; ++d) {
        if (d < P.g) {
            float v = proj ? __ldg(&proj[(long long)i * kProjStride + d]) : __ldg(&pts[(long long)d * P.n + i]);
            c += (long long)cell_coord(v, P.origin[d], P.inv_cell, P.res[d]) * P.stride[d];
        }
    }
    int cell = (int)c;
    int rank = atomicAdd(&counts[cell], 1);
    cellrank[i] = make_int2(cell, rank);
}

// ---- single-pass exclusive scan with decoupled look-back ----------------------

constexpr int kScanThreads = 256;
constexpr int kScanItems = 16;
constexpr int kScanTile = kScanThreads * kScanItems;

constexpr unsigned kFlagAgg = 1u, kFlagPrefix = 2u;

__device__ __forceinline__ unsigned long long pack_status(unsigned epoch, unsigned flag,
                                                          unsigned value) {
    return ((unsigned long long)((epoch << 2) | flag) << 32) | value;
}

// cells_dev (optional): the cell count of a plan written on the device (the
// launch then covers the largest table the plan may have; tiles past the
// plan's table return at once).
__global__ void __launch_bounds__(kScanThreads) scan_kernel(const int* __restrict__ counts,
                                                            int* __restrict__ starts,
                                                            long long cells,
                                                            unsigned long long* __restrict__ status,
                                                            int* __restrict__ ticket, unsigned epoch,
                                                            int* __restrict__ err, int withhold,
                                                            const long long* __restrict__ cells_dev) {
    // withhold >= 0 (a test of the bounded wait only): that tile never
    // publishes its status, so the tile after it must give up waiting
    __shared__ int s_tile;
    __shared__ int s_warp[kScanThreads / 32];
    __shared__ unsigned s_excl;
    if (cells_dev) cells = *cells_dev;
    if (threadIdx.x == 0) s_tile = atomicAdd(ticket, 1);
    __syncthreads();
    const int tile = s_tile;
    const long long base = (long long)tile * kScanTile;
    if (base >= cells) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long first = base + (long long)threadIdx.x * kScanItems;

    int v[kScanItems];
    if (first + kScanItems <= cells) {
        const int4* src = reinterpret_cast<const int4*>(counts + first);
#pragma unroll
        for (int j = 0; j < kScanItems / 4; ++j) {
            int4 t = __ldg(src + j);
            v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < kScanItems; ++j) v[j] = first + j < cells ? counts[first + j] : 0;
    }
    int tsum = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) tsum += v[j];

    // exclusive scan of thread sums inside the block
    int incl = tsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = lane < kScanThreads / 32 ? s_warp[lane] : 0;
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += y;
        }
        if (lane < kScanThreads / 32) s_warp[lane] = wi - w;  // exclusive warp offsets
        unsigned agg = (unsigned)__shfl_sync(0xffffffffu, wi, kScanThreads / 32 - 1);
        // publish this tile's aggregate, then look back for its prefix
        unsigned excl = 0;
        const bool publish = tile != withhold;
        if (tile == 0) {
            if (lane == 0 && publish) atomicExch(&status[0], pack_status(epoch, kFlagPrefix, agg));
        } else {
            if (lane == 0 && publish) atomicExch(&status[tile], pack_status(epoch, kFlagAgg, agg));
            long long look = tile - 1;
            int spins = 0;
            while (true) {
                long long idx = look - lane;
                unsigned long long s =
                    idx >= 0 ? atomicAdd(&status[idx], 0ull) : pack_status(epoch, kFlagPrefix, 0u);
                unsigned hi = (unsigned)(s >> 32);
                unsigned flag = (hi >> 2) == (epoch & 0x3fffffffu) ? (hi & 3u) : 0u;
                unsigned pmask = __ballot_sync(0xffffffffu, flag == kFlagPrefix);
                unsigned bad = __ballot_sync(0xffffffffu, flag == 0u);
                int firstp = pmask ? __ffs(pmask) - 1 : 32;
                unsigned need = firstp >= 31 ? 0xffffffffu : ((2u << firstp) - 1u);
                if (bad & need) {
                    // a test that withholds a tile's status waits briefly
                    if (++spins > (withhold >= 0 ? 4096 : (1 << 22))) {
                        if (lane == 0) atomicExch(err, 1);
                        break;
                    }
                    __nanosleep(32);
                    continue;
                }
                unsigned val = (lane <= firstp) ? (unsigned)(s & 0xffffffffu) : 0u;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) val += __shfl_xor_sync(0xffffffffu, val, o);
                excl += val;
                if (firstp < 32) break;
                look -= 32;
            }
            if (lane == 0 && publish) atomicExch(&status[tile], pack_status(epoch, kFlagPrefix, excl + agg));
        }
        if (lane == 0) s_excl = excl;
        if (lane == 0 && base + kScanTile >= cells) starts[cells] = (int)(excl + agg);
    }
    __syncthreads();
    int run = (int)s_excl + s_warp[warp] + (incl - tsum);
    if (first + kScanItems <= cells) {
        int4* dst = reinterpret_cast<int4*>(starts + first);
#pragma unroll
        for (int j = 0; j < kScanItems / 4; ++j) {
            int4 t;
            t.x = run; run += v[4 * j];
            t.y = run; run += v[4 * j + 1];
            t.z = run; run += v[4 * j + 2];
            t.w = run; run += v[4 * j + 3];
            dst[j] = t;
        }
    } else {
#pragma unroll
        for (int j = 0; j < kScanItems; ++j) {
            if (first + j < cells) starts[first + j] = run;
            run += v[j];
        }
    }
}

// ---- zeroed count table for a plan made on the device -------------------------

// counts[0, Pd->cells) = 0: the memset of the host-planned build, for a table
// whose size only the device knows.  Like that memset, it leaves the table in
// L2 for the histogram's atomics that follow.  zero0 / zero1 (optional): two
// more words to clear (the scan's ticket, the overflow count), so the
// device-planned search needs no separate memsets between its kernels.
__global__ void __launch_bounds__(256) clear_counts_kernel(int* __restrict__ counts,
                                                           const GridPlan* __restrict__ Pd,
                                                           int* __restrict__ zero0, int* __restrict__ zero1) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (zero0) *zero0 = 0;
        if (zero1) *zero1 = 0;
    }
    const long long cells = Pd->cells;
    const long long n4 = cells >> 2;
    const long long step = (long long)gridDim.x * blockDim.x;
    int4* c4 = reinterpret_cast<int4*>(counts);
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += step)
        c4[i] = make_int4(0, 0, 0, 0);
    if (blockIdx.x == 0 && threadIdx.x < (cells & 3)) counts[(n4 << 2) + threadIdx.x] = 0;
}

// ---- counting-sort scatter into cell order ------------------------------------

__global__ void __launch_bounds__(256) scatter_d3_kernel(const float* __restrict__ pts, int n,
                                                         const int2* __restrict__ cellrank,
                                                         const int* __restrict__ starts,
                                                         float4* __restrict__ rows,
                                                         int* __restrict__ ids,
                                                         int* __restrict__ inv,
                                                         const GridPlan* __restrict__ Pd) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || (Pd && Pd->cells == 0)) return;
    int2 cr = cellrank[i];
    int pos = __ldg(&starts[cr.x]) + cr.y;
    if (pos < 0 || pos >= n) return;  // only reachable if the scan gave up (error flag set)
    float x = __ldg(&pts[i]), y = __ldg(&pts[(long long)n + i]), z = __ldg(&pts[2LL * n + i]);
    rows[pos] = make_float4(x, y, z, __int_as_float(i));
    ids[pos] = i;
    if (inv) inv[i] = pos;
}

__global__ void __launch_bounds__(256) scatter_rows_kernel(const float* __restrict__ pts, int n,
                                                           int dim, int row,
                                                           const int2* __restrict__ cellrank,
                                                           const int* __restrict__ starts,
                                                           float* __restrict__ rows,
                                                           int* __restrict__ ids,
                                                           int* __restrict__ inv,
                                                           const float4* __restrict__ proj,
                                                           float4* __restrict__ proj_sorted,
                                                           const GridPlan* __restrict__ Pd) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || (Pd && Pd->cells == 0)) return;
    int2 cr = cellrank[i];
    long long pos = __ldg(&starts[cr.x]) + cr.y;
    if (pos < 0 || pos >= n) return;  // only reachable if the scan gave up (error flag set)
    if (proj) {
#pragma unroll
        for (int v = 0; v < kProjStride / 4; ++v)
            proj_sorted[pos * (kProjStride / 4) + v] = __ldg(&proj[(long long)i * (kProjStride / 4) + v]);
    }
    float4* dst = reinterpret_cast<float4*>(rows + pos * row);
    for (int d = 0; d < row; d += 4) {
        float4 t;
        t.x = d < dim ? __ldg(&pts[(long long)d * n + i]) : 0.0f;
        t.y = d + 1 < dim ? __ldg(&pts[(long long)(d + 1) * n + i]) : 0.0f;
        t.z = d + 2 < dim ? __ldg(&pts[(long long)(d + 2) * n + i]) : 0.0f;
        t.w = d + 3 < dim ? __ldg(&pts[(long long)(d + 3) * n + i]) : 0.0f;
        dst[d >> 2] = t;
    }
    ids[pos] = i;
    if (inv) inv[i] = (int)pos;
}

}  // namespace

// ---- launchers ----------------------------------------------------------------

cudaError_t launch_bbox(const float* pts, int n, int g, float* partial, unsigned int* ticket,
                        float* out, int blocks, cudaStream_t s, GridPlan* plan_out, int dim,
                        float radius, long long max_cells) {
    bbox_kernel<<<blocks, kBoxThreads, 0, s>>>(pts, n, g, partial, ticket, out, plan_out, dim, radius,
                                                max_cells);
    return cudaGetLastError();
}

int bbox_blocks(int n, int sms) {
    int b = (n + kBoxThreads * 4 - 1) / (kBoxThreads * 4);
    return b < 1 ? 1 : (b > 2 * sms ? 2 * sms : b);
}

cudaError_t launch_hash_count(const float* pts, const GridPlan& P, int* counts, int2* cellrank,
                              cudaStream_t s, const float* proj, const GridPlan* Pd) {
    hash_count_kernel<<<(P.n + 255) / 256, 256, 0, s>>>(pts, P, counts, cellrank, proj, Pd);
    return cudaGetLastError();
}

long long scan_tiles(long long cells) { return (cells + kScanTile - 1) / kScanTile; }

cudaError_t launch_scan(const int* counts, int* starts, long long cells,
                        unsigned long long* status, int* ticket, unsigned epoch, int* err,
                        cudaStream_t s, int withhold, const GridPlan* Pd) {
    long long tiles = scan_tiles(cells);
    scan_kernel<<<(unsigned)tiles, kScanThreads, 0, s>>>(counts, starts, cells, status, ticket,
                                                         epoch & 0x3fffffffu, err, withhold,
                                                         Pd ? &Pd->cells : nullptr);
    return cudaGetLastError();
}

cudaError_t launch_clear_counts(int* counts, long long max_cells, const GridPlan* Pd, int sms,
                                cudaStream_t s, int* zero0, int* zero1) {
    const long long want = (max_cells / 4 + 255) / 256;
    const int blocks = (int)std::max<long long>(1, std::min<long long>(want, 8LL * sms));
    clear_counts_kernel<<<blocks, 256, 0, s>>>(counts, Pd, zero0, zero1);
    return cudaGetLastError();
}

cudaError_t launch_scatter(const float* pts, const GridPlan& P, const int2* cellrank,
                           const int* starts, float* rows, int* ids, cudaStream_t s, int* inv,
                           const float* proj, float* proj_sorted, const GridPlan* Pd) {
    if (proj && P.dim == 3) return cudaErrorInvalidValue;  // principal axes are for D > 4
    if (P.dim == 3)
        scatter_d3_kernel<<<(P.n + 255) / 256, 256, 0, s>>>(pts, P.n, cellrank, starts,
                                                            reinterpret_cast<float4*>(rows), ids, inv, Pd);
    else
        scatter_rows_kernel<<<(P.n + 255) / 256, 256, 0, s>>>(
            pts, P.n, P.dim, P.row, cellrank, starts, rows, ids, inv,
            reinterpret_cast<const float4*>(proj), reinterpret_cast<float4*>(proj_sorted), Pd);
    return cudaGetLastError();
}

}  // namespace frnn
