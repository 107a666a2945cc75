// grid_coop.cuh -- warp-cooperative neighbour search over the cell-sorted points.
//
// Replaces the reference's one-thread-per-query search kernels
// (frnn/csrc/grid/find_nbrs.cu: FindNbrsAoS3Kernel :400-491, FindNbrsNDKernel
// :116-214, FindNbrsGridDimKernel :243-353).  Same candidate set (the 3^G cell
// shell of the query's cell), same arithmetic, same acceptance rule; a
// different mapping onto the machine:
//
//   * a warp takes up to kGroup consecutive sorted queries that share a cell
//     (a "group"); every query of the group has the same candidate cells;
//   * the lanes walk the group's candidates 32 at a time (coalesced row loads,
//     each loaded once for the whole group); for every query of the group a
//     ballot finds the lanes whose candidate is accepted and a popc-prefix
//     appends them to that query's list in shared memory;
//   * a list that could overflow on the next chunk is compacted: a warp-wide
//     bitonic sort keeps its K smallest keys and the K-th becomes the
//     acceptance bound; the final emit is the same sort.
//
// There is no per-lane control flow on the candidate path, so the warp's lanes
// stay converged; per-query state lives in a few hundred bytes of shared
// memory per warp.
#pragma once

#include "frnn_device.cuh"

namespace frnn {
namespace coop {

constexpr int kWarps = 4;    // warps per block
constexpr int kGroup = 8;    // queries per group
// Queries per group of the principal-axis search (grid_prj.cuh).  Build-time
// launch-policy knob.
#ifndef FRNN_COOP_PRJ_GROUP
#define FRNN_COOP_PRJ_GROUP 8
#endif
constexpr int kGroupPrj = FRNN_COOP_PRJ_GROUP;
static_assert(kGroupPrj >= 1 && kGroupPrj <= 8, "group slots fit the 8-bit pair masks");

// Launch policy: minimum resident blocks per SM (which caps registers per
// thread) for the D = 3 kernel and for the wider-row kernels; build-time
// knobs like the reference's FRNN_GRID_*_MIN_BLOCKS cache variables
// (CMakeLists.txt:17-22); PRJ: the principal-axis search (grid_prj.cuh).
// Defaults measured on B200 (cfg1/cfg2 for D = 3, cfg3/cfg4 for the others).
#ifndef FRNN_COOP_D3_MIN_BLOCKS
#define FRNN_COOP_D3_MIN_BLOCKS 6
#endif
#ifndef FRNN_COOP_ND_MIN_BLOCKS
#define FRNN_COOP_ND_MIN_BLOCKS 4
#endif
#ifndef FRNN_COOP_PRJ_MIN_BLOCKS
#define FRNN_COOP_PRJ_MIN_BLOCKS 5
#endif

// List capacity for K: room for a whole chunk of acceptances (32) on top of K,
// rounded to the bitonic network sizes the warp sort handles.
__host__ __device__ constexpr int list_cap(int K) { return K <= 32 ? 64 : (K <= 96 ? 128 : 256); }

// Per-warp shared memory: the group's query rows, its 64-bit acceptance
// bounds, then the group's candidate lists.
template <int NV, bool D3, int GR = kGroup>
__host__ __device__ constexpr size_t rows_bytes() {
    return (size_t)GR * NV * 16 + (size_t)GR * 8;
}
template <int NV, bool D3, int GR = kGroup>
__host__ __device__ constexpr size_t warp_bytes(int K) {
    return rows_bytes<NV, D3, GR>() + (size_t)GR * list_cap(K) * 8;
}

// Warp-wide ascending bitonic sort of 32*E keys held E per lane; element p of
// the sequence is lane (p % 32), slot (p / 32).
template <int E>
__device__ __forceinline__ void warp_bitonic(unsigned long long (&v)[E], int lane) {
    constexpr int N = 32 * E;
#pragma unroll
    for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j >= 32) {
                const int je = j >> 5;
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const int f = e ^ je;
                    if (f > e) {
                        const int p = lane + 32 * e;
                        const bool up = (p & k) == 0;
                        const unsigned long long a = v[e], b = v[f];
                        const bool sw = up ? (a > b) : (a < b);
                        v[e] = sw ? b : a;
                        v[f] = sw ? a : b;
                    }
                }
            } else {
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const int p = lane + 32 * e;
                    const unsigned long long o = __shfl_xor_sync(0xffffffffu, v[e], j);
                    const bool up = (p & k) == 0;
                    const bool lower = (lane & j) == 0;
                    // the lower partner keeps the smaller key in an ascending block
                    const bool keep_min = (up == lower);
                    v[e] = keep_min ? (o < v[e] ? o : v[e]) : (o > v[e] ? o : v[e]);
                }
            }
        }
    }
}

// Sort list[0..n) (n <= 32*E) ascending into registers, padding with ~0.
template <int E>
__device__ __forceinline__ void load_sort(const unsigned long long* list, int n, int lane,
                                          unsigned long long (&v)[E]) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int p = lane + 32 * e;
        v[e] = p < n ? list[p] : ~0ull;
    }
    warp_bitonic<E>(v, lane);
}

// Keep the K smallest keys of list[0..n): written back sorted to list[0..K);
// returns the K-th smallest (the new acceptance bound).
template <int E>
__device__ __forceinline__ unsigned long long compact_sorted(unsigned long long* list, int n, int K,
                                                             int lane) {
    unsigned long long v[E];
    load_sort<E>(list, n, lane, v);
    __syncwarp();
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int p = lane + 32 * e;
        if (p < K) list[p] = v[e];
    }
    // element K-1 lives in lane (K-1)%32, slot (K-1)/32
    unsigned long long kth = 0;
#pragma unroll
    for (int e = 0; e < E; ++e)
        if (e == (K - 1) / 32) kth = v[e];
    __syncwarp();
    return __shfl_sync(0xffffffffu, kth, (K - 1) & 31);
}

template <int E>
__device__ __forceinline__ void emit_sorted(const unsigned long long* list, int n, int K, int lane,
                                            float r2, int* __restrict__ oidx,
                                            float* __restrict__ odist, long long ostride) {
    unsigned long long v[E];
    load_sort<E>(list, n, lane, v);
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int p = lane + 32 * e;
        if (p < K) {
            const bool real = p < n;
            oidx[p * ostride] = real ? key_idx(v[e]) : -1;
            odist[p * ostride] = real ? key_d2(v[e]) : r2;
        }
    }
}

// Emit for n <= 32 and K <= 32: lane i takes list entry i and counts the
// entries below it (keys are unique, so the counts are the ranks 0..n-1);
// about four instructions per entry instead of a 15-stage network.  The list
// may hold more than K entries (it is compacted only when it nears its
// capacity), so only ranks below K are written: output rows stop at K-1.
__device__ __forceinline__ void emit_rank32(const unsigned long long* list, int n, int K, int lane,
                                            float r2, int* __restrict__ oidx,
                                            float* __restrict__ odist, long long ostride) {
    const unsigned long long mine = lane < n ? list[lane] : ~0ull;
    int rank = 0;
    for (int j = 0; j < n; ++j) rank += list[j] < mine ? 1 : 0;
    if (lane < n) {
        if (rank < K) {
            oidx[rank * ostride] = key_idx(mine);
            odist[rank * ostride] = key_d2(mine);
        }
    } else if (lane < K) {
        oidx[lane * ostride] = -1;
        odist[lane * ostride] = r2;
    }
}

// Out of line (value and pointer arguments only) so the sort registers do not
// weigh on the candidate loop.  Called by all 32 lanes of a warp.
static __device__ __noinline__ unsigned long long compact_list(unsigned long long* list, int n,
                                                               int K) {
    const int lane = threadIdx.x & 31;
    if (n <= 64) return compact_sorted<2>(list, n, K, lane);
    if (n <= 128) return compact_sorted<4>(list, n, K, lane);
    return compact_sorted<8>(list, n, K, lane);
}

static __device__ __noinline__ void emit_list(const unsigned long long* list, int n, int K,
                                              float r2, int* oidx, float* odist,
                                              long long ostride) {
    const int lane = threadIdx.x & 31;
    const int m = n > K ? n : K;  // the network must also cover the K output slots
    if (m <= 32) emit_sorted<1>(list, n, K, lane, r2, oidx, odist, ostride);
    else if (m <= 64) emit_sorted<2>(list, n, K, lane, r2, oidx, odist, ostride);
    else if (m <= 128) emit_sorted<4>(list, n, K, lane, r2, oidx, odist, ostride);
    else emit_sorted<8>(list, n, K, lane, r2, oidx, odist, ostride);
}

// Canonical chain distance from a query row to a candidate row (D > 3).
template <int NV>
__device__ __forceinline__ float chain_dist2(const float4* __restrict__ qrow, const float4 (&p)[NV]) {
    float d2 = 0.0f;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
        const float4 qv = qrow[v];
        float df = qv.x - p[v].x;
        d2 = __fmaf_rn(df, df, d2);
        df = qv.y - p[v].y;
        d2 = __fmaf_rn(df, df, d2);
        df = qv.z - p[v].z;
        d2 = __fmaf_rn(df, df, d2);
        df = qv.w - p[v].w;
        d2 = __fmaf_rn(df, df, d2);
    }
    return d2;
}

template <int G>
struct Shell {
    static constexpr int rows = 3 * Shell<G - 1>::rows;
};
template <>
struct Shell<1> {
    static constexpr int rows = 1;
};

// NV float4 per sorted row; G grid axes (the leading coordinates); D3: rows
// are (x, y, z, index bits) and the index comes from .w, otherwise from
// ids[].  Grids on principal axes use grid_prj_kernel (grid_prj.cuh).
//
// Group state (query rows, bounds, list lengths) is warp-uniform and lives in
// registers of every lane; the group loop is unrolled over GR slots.
template <int NV, int G, bool D3, int GR = kGroup>
__global__ void __launch_bounds__(kWarps * 32, D3 ? FRNN_COOP_D3_MIN_BLOCKS : FRNN_COOP_ND_MIN_BLOCKS)
    grid_coop_kernel(const float4* __restrict__ rows, const int* __restrict__ ids,
                     const int* __restrict__ starts, GridPlan Pv, int K, float r2, int q0, int q1,
                     int* __restrict__ oidx, float* __restrict__ odist, long long ostride,
                     const int* __restrict__ scatter_ids, const int* __restrict__ qlist,
                     const int* __restrict__ qcount, long long row_base,
                     const float4* __restrict__ queries, const GridPlan* __restrict__ Pd) {
    // queries: the queries' rows (a separate query set in the same grid's
    // cell order, or the points' own).  Pd: the plan, when the GPU made it
    // (cells = 0: no grid, nothing to do)
    extern __shared__ __align__(16) unsigned char smem[];
    const GridPlan P = Pd ? *Pd : Pv;
    if (P.cells == 0) return;
    if (qcount) q1 = min(q1, q0 + __ldg(qcount));  // list length known only on the device
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cap = list_cap(K);
    unsigned char* wbase = smem + (size_t)warp * warp_bytes<NV, D3, GR>(K);
    float4* qrows = reinterpret_cast<float4*>(wbase);  // [GR][NV]
    unsigned long long* gthr =
        reinterpret_cast<unsigned long long*>(wbase + (size_t)GR * NV * 16);  // [GR]
    unsigned long long* lists = reinterpret_cast<unsigned long long*>(wbase + rows_bytes<NV, D3, GR>());

    const int base = q0 + (blockIdx.x * kWarps + warp) * 32;
    if (base >= q1) return;
    const int nq = min(32, q1 - base);
    const unsigned lt_mask = (1u << lane) - 1u;

    // this lane's query: row and cell
    float4 myq[NV];
    long long mycell = -1;
    int mygc[G];
    const long long mysq = lane < nq ? (qlist ? __ldg(&qlist[base + lane]) : base + lane) : 0;
#pragma unroll
    for (int v = 0; v < NV; ++v)
        myq[v] = lane < nq ? __ldg(&queries[mysq * NV + v]) : make_float4(0, 0, 0, 0);
    {
        // grid coordinates: the leading coordinates of the row
        long long c = 0;
#pragma unroll
        for (int a = 0; a < G; ++a) {
            const float4 f = myq[a >> 2];
            const float x = (a & 3) == 0 ? f.x : (a & 3) == 1 ? f.y : (a & 3) == 2 ? f.z : f.w;
            mygc[a] = cell_coord(x, P.origin[a], P.inv_cell, P.res[a]);
            c += (long long)mygc[a] * P.stride[a];
        }
        if (lane < nq) mycell = c;
    }

    constexpr int kRows = Shell<G>::rows;  // rows of the shell (axis 0 merged), 32 per pass
    int g0 = 0;
    while (g0 < nq) {
        // ---- the group: lanes g0.. with the same cell, at most GR -------
        const long long c0 = __shfl_sync(0xffffffffu, mycell, g0);
        const unsigned same = __ballot_sync(0xffffffffu, mycell == c0);
        const unsigned from = same >> g0;
        const int run = (~from == 0u) ? 32 - g0 : __ffs(~from) - 1;
        const int gq = min(run, GR);

        // group state: bounds and list lengths are warp-uniform registers;
        // query rows and the 64-bit bounds (read only on exact ties) are in
        // shared memory
        float glim[GR];
        int gcnt[GR];
#pragma unroll
        for (int g = 0; g < GR; ++g) {
            glim[g] = r2;
            gcnt[g] = 0;
        }
        {
            const int g = lane - g0;  // lanes g0..g0+gq-1 own the group's queries
            if (g >= 0 && g < gq) {
#pragma unroll
                for (int v = 0; v < NV; ++v) qrows[g * NV + v] = myq[v];
                gthr[g] = make_key(r2, 0);
            }
            __syncwarp();
        }
        int gc[G];
#pragma unroll
        for (int a = 0; a < G; ++a) gc[a] = __shfl_sync(0xffffffffu, mygc[a], g0);

        for (int sb = 0; sb < kRows; sb += 32) {
        // ---- candidate spans: one shell row per lane -----------------------
        int sstart = 0, slen = 0;
        if (sb + lane < kRows) {
            int t = sb + lane;
            long long rb = 0;
            bool ok = true;
#pragma unroll
            for (int a = 1; a < G; ++a) {
                const int c = gc[a] + (t % 3) - 1;
                t /= 3;
                ok &= (c >= 0) & (c < P.res[a]);
                rb += (long long)c * P.stride[a];
            }
            if (ok) {
                const int xlo = max(gc[0] - 1, 0), xhi = min(gc[0] + 1, P.res[0] - 1);
                // clamped to [0, n): a corrupt start table never reads out of bounds
                sstart = min(max(__ldg(&starts[rb + xlo]), 0), P.n);
                const int e = min(max(__ldg(&starts[rb + xhi + 1]), sstart), P.n);
                slen = e - sstart;
            }
        }
        int pre = slen;  // inclusive prefix over lanes
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, pre, o);
            if (lane >= o) pre += y;
        }
        const int total = __shfl_sync(0xffffffffu, pre, 31);
        const int excl = pre - slen;

        // ---- chunks of 32 candidates ---------------------------------------
        for (int t0 = 0; t0 < total; t0 += 32) {
            const int t = t0 + lane;
            const bool valid = t < total;
            // span of candidate t: number of lanes whose inclusive prefix <= t
            int k = 0;
#pragma unroll
            for (int s = 16; s > 0; s >>= 1) {
                const int v = __shfl_sync(0xffffffffu, pre, k + s - 1);
                if (v <= t) k += s;
            }
            const int js = __shfl_sync(0xffffffffu, sstart, k);
            const int je = __shfl_sync(0xffffffffu, excl, k);
            const int j = valid ? js + (t - je) : 0;
            float4 p[NV];
#pragma unroll
            for (int v = 0; v < NV; ++v)
                p[v] = valid ? __ldg(&rows[(long long)j * NV + v]) : make_float4(0, 0, 0, 0);
            const int pid = D3 ? __float_as_int(p[0].w) : (valid ? __ldg(&ids[j]) : 0);

#pragma unroll
            for (int g = 0; g < GR; ++g) {
                if (g < gq) {
                    float d2;
                    if constexpr (D3) {
                        const float4 qv = qrows[g];
                        d2 = dist2_d3(qv.x, qv.y, qv.z, p[0].x, p[0].y, p[0].z);
                    } else {
                        d2 = chain_dist2<NV>(qrows + g * NV, p);
                    }
                    const bool cand = valid;
                    bool acc = cand && d2 < glim[g];
                    const bool tie = cand && d2 == glim[g];
                    if (__any_sync(0xffffffffu, tie)) acc |= tie && make_key(d2, pid) < gthr[g];
                    const unsigned m = __ballot_sync(0xffffffffu, acc);
                    if (m) {
                        unsigned long long* list = lists + (size_t)g * cap;
                        if (acc) list[gcnt[g] + __popc(m & lt_mask)] = make_key(d2, pid);
                        gcnt[g] += __popc(m);
                        // keep room for a full chunk of acceptances: shrink to
                        // the K smallest and make the K-th the bound
                        if (gcnt[g] > cap - 32) {
                            __syncwarp();
                            const unsigned long long kth = compact_list(list, gcnt[g], K);
                            if (lane == 0) gthr[g] = kth;
                            glim[g] = key_d2(kth);
                            gcnt[g] = K;
                            __syncwarp();
                        }
                    }
                }
            }
        }
        }  // shell rows, 32 per pass
        __syncwarp();

        // ---- emit the group ------------------------------------------------
#pragma unroll
        for (int g = 0; g < GR; ++g) {
            if (g < gq) {
                const int n = gcnt[g];
                const int sq = qlist ? __ldg(&qlist[base + g0 + g]) : base + g0 + g;
                const long long orow =
                    (scatter_ids ? (long long)__ldg(&scatter_ids[sq]) : (long long)sq) - row_base;
                const unsigned long long* list = lists + (size_t)g * cap;
                // an output row outside [0, ostride) only comes from a
                // permutation left incomplete by a scan that gave up
                if ((unsigned long long)orow >= (unsigned long long)ostride) continue;
                if (n <= 32 && K <= 32) {
                    emit_rank32(list, n, K, lane, r2, oidx + orow, odist + orow, ostride);
                } else {
                    emit_list(list, n, K, r2, oidx + orow, odist + orow, ostride);
                }
            }
        }
        __syncwarp();
        g0 += gq;
    }
}

}  // namespace coop
}  // namespace frnn
