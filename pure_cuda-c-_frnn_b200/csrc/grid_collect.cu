// grid_collect.cu -- the list search: a grid search as two kernels, collect
// then emit (K <= 32).
//
// Replaces, for D = 3, the reference's FindNbrsAoS3Kernel (find_nbrs.cu:400-491)
// and, for other dimensions, FindNbrsNDKernel (:116-214) and
// FindNbrsGridDimKernel (:243-353), each followed by ScatterToOrigKernel
// (:505-523).  Same candidates (the 3^g cell shell), same arithmetic, same
// acceptance rule (d2 < r2 strict, K smallest, ties to the smaller index); the
// work is split where the GPU wants it split:
//
//   collect  one thread per query in cell order (the lanes of a warp walk
//            neighbouring cells, so candidate rows come from L1): every
//            candidate with d2 < r2 is appended, as a 64-bit (d2, index) key,
//            to the query's own list in global memory.  No selection and no
//            sorting here, so the loop stays small and the kernel runs at high
//            occupancy.  The lists are in cell order (lists[sq*cap + j]): a
//            list fills whole 32-byte sectors as it grows, and the lists of a
//            warp's queries are neighbours in memory.  collect_d3_kernel is
//            the D = 3 form (float4 rows carrying the index);
//            collect_nd_kernel<NV, G> covers every other grid the planner
//            makes (NV float4 per row, G axes, leading or principal).
//   emit     one thread per query in ORIGINAL order (inv[] maps it to its cell
//            order position), so the K result rows are written coalesced and no
//            unpermute pass is needed.  Each thread keeps its K smallest keys in
//            registers, folding its list in 16 at a time (sort the batch, keep
//            the KN smallest of both with a half-cleaner, re-sort with a
//            bitonic merge).  No shuffles and no warp-wide serialisation.
//
// A query with more than `cap` in-radius candidates is listed as overflowing
// and searched again by the warp-cooperative kernel (grid_coop.cuh), which
// has no such limit.
#include "frnn_device.cuh"
#include "frnn_internal.h"

namespace frnn {
namespace {

// Appends the key (d, idx) to a list when ok, as a predicated store.  A list
// that overflows keeps overwriting its last slot: its query is searched again
// by the cooperative kernel, so the slot's content no longer matters.
__device__ __forceinline__ void append_if(bool ok, unsigned long long* list, int& n, int cap, float d, int idx) {
    unsigned long long* dst = list + min(n, cap - 1);
    const unsigned long long key = make_key(d, idx);
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %2, 0;\n\t@p st.global.u64 [%0], %1;\n\t}" ::"l"(dst),
        "l"(key), "r"((int)ok)
        : "memory");
    n += ok ? 1 : 0;
}

__global__ void __launch_bounds__(256)
    collect_d3_kernel(const float4* __restrict__ rows, const int* __restrict__ starts, GridPlan Pv,
                      float r2, int cap, unsigned long long* __restrict__ lists,
                      int* __restrict__ counts, int* __restrict__ overflow,
                      int* __restrict__ n_overflow, int q0, int q1,
                      const float4* __restrict__ qrows, const int* __restrict__ qlist,
                      const GridPlan* __restrict__ Pd) {
    // queries: the points themselves (qrows == rows) or a separate set in
    // the same grid's cell order; sorted positions [q0, q1), or qlist[q0..q1)
    // Pd: the plan, when the GPU made it (cells = 0: no grid, nothing to do)
    const GridPlan P = Pd ? *Pd : Pv;
    const int qi = q0 + blockIdx.x * blockDim.x + threadIdx.x;
    if (qi >= q1 || P.cells == 0) return;
    const int sq = qlist ? __ldg(&qlist[qi]) : qi;
    const float4 q = __ldg(&qrows[sq]);
    const float cs = P.cell, eps = P.eps;
    const int gx = cell_coord(q.x, P.origin[0], P.inv_cell, P.res[0]);
    const int gy = cell_coord(q.y, P.origin[1], P.inv_cell, P.res[1]);
    const int gz = cell_coord(q.z, P.origin[2], P.inv_cell, P.res[2]);
    unsigned long long* mine = lists + (long long)sq * cap;
    int n = 0;
    // every row's span bounds loaded before the first span is walked: the
    // 18 start-table loads of a query are in flight together
    int js[9], es[9];
#pragma unroll
    for (int rr = 0; rr < 9; ++rr) {
        const int cz = gz - 1 + rr / 3, cy = gy - 1 + rr % 3;
        js[rr] = 0;
        es[rr] = 0;
        if (cz < 0 || cz >= P.res[2] || cy < 0 || cy >= P.res[1]) continue;
        const float byz = axis_gap(q.z, cz, P.origin[2], cs, eps) + axis_gap(q.y, cy, P.origin[1], cs, eps);
        if (byz * kPruneScale > r2) continue;
        int xlo = max(gx - 1, 0), xhi = min(gx + 1, P.res[0] - 1);
        if (xlo < gx && (byz + axis_gap(q.x, xlo, P.origin[0], cs, eps)) * kPruneScale > r2) xlo = gx;
        if (xhi > gx && (byz + axis_gap(q.x, xhi, P.origin[0], cs, eps)) * kPruneScale > r2) xhi = gx;
        const long long rb = (long long)cz * P.stride[2] + (long long)cy * P.stride[1];
        js[rr] = __ldg(&starts[rb + xlo]);
        es[rr] = __ldg(&starts[rb + xhi + 1]);
    }
#pragma unroll
    for (int rr = 0; rr < 9; ++rr) {
        int j = min(max(js[rr], 0), P.n);
        const int e = min(max(es[rr], j), P.n);
        for (; j < e; j += kCollectRowPad) {
            float4 p[kCollectRowPad];
#pragma unroll
            for (int u = 0; u < kCollectRowPad; ++u) p[u] = __ldg(&rows[j + u]);
#pragma unroll
            for (int u = 0; u < kCollectRowPad; ++u) {
                const float d = dist2_d3(q.x, q.y, q.z, p[u].x, p[u].y, p[u].z);
                append_if(j + u < e && d < r2, mine, n, cap, d, __float_as_int(p[u].w));
            }
        }
    }
    counts[sq] = n;
    if (n > cap) overflow[atomicAdd(n_overflow, 1)] = sq;
}

// The same collect for D != 3: one thread per query over its 3^G shell
// (axis 0 merged into spans, 3^(G-1) spans), the canonical chain distance
// over NV float4 per row, the index from ids[] (loaded only for accepted
// candidates).  Grid coordinates are the row's leading coordinates, or the
// query's projected coordinates (qproj, kProjStride floats per point) on a
// principal-axis grid.  Spans whose cell box lies beyond the acceptance
// bound are skipped: on leading coordinates the gaps bound the full distance
// from below (bound r2); on principal axes they bound the computed projected
// distance, whose bound P.pre_r2 carries the projections' rounding slack.
template <int NV, int G>
__global__ void __launch_bounds__(256)
    collect_nd_kernel(const float4* __restrict__ rows, const int* __restrict__ ids,
                      const int* __restrict__ starts, GridPlan Pv, float r2, int cap,
                      unsigned long long* __restrict__ lists, int* __restrict__ counts,
                      int* __restrict__ overflow, int* __restrict__ n_overflow, int q0, int q1,
                      const float4* __restrict__ qrows, const float4* __restrict__ qproj,
                      const int* __restrict__ qlist, const GridPlan* __restrict__ Pd) {
    const GridPlan P = Pd ? *Pd : Pv;
    if (P.cells == 0) return;
    // the bound span gaps are tested against
    const float gap_r2 = qproj ? P.pre_r2 : r2;
    constexpr int W = NV == 1 ? 8 : (NV == 2 ? 4 : 2);  // rows in flight per pass
    static_assert(W <= kCollectRowPad, "passes read at most kCollectRowPad rows past a span");
    const int qi = q0 + blockIdx.x * blockDim.x + threadIdx.x;
    if (qi >= q1) return;
    const int sq = qlist ? __ldg(&qlist[qi]) : qi;
    float4 q[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) q[v] = __ldg(&qrows[(long long)sq * NV + v]);
    float y[G];
    int gc[G];
#pragma unroll
    for (int a = 0; a < G; ++a) {
        const float4 f = qproj ? __ldg(&qproj[(long long)sq * (kProjStride / 4) + (a >> 2)]) : q[a >> 2];
        y[a] = (a & 3) == 0 ? f.x : (a & 3) == 1 ? f.y : (a & 3) == 2 ? f.z : f.w;
        gc[a] = cell_coord(y[a], P.origin[a], P.inv_cell, P.res[a]);
    }
    unsigned long long* mine = lists + (long long)sq * cap;
    int n = 0;
    int spans = 1;
#pragma unroll
    for (int a = 1; a < G; ++a) spans *= 3;
    for (int t = 0; t < spans; ++t) {
        int u = t;
        long long rb = 0;
        float gap = 0.0f;
        bool ok = true;
#pragma unroll
        for (int a = 1; a < G; ++a) {
            const int c = gc[a] + (u % 3) - 1;
            u /= 3;
            ok &= (c >= 0) & (c < P.res[a]);
            gap += axis_gap(y[a], c, P.origin[a], P.cell, P.eps);
            rb += (long long)c * P.stride[a];
        }
        if (!ok || gap * kPruneScale > gap_r2) continue;
        int xlo = max(gc[0] - 1, 0), xhi = min(gc[0] + 1, P.res[0] - 1);
        if (xlo < gc[0] && (gap + axis_gap(y[0], xlo, P.origin[0], P.cell, P.eps)) * kPruneScale > gap_r2) xlo = gc[0];
        if (xhi > gc[0] && (gap + axis_gap(y[0], xhi, P.origin[0], P.cell, P.eps)) * kPruneScale > gap_r2) xhi = gc[0];
        // clamped to [0, n): a corrupt start table never reads out of bounds
        int j = min(max(__ldg(&starts[rb + xlo]), 0), P.n);
        const int e = min(max(__ldg(&starts[rb + xhi + 1]), j), P.n);
        for (; j < e; j += W) {
            float4 p[W][NV];
#pragma unroll
            for (int w = 0; w < W; ++w)
#pragma unroll
                for (int v = 0; v < NV; ++v) p[w][v] = __ldg(&rows[(long long)(j + w) * NV + v]);
#pragma unroll
            for (int w = 0; w < W; ++w) {
                float d = 0.0f;
#pragma unroll
                for (int v = 0; v < NV; ++v) {
                    float df = q[v].x - p[w][v].x;
                    d = __fmaf_rn(df, df, d);
                    df = q[v].y - p[w][v].y;
                    d = __fmaf_rn(df, df, d);
                    df = q[v].z - p[w][v].z;
                    d = __fmaf_rn(df, df, d);
                    df = q[v].w - p[w][v].w;
                    d = __fmaf_rn(df, df, d);
                }
                const bool acc = j + w < e && d < r2;
                const int idx = acc ? __ldg(&ids[j + w]) : 0;
                append_if(acc, mine, n, cap, d, idx);
            }
        }
    }
    counts[sq] = n;
    if (n > cap) overflow[atomicAdd(n_overflow, 1)] = sq;
}

// Ascending bitonic merge of a bitonic register array.
template <int N>
__device__ __forceinline__ void bitonic_merge(unsigned long long (&a)[N]) {
#pragma unroll
    for (int j = N >> 1; j > 0; j >>= 1) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int l = i ^ j;
            if (l > i) {
                const unsigned long long x = a[i], y = a[l];
                a[i] = x < y ? x : y;
                a[l] = x < y ? y : x;
            }
        }
    }
}

__device__ __forceinline__ void cas_key(unsigned long long& x, unsigned long long& y) {
    const unsigned long long u = x, v = y;
    x = u < v ? u : v;
    y = u < v ? v : u;
}

// Batcher's odd-even merge sort over a[LO, LO + N), N a power of two, unrolled
// at compile time: 63 compare-exchanges for 16 keys, against 80 for the
// bitonic network.  oe_merge merges the two sorted halves of a[LO, LO + N)
// by comparing elements R apart.
template <int S, int LO, int N, int R>
__device__ __forceinline__ void oe_merge(unsigned long long (&a)[S]) {
    constexpr int M = 2 * R;
    if constexpr (M < N) {
        oe_merge<S, LO, N, M>(a);
        oe_merge<S, LO + R, N, M>(a);
#pragma unroll
        for (int i = LO + R; i + R < LO + N; i += M) cas_key(a[i], a[i + R]);
    } else {
        cas_key(a[LO], a[LO + R]);
    }
}
template <int S, int LO, int N>
__device__ __forceinline__ void oe_sort(unsigned long long (&a)[S]) {
    if constexpr (N > 1) {
        oe_sort<S, LO, N / 2>(a);
        oe_sort<S, LO + N / 2, N / 2>(a);
        oe_merge<S, LO, N, 1>(a);
    }
}

// The KN smallest keys of list[0..cnt) ascending in registers, folded in
// batches of 16.  One sort-16 / merge-KN body for every batch keeps the
// kernel's code small enough for the instruction cache (a separate KN-wide
// first sort doubled it, and nearly every warp has a lane with more than KN
// keys, so every warp ran both bodies).  The first batch, the same loop
// iteration for every lane, fills the top keys directly instead of merging
// into an empty set (B200, cfg2: emit 0.284 ms against 0.316 with a merge on
// every batch and bitonic batch sorts).
template <int KN>
__device__ __forceinline__ void top_keys(const unsigned long long* list, int cnt,
                                         unsigned long long (&a)[KN]) {
#pragma unroll
    for (int i = 0; i < KN; ++i) a[i] = ~0ull;
    for (int base = 0; base < cnt; base += 16) {
        unsigned long long b[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) b[i] = base + i < cnt ? list[base + i] : ~0ull;
        oe_sort<16, 0, 16>(b);
        if (base == 0) {
#pragma unroll
            for (int i = 0; i < 16; ++i) a[i] = b[i];
            continue;
        }
        // a ascending, b ascending padded with ~0 to KN: min(a[i], b'[KN-1-i])
        // is bitonic and holds the KN smallest of both
#pragma unroll
        for (int i = KN - 16; i < KN; ++i) {
            const unsigned long long v = b[KN - 1 - i];
            a[i] = v < a[i] ? v : a[i];
        }
        bitonic_merge<KN>(a);
    }
}

constexpr int kEmitClasses = 10;  // 16-key batch counts 0..8 (lists up to 128), and overflow

// At most 102 registers (5 blocks of 128 threads per SM): the few spills this
// costs in the batch loop are cheaper than 4 blocks' latency hiding (B200,
// cfg2: 0.314 against 0.336 ms).
template <int KN>
__global__ void __launch_bounds__(128, 5)
    emit_lists_kernel(const unsigned long long* __restrict__ lists, const int* __restrict__ counts,
                      const int* __restrict__ map, int q0, int n, int K, int cap, float r2,
                      int* __restrict__ oidx, float* __restrict__ odist, int map_range,
                      const GridPlan* __restrict__ Pd) {
    if (Pd && Pd->cells == 0) return;  // a plan made on the GPU found no grid
    // output row q: sorted position map[q] (original order), or q0 + q (a
    // slice of the sorted order).  The block's 128 rows are dealt to its
    // threads by the number of 16-key batches their lists need, so a warp's
    // lanes do similar work (a warp runs as many batches as its longest
    // list); the stores stay within the block's 128 consecutive rows.
    __shared__ int hist[kEmitClasses + 1];
    __shared__ short order[128];
    const int t = threadIdx.x;
    const int q_own = blockIdx.x * 128 + t;
    int cls = 0, cnt_own = 0, sq_own = 0;
    if (q_own < n) {
        sq_own = map ? __ldg(&map[q_own]) : q0 + q_own;
        // a map entry outside [0, n) only exists after a scan gave up
        cnt_own = (unsigned)sq_own < (unsigned)(map ? map_range : q0 + n) ? __ldg(&counts[sq_own]) : 0;
        cls = cnt_own > cap ? 0 : min((cnt_own + 15) >> 4, kEmitClasses - 1);
    }
    if (t <= kEmitClasses) hist[t] = 0;
    __syncthreads();
    const int rank = atomicAdd(&hist[cls + 1], 1);
    __syncthreads();
    if (t == 0)
        for (int c = 1; c <= kEmitClasses; ++c) hist[c] += hist[c - 1];
    __syncthreads();
    order[hist[cls] + rank] = (short)t;
    __syncthreads();
    const int src = order[t];
    const int q = blockIdx.x * 128 + src;
    if (q >= n) return;
    const int sq = map ? __ldg(&map[q]) : q0 + q;
    if (map && (unsigned)sq >= (unsigned)map_range) return;  // only after a scan gave up
    const int cnt = __ldg(&counts[sq]);
    if (cnt > cap) return;  // searched by the overflow pass
    unsigned long long a[KN];
    top_keys<KN>(lists + (long long)sq * cap, cnt, a);
#pragma unroll
    for (int i = 0; i < KN; ++i) {
        if (i < K) {
            const bool real = i < cnt;
            oidx[(long long)i * n + q] = real ? key_idx(a[i]) : -1;
            odist[(long long)i * n + q] = real ? key_d2(a[i]) : r2;
        }
    }
}

}  // namespace

cudaError_t launch_collect_d3(const float* rows, const int* starts, const GridPlan& P, float r2,
                              int cap, unsigned long long* lists, int* counts, int* overflow,
                              int* n_overflow, int q0, int q1, cudaStream_t s, const float* qrows,
                              const int* qlist, const GridPlan* Pd) {
    if (q1 <= q0) return cudaSuccess;
    collect_d3_kernel<<<(q1 - q0 + 255) / 256, 256, 0, s>>>(
        reinterpret_cast<const float4*>(rows), starts, P, r2, cap, lists, counts, overflow, n_overflow,
        q0, q1, reinterpret_cast<const float4*>(qrows ? qrows : rows), qlist, Pd);
    return cudaGetLastError();
}

namespace {
template <int NV, int G>
cudaError_t launch_nd(const float* rows, const int* ids, const int* starts, const GridPlan& P, float r2,
                      int cap, unsigned long long* lists, int* counts, int* overflow, int* n_overflow, int q0,
                      int q1, cudaStream_t s, const float* qrows, const float* qproj, const int* qlist,
                      const GridPlan* Pd) {
    collect_nd_kernel<NV, G><<<(q1 - q0 + 255) / 256, 256, 0, s>>>(
        reinterpret_cast<const float4*>(rows), ids, starts, P, r2, cap, lists, counts, overflow, n_overflow,
        q0, q1, reinterpret_cast<const float4*>(qrows ? qrows : rows), reinterpret_cast<const float4*>(qproj),
        qlist, Pd);
    return cudaGetLastError();
}
}  // namespace

cudaError_t launch_collect_nd(const float* rows, const int* ids, const int* starts, const GridPlan& P,
                              float r2, int cap, unsigned long long* lists, int* counts, int* overflow,
                              int* n_overflow, int q0, int q1, cudaStream_t s, const float* qrows,
                              const float* qproj, const int* qlist, const GridPlan* Pd) {
    if (q1 <= q0) return cudaSuccess;
    if (qproj && !(P.pre_r2 > 0.0f)) return cudaErrorInvalidValue;  // a principal grid carries its bound
    const int nv = P.row / 4;
#define FRNN_ND(NV, G) return launch_nd<NV, G>(rows, ids, starts, P, r2, cap, lists, counts, overflow, \
                                                n_overflow, q0, q1, s, qrows, qproj, qlist, Pd)
    if (nv == 1 && !qproj) {
        if (P.g == 1) FRNN_ND(1, 1);
        if (P.g == 2) FRNN_ND(1, 2);
        if (P.g == 3) FRNN_ND(1, 3);
        if (P.g == 4) FRNN_ND(1, 4);
        return cudaErrorInvalidValue;
    }
#define FRNN_ND_G(NV)                      \
    switch (P.g) {                         \
        case 2: FRNN_ND(NV, 2);            \
        case 3: FRNN_ND(NV, 3);            \
        case 4: FRNN_ND(NV, 4);            \
        case 5: FRNN_ND(NV, 5);            \
        case 6: FRNN_ND(NV, 6);            \
        default: return cudaErrorInvalidValue; \
    }
    if (!qproj && P.g != 4) return cudaErrorInvalidValue;
    switch (nv) {
        case 2: FRNN_ND_G(2)
        case 3: FRNN_ND_G(3)
        case 4: FRNN_ND_G(4)
        case 8: FRNN_ND_G(8)
        default: return cudaErrorInvalidValue;
    }
#undef FRNN_ND_G
#undef FRNN_ND
}

cudaError_t launch_emit_lists(const unsigned long long* lists, const int* counts, const int* map,
                              int q0, int n, int K, int cap, float r2, int* oidx, float* odist,
                              cudaStream_t s, int map_range, const GridPlan* Pd) {
    if (K > 32) return cudaErrorInvalidValue;  // the register top-K holds at most 32 keys
    if (n <= 0) return cudaSuccess;
    if (map_range < 0) map_range = n;
    if (K <= 16)
        emit_lists_kernel<16><<<(n + 127) / 128, 128, 0, s>>>(lists, counts, map, q0, n, K, cap, r2,
                                                              oidx, odist, map_range, Pd);
    else
        emit_lists_kernel<32><<<(n + 127) / 128, 128, 0, s>>>(lists, counts, map, q0, n, K, cap, r2,
                                                              oidx, odist, map_range, Pd);
    return cudaGetLastError();
}

}  // namespace frnn
