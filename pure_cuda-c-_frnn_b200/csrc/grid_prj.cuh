// grid_prj.cuh -- neighbour search on principal-axis grids: projected
// screening of every (candidate, query) pair, exact distances only for the
// pairs that pass, gathered 32 at a time.
//
// Replaces, for grids on principal axes, the reference's
// FindNbrsGridDimKernel (frnn/csrc/grid/find_nbrs.cu:243-353): same candidate
// cells (the 3^G shell of the query's cell), same exact distance (the chain
// over all D coordinates), same acceptance rule (d2 < r2, the K smallest
// (d2, index) kept).  The mapping onto the machine:
//
//   * a warp takes up to GR consecutive sorted queries that share a cell (a
//     group) and walks the group's shell candidates 32 at a time, as the
//     cooperative kernel does (grid_coop.cuh);
//   * every candidate is screened against every group query on its projected
//     coordinates (packed fp32x2 arithmetic): projection onto orthonormal axes
//     never lengthens a distance, so a pair whose projected squared distance
//     exceeds P.pre_r2 (the radius widened by the projections' rounding
//     bound) cannot be within r;
//   * the pairs that pass go to a per-warp queue in shared memory; whenever
//     32 are queued, each lane takes one pair, loads the candidate's full row
//     and computes the exact chain distance.  The exact work is then done
//     once per passing pair instead of once per (candidate, group query)
//     whenever any lane of the chunk passes;
//   * the projected rows of the next chunk are loaded while the current chunk
//     is screened.
//
// Acceptances append (d2, index) keys to the query's list in shared memory
// (an atomic slot per append: the final K smallest do not depend on the
// order); a list that could overflow on the next pass keeps its K smallest
// and the K-th becomes the acceptance bound, as in the cooperative kernel.
#pragma once

#include "grid_coop.cuh"

namespace frnn {
namespace coop {

// Pairs a warp can hold: fewer than 32 wait between passes, and one chunk
// adds at most 32 * GR.
template <int GR>
__host__ __device__ constexpr int prj_pair_cap() {
    return 32 + 32 * GR;
}

// Per-warp shared memory: query rows [GR][NV] float4, projected query rows
// [GR][kProjStride/4] float4, 64-bit bounds [GR], float bounds [GR], list
// lengths [GR], the queue length (16 bytes), queued candidate positions
// [cap] int and group slots [cap] bytes, then the lists [GR][list_cap(K)].
template <int NV, int GR>
__host__ __device__ constexpr size_t prj_head_bytes() {
    return (size_t)GR * NV * 16 + (size_t)GR * kProjStride * 4 + (size_t)GR * 16 + 16 +
           (size_t)prj_pair_cap<GR>() * 5;
}
template <int NV, int GR>
__host__ __device__ constexpr size_t prj_warp_bytes(int K) {
    return (prj_head_bytes<NV, GR>() + 15) / 16 * 16 + (size_t)GR * list_cap(K) * 8;
}

// Projected squared distance over the first G coordinates of two projected
// rows, pairs of coordinates at a time (fp32x2: each lane rounds as a scalar
// operation would).
template <int G>
__device__ __forceinline__ float prj_dist2(const float4 (&q)[kProjStride / 4], const float4 (&p)[kProjStride / 4]) {
    float c[8] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w};
    float d[8] = {p[0].x, p[0].y, p[0].z, p[0].w, p[1].x, p[1].y, p[1].z, p[1].w};
    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
    for (int a = 0; a + 1 < G; a += 2) {
        asm("{\n\t.reg .b64 x, y, z, acc;\n\t"
            "mov.b64 x, {%2, %3};\n\t"
            "mov.b64 y, {%4, %5};\n\t"
            "sub.rn.f32x2 z, x, y;\n\t"
            "mov.b64 acc, {%0, %1};\n\t"
            "fma.rn.f32x2 acc, z, z, acc;\n\t"
            "mov.b64 {%0, %1}, acc;\n\t}"
            : "+f"(s0), "+f"(s1)
            : "f"(c[a]), "f"(c[a + 1]), "f"(d[a]), "f"(d[a + 1]));
    }
    if (G & 1) {
        const float df = c[G - 1] - d[G - 1];
        s0 = __fmaf_rn(df, df, s0);
    }
    return s0 + s1;
}

template <int NV, int G, int GR>
__global__ void __launch_bounds__(kWarps * 32, FRNN_COOP_PRJ_MIN_BLOCKS)
    grid_prj_kernel(const float4* __restrict__ rows, const int* __restrict__ ids,
                    const int* __restrict__ starts, GridPlan P, int K, float r2, int q0, int q1,
                    int* __restrict__ oidx, float* __restrict__ odist, long long ostride,
                    const int* __restrict__ scatter_ids, const int* __restrict__ qlist,
                    const int* __restrict__ qcount, long long row_base, const float4* __restrict__ proj,
                    const float4* __restrict__ queries, const float4* __restrict__ qproj) {
    static_assert(G >= 2 && G <= kMaxGridAxes && G <= kProjStride, "grid axes");
    static_assert(GR >= 1 && GR <= 8, "group slots fit the 8-bit pair masks");
    constexpr int PV = kProjStride / 4;
    constexpr int kPairs = prj_pair_cap<GR>();
    extern __shared__ __align__(16) unsigned char smem[];
    if (qcount) q1 = min(q1, q0 + __ldg(qcount));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cap = list_cap(K);
    unsigned char* wbase = smem + (size_t)warp * prj_warp_bytes<NV, GR>(K);
    float4* qrows = reinterpret_cast<float4*>(wbase);                              // [GR][NV]
    float4* qprj = qrows + GR * NV;                                                 // [GR][PV]
    unsigned long long* gthr = reinterpret_cast<unsigned long long*>(qprj + GR * PV);  // [GR]
    float* glim = reinterpret_cast<float*>(gthr + GR);                              // [GR]
    int* gcnt = reinterpret_cast<int*>(glim + GR);                                  // [GR]
    int* qn = gcnt + GR;                                                            // queue length
    int* pair_j = qn + 4;                                                           // [kPairs]
    unsigned char* pair_g = reinterpret_cast<unsigned char*>(pair_j + kPairs);      // [kPairs]
    unsigned long long* lists =
        reinterpret_cast<unsigned long long*>(wbase + (prj_head_bytes<NV, GR>() + 15) / 16 * 16);

    const int base = q0 + (blockIdx.x * kWarps + warp) * 32;
    if (base >= q1) return;
    const int nq = min(32, q1 - base);

    // this lane's query: row and cell (from its projected coordinates)
    float4 myq[NV];
    long long mycell = -1;
    int mygc[G];
    const long long mysq = lane < nq ? (qlist ? __ldg(&qlist[base + lane]) : base + lane) : 0;
#pragma unroll
    for (int v = 0; v < NV; ++v)
        myq[v] = lane < nq ? __ldg(&queries[mysq * NV + v]) : make_float4(0, 0, 0, 0);
    {
        long long c = 0;
#pragma unroll
        for (int a = 0; a < G; ++a) {
            const float4 f = __ldg(&qproj[mysq * PV + (a >> 2)]);
            const float x = (a & 3) == 0 ? f.x : (a & 3) == 1 ? f.y : (a & 3) == 2 ? f.z : f.w;
            mygc[a] = cell_coord(x, P.origin[a], P.inv_cell, P.res[a]);
            c += (long long)mygc[a] * P.stride[a];
        }
        if (lane < nq) mycell = c;
    }

    // Exact distances for the queued pairs [first, first + cnt) (cnt <= 32),
    // acceptances appended; lists near capacity are compacted.  All lanes.
    auto exact_pass = [&](int first, int cnt, int gq) {
        const bool has = lane < cnt;
        const int j = has ? pair_j[first + lane] : 0;
        const int g = has ? pair_g[first + lane] : 0;
        float4 p[NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) p[v] = has ? __ldg(&rows[(long long)j * NV + v]) : make_float4(0, 0, 0, 0);
        const int pid = has ? __ldg(&ids[j]) : 0;
        const float d2 = chain_dist2<NV>(qrows + g * NV, p);
        const float lim = glim[g];
        bool acc = has && d2 < lim;
        if (has && d2 == lim) acc = make_key(d2, pid) < gthr[g];
        if (acc) {
            const int slot = atomicAdd(&gcnt[g], 1);
            lists[(size_t)g * cap + slot] = make_key(d2, pid);
        }
        __syncwarp();
        // every list holds at most cap - 32 keys before a pass, so a pass
        // (at most 32 acceptances) never overflows it
        unsigned over = __ballot_sync(0xffffffffu, lane < gq && gcnt[lane < GR ? lane : 0] > cap - 32);
        while (over) {
            const int h = __ffs(over) - 1;
            over &= over - 1;
            const unsigned long long kth = compact_list(lists + (size_t)h * cap, gcnt[h], K);
            if (lane == 0) {
                gthr[h] = kth;
                glim[h] = key_d2(kth);
                gcnt[h] = K;
            }
            __syncwarp();
        }
    };

    constexpr int kRows = Shell<G>::rows;  // shell rows (axis 0 merged), 32 per pass
    int g0 = 0;
    while (g0 < nq) {
        // ---- the group: lanes g0.. with the same cell, at most GR -------
        const long long c0 = __shfl_sync(0xffffffffu, mycell, g0);
        const unsigned same = __ballot_sync(0xffffffffu, mycell == c0);
        const unsigned from = same >> g0;
        const int run = (~from == 0u) ? 32 - g0 : __ffs(~from) - 1;
        const int gq = min(run, GR);
        {
            const int g = lane - g0;  // lanes g0..g0+gq-1 own the group's queries
            if (g >= 0 && g < gq) {
#pragma unroll
                for (int v = 0; v < NV; ++v) qrows[g * NV + v] = myq[v];
#pragma unroll
                for (int v = 0; v < PV; ++v) qprj[g * PV + v] = __ldg(&qproj[mysq * PV + v]);
                gthr[g] = make_key(r2, 0);
                glim[g] = r2;
                gcnt[g] = 0;
            }
            if (lane == 0) *qn = 0;
            __syncwarp();
        }
        int gc[G];
#pragma unroll
        for (int a = 0; a < G; ++a) gc[a] = __shfl_sync(0xffffffffu, mygc[a], g0);

        for (int sb = 0; sb < kRows; sb += 32) {
            // ---- candidate spans: one shell row per lane -------------------
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
            // sorted position of candidate t (or -1 past the end)
            auto cand = [&](int t) {
                int k = 0;
#pragma unroll
                for (int s = 16; s > 0; s >>= 1) {
                    const int v = __shfl_sync(0xffffffffu, pre, k + s - 1);
                    if (v <= t) k += s;
                }
                const int js = __shfl_sync(0xffffffffu, sstart, k);
                const int je = __shfl_sync(0xffffffffu, excl, k);
                return t < total ? js + (t - je) : -1;
            };
            int jn = total > 0 ? cand(lane) : -1;
            float4 pn[PV];
#pragma unroll
            for (int v = 0; v < PV; ++v)
                pn[v] = jn >= 0 ? __ldg(&proj[(long long)jn * PV + v]) : make_float4(0, 0, 0, 0);

            // ---- chunks of 32 candidates -----------------------------------
            for (int t0 = 0; t0 < total; t0 += 32) {
                const int j = jn;
                float4 pp[PV];
#pragma unroll
                for (int v = 0; v < PV; ++v) pp[v] = pn[v];
                if (t0 + 32 < total) {
                    jn = cand(t0 + 32 + lane);
#pragma unroll
                    for (int v = 0; v < PV; ++v)
                        pn[v] = jn >= 0 ? __ldg(&proj[(long long)jn * PV + v]) : make_float4(0, 0, 0, 0);
                }
                unsigned near = 0u;
                if (j >= 0) {
#pragma unroll
                    for (int g = 0; g < GR; ++g) {
                        if (g < gq) {
                            float4 qv[PV];
#pragma unroll
                            for (int v = 0; v < PV; ++v) qv[v] = qprj[g * PV + v];
                            near |= (prj_dist2<G>(qv, pp) <= P.pre_r2 ? 1u : 0u) << g;
                        }
                    }
                }
                if (!__any_sync(0xffffffffu, near != 0u)) continue;
                if (near) {
                    int pos = atomicAdd(qn, __popc(near));
                    while (near) {
                        const int g = __ffs(near) - 1;
                        near &= near - 1;
                        pair_j[pos] = j;
                        pair_g[pos] = (unsigned char)g;
                        ++pos;
                    }
                }
                __syncwarp();
                int n = *reinterpret_cast<volatile int*>(qn);
                __syncwarp();
                while (n >= 32) {
                    n -= 32;
                    exact_pass(n, 32, gq);
                }
                if (lane == 0) *qn = n;
                __syncwarp();
            }
        }  // shell rows, 32 per pass
        {
            const int n = *reinterpret_cast<volatile int*>(qn);
            __syncwarp();
            if (n > 0) exact_pass(0, n, gq);
        }
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
