// frnn_oracle.cpp -- CPU restatement of the reference FRNN engine.
//
// TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
// engine in pure_cuda-c-_frnn_b200/csrc.  Only tests/, __graft_entry__.smoke()
// and bench.py's cpu_baseline leg load it; the engine never links or calls it.
//
// Reference: DebuRatnam/Pure_CUDA-C-_FRNN (paths below are relative to that
// project).  What is restated here:
//
//   * the dispatcher of FRNNEngine::search_gpu / search
//       python_interface/frnn_engine.cu:195-250 and :104-176, and the first-d
//       feasibility rule of run_firstd_search :64-86            -> oracle_ref_plan
//   * the cell hash (floorf((x-min)*inv_cell), points outside [0,res) dropped)
//       frnn/csrc/grid/insert_points.cu:45-88                   -> ref_cell_of
//   * the per-path squared-distance arithmetic:
//       D=3 grid  fma(dx,dx,fma(dy,dy,dz*dz))  find_nbrs.cu:474-477
//       ND / first-d grid  d2=fma(diff,diff,d2) in d order
//                                   find_nbrs.cu:193-199, :335-340
//       brute force (no_grid_frnn.cu:52-74): float4 groups when dim%4==0,
//                                   else the scalar d order     -> dist2_*
//   * the acceptance/selection rule: heap initialised to (r^2,-1), a candidate
//       enters only if d2 < current worst (strict), K smallest kept
//       find_nbrs.cu:77-97, :136-143, no_grid_frnn.cu:88-105
//   * padding idx=-1, dist=r^2 and the SoA output layout out[k*N+q]
//       find_nbrs.cu:206-213, no_grid_frnn.cu:170-176
//
// Deliberate, documented difference: the reference breaks ties at the K-th
// distance by visit order, which depends on atomicAdd slot order and is not
// reproducible.  This oracle ranks by the pair (d2, index) so the result is a
// deterministic function of the input; the K slots are returned in ascending
// (d2, index) order instead of heap order.
//
// Exact mode (oracle_search) is path independent: every point with fp32
// d2 < fl(r*r) is a candidate, whatever grid a GPU path would use.  The grid
// used here is only an accelerator built in double precision with a 1e-4*r
// safety margin, so it never drops a point whose fp32 d2 could be < r^2.
//
// Reference mode (oracle_ref_search) additionally reproduces the reference's
// domain rule: on grid paths, points whose cell lies outside [0,res) are not
// candidates and are not valid queries (the reference leaves their output
// slots undefined); the mask output marks them.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <vector>
#include <immintrin.h>
#include <omp.h>

namespace {

enum Order { ORDER_ENGINE = 0, ORDER_CHAIN = 1, ORDER_AOS3 = 2, ORDER_BF4 = 3 };
enum Path {
    PATH_BF_SMALL = 0,     // frnn_engine.cu:215-219 use_bf
    PATH_GRID_AOS3 = 1,    // frnn_engine.cu:237-240 (dim == 3)
    PATH_GRID_ND = 2,      // frnn_engine.cu:241-244
    PATH_FIRSTD = 3,       // frnn_engine.cu:225-226 -> run_firstd_search
    PATH_BF_FALLBACK = 4,  // frnn_engine.cu:227-229
};

// ---- squared distance in the reference's per-path orders --------------------

inline float dist2_chain(const float* q, const float* p, long long stride, int D) {
    // find_nbrs.cu:193-199 / :335-340: d2 = fma(diff, diff, d2), d = 0..D-1
    float d2 = 0.0f;
    for (int d = 0; d < D; ++d) {
        float diff = q[d] - p[(long long)d * stride];
        d2 = std::fmaf(diff, diff, d2);
    }
    return d2;
}

inline float dist2_aos3(const float* q, const float* p, long long stride) {
    // find_nbrs.cu:474-477: fma(dx, dx, fma(dy, dy, dz*dz))
    float dx = q[0] - p[0];
    float dy = q[1] - p[stride];
    float dz = q[2] - p[2 * stride];
    return std::fmaf(dx, dx, std::fmaf(dy, dy, dz * dz));
}

inline float dist2_bf4(const float* q, const float* p, long long stride, int D) {
    // no_grid_frnn.cu:56-66: d2 += dx*dx + dy*dy + dz*dz + dw*dw per float4,
    // with nvcc's default contraction of a*b+c into fma; the scalar branch
    // (dim % 4 != 0) is the chain order.
    if (D & 3) return dist2_chain(q, p, stride, D);
    float d2 = 0.0f;
    for (int v = 0; v < D; v += 4) {
        float dx = q[v] - p[(long long)v * stride];
        float dy = q[v + 1] - p[(long long)(v + 1) * stride];
        float dz = q[v + 2] - p[(long long)(v + 2) * stride];
        float dw = q[v + 3] - p[(long long)(v + 3) * stride];
        float t = dx * dx;
        t = std::fmaf(dy, dy, t);
        t = std::fmaf(dz, dz, t);
        t = std::fmaf(dw, dw, t);
        d2 = d2 + t;
    }
    return d2;
}

inline float dist2(int order, int D, const float* q, const float* p, long long stride) {
    switch (order) {
        case ORDER_AOS3: return dist2_aos3(q, p, stride);
        case ORDER_BF4: return dist2_bf4(q, p, stride, D);
        case ORDER_CHAIN: return dist2_chain(q, p, stride, D);
        default: return D == 3 ? dist2_aos3(q, p, stride) : dist2_chain(q, p, stride, D);
    }
}

// ---- K-selection: K smallest (d2, idx) pairs with d2 < r2 -------------------

struct Cand {
    float d2;
    int idx;
};
inline bool cand_less(const Cand& a, const Cand& b) {
    return a.d2 < b.d2 || (a.d2 == b.d2 && a.idx < b.idx);
}

void emit(std::vector<Cand>& c, int K, float r2, int N, int q, int* idx_out, float* dist_out) {
    int take = std::min<int>(K, (int)c.size());
    std::partial_sort(c.begin(), c.begin() + take, c.end(), cand_less);
    for (int k = 0; k < K; ++k) {
        long long o = (long long)k * N + q;
        if (k < take) {
            idx_out[o] = c[k].idx;
            dist_out[o] = c[k].d2;
        } else {
            idx_out[o] = -1;
            dist_out[o] = r2;
        }
    }
}

// ---- acceleration grid for the exact search (double precision, margin) ------

struct CpuGrid {
    int g = 0;                       // grid dims (first g coordinates)
    double lo[4], cell = 0.0, w = 0.0;
    long long res[4], stride[4];
    long long cells = 0;
    std::vector<int> start;          // cells + 1
    std::vector<int> order;          // sorted point ids
};

bool build_grid(const float* soa, int N, int D, float r, const unsigned char* include,
                CpuGrid& G) {
    // Window half-width: any point whose fp32 d2 < fl(r*r) has every
    // coordinate difference below r*(1+D*2^-23) < 1.0001*r.
    G.w = (double)r * 1.0001 + 1e-30;
    G.cell = G.w;
    int gmax = std::min(D, 3);
    for (int g = gmax; g >= 1; --g) {
        long long cells = 1;
        bool ok = true;
        for (int d = 0; d < g; ++d) {
            double mn = INFINITY, mx = -INFINITY;
            for (int i = 0; i < N; ++i) {
                if (include && !include[i]) continue;
                double v = soa[(long long)d * N + i];
                mn = std::min(mn, v);
                mx = std::max(mx, v);
            }
            if (!(mn <= mx)) { mn = 0; mx = 0; }
            G.lo[d] = mn;
            G.res[d] = (long long)std::floor((mx - mn) / G.cell) + 1;
            if (G.res[d] > (1LL << 24)) { ok = false; break; }
            cells *= G.res[d];
            if (cells > std::max<long long>(32LL * N, 1LL << 22)) { ok = false; break; }
        }
        if (!ok) continue;
        // A grid that is a single cell per axis buys nothing.
        bool useful = false;
        for (int d = 0; d < g; ++d) useful |= G.res[d] > 3;
        if (!useful) continue;
        G.g = g;
        G.cells = cells;
        long long s = 1;
        for (int d = 0; d < g; ++d) { G.stride[d] = s; s *= G.res[d]; }
        std::vector<int> cnt(cells + 1, 0);
        std::vector<long long> cid(N, -1);
        for (int i = 0; i < N; ++i) {
            if (include && !include[i]) continue;
            long long c = 0;
            for (int d = 0; d < g; ++d) {
                long long k = (long long)std::floor(((double)soa[(long long)d * N + i] - G.lo[d]) / G.cell);
                k = std::min(std::max(k, 0LL), G.res[d] - 1);
                c += k * G.stride[d];
            }
            cid[i] = c;
            cnt[c + 1]++;
        }
        for (long long c = 0; c < cells; ++c) cnt[c + 1] += cnt[c];
        G.start = cnt;
        G.order.assign(cnt[cells], 0);
        std::vector<int> fill(cnt.begin(), cnt.end() - 1);
        for (int i = 0; i < N; ++i)
            if (cid[i] >= 0) G.order[fill[cid[i]]++] = i;
        return true;
    }
    G.g = 0;
    return false;
}

// Visit every point that could be within the window of query coordinates q.
template <class F>
void grid_visit(const CpuGrid& G, const float* q, F&& f) {
    long long lo[4], hi[4];
    for (int d = 0; d < G.g; ++d) {
        lo[d] = (long long)std::floor(((double)q[d] - G.w - G.lo[d]) / G.cell);
        hi[d] = (long long)std::floor(((double)q[d] + G.w - G.lo[d]) / G.cell);
        lo[d] = std::max(lo[d], 0LL);
        hi[d] = std::min(hi[d], G.res[d] - 1);
        if (lo[d] > hi[d]) return;
    }
    long long c[4] = {0, 0, 0, 0};
    for (int d = 0; d < G.g; ++d) c[d] = lo[d];
    // The first grid axis is contiguous in the sorted order: one span per row.
    while (true) {
        long long base = 0;
        for (int d = 1; d < G.g; ++d) base += c[d] * G.stride[d];
        int s = G.start[base + lo[0]];
        int e = G.start[base + hi[0] + 1];
        for (int j = s; j < e; ++j) f(G.order[j]);
        int d = 1;
        for (; d < G.g; ++d) {
            if (++c[d] <= hi[d]) break;
            c[d] = lo[d];
        }
        if (d >= G.g) break;
    }
}

// Mean candidates per query that grid_visit would enumerate, over up to 64
// evenly spaced queries (an estimate used only to choose the accelerator).
double grid_candidates(const CpuGrid& G, const float* qsoa, long long qstride, const int* qids, int nq,
                       int D) {
    const int m = std::min(nq, 64);
    std::vector<float> q(D);
    double sum = 0.0;
    for (int t = 0; t < m; ++t) {
        const int qi = qids ? qids[(long long)t * nq / m] : (int)((long long)t * nq / m);
        for (int d = 0; d < D; ++d) q[d] = qsoa[(long long)d * qstride + qi];
        grid_visit(G, q.data(), [&](int) { sum += 1.0; });
    }
    return m ? sum / m : 0.0;
}

// Exhaustive chain-order search (d2 = fma(diff, diff, d2), d = 0..D-1) with
// AVX2: 4 queries x 16 points per step, each lane its own chain, so every d2
// is bit-identical to dist2_chain.  Points are visited in tiles of kTile so a
// tile stays in cache while all of a thread's queries pass over it.  Used
// for D > 3 when the leading-coordinate grid would enumerate most points.
void brute_chain_search(const float* soa, int N, int D, int K, float r2, const float* qsoa,
                        long long qstride, const int* qids, int nq, int threads, int* idx_out,
                        float* dist_out, int out_stride) {
    constexpr int kTile = 2048, kQB = 4, kChunk = 64;
    const int nchunks = (nq + kChunk - 1) / kChunk;
#pragma omp parallel for num_threads(threads) schedule(dynamic, 1)
    for (int ch = 0; ch < nchunks; ++ch) {
        const int t0 = ch * kChunk, t1 = std::min(nq, t0 + kChunk), nt = t1 - t0;
        std::vector<float> q((size_t)kChunk * D);
        for (int t = 0; t < nt; ++t) {
            const int qi = qids ? qids[t0 + t] : t0 + t;
            for (int d = 0; d < D; ++d) q[(size_t)t * D + d] = qsoa[(long long)d * qstride + qi];
        }
        std::vector<std::vector<Cand>> cand(nt);
        const __m256 vr2 = _mm256_set1_ps(r2);
        for (int j0 = 0; j0 < N; j0 += kTile) {
            const int j1 = std::min(N, j0 + kTile);
            const int jv = j0 + (j1 - j0) / 16 * 16;  // vector part [j0, jv)
            for (int b = 0; b < nt; b += kQB) {
                const int nb = std::min(kQB, nt - b);
                const float* qb[kQB];
                for (int u = 0; u < kQB; ++u) qb[u] = &q[(size_t)(b + std::min(u, nb - 1)) * D];
                for (int j = j0; j < jv; j += 16) {
                    __m256 a00 = _mm256_setzero_ps(), a01 = a00, a10 = a00, a11 = a00, a20 = a00, a21 = a00,
                           a30 = a00, a31 = a00;
                    const float* pj = soa + j;
                    for (int d = 0; d < D; ++d) {
                        const __m256 p0 = _mm256_loadu_ps(pj + (long long)d * N);
                        const __m256 p1 = _mm256_loadu_ps(pj + (long long)d * N + 8);
                        __m256 x = _mm256_set1_ps(qb[0][d]), t;
                        t = _mm256_sub_ps(x, p0); a00 = _mm256_fmadd_ps(t, t, a00);
                        t = _mm256_sub_ps(x, p1); a01 = _mm256_fmadd_ps(t, t, a01);
                        x = _mm256_set1_ps(qb[1][d]);
                        t = _mm256_sub_ps(x, p0); a10 = _mm256_fmadd_ps(t, t, a10);
                        t = _mm256_sub_ps(x, p1); a11 = _mm256_fmadd_ps(t, t, a11);
                        x = _mm256_set1_ps(qb[2][d]);
                        t = _mm256_sub_ps(x, p0); a20 = _mm256_fmadd_ps(t, t, a20);
                        t = _mm256_sub_ps(x, p1); a21 = _mm256_fmadd_ps(t, t, a21);
                        x = _mm256_set1_ps(qb[3][d]);
                        t = _mm256_sub_ps(x, p0); a30 = _mm256_fmadd_ps(t, t, a30);
                        t = _mm256_sub_ps(x, p1); a31 = _mm256_fmadd_ps(t, t, a31);
                    }
                    const __m256 acc[kQB][2] = {{a00, a01}, {a10, a11}, {a20, a21}, {a30, a31}};
                    for (int u = 0; u < nb; ++u)
                        for (int h = 0; h < 2; ++h) {
                            int m = _mm256_movemask_ps(_mm256_cmp_ps(acc[u][h], vr2, _CMP_LT_OQ));
                            if (!m) continue;
                            alignas(32) float v[8];
                            _mm256_store_ps(v, acc[u][h]);
                            for (; m; m &= m - 1) {
                                const int l = __builtin_ctz(m);
                                cand[b + u].push_back({v[l], j + 8 * h + l});
                            }
                        }
                }
                for (int u = 0; u < nb; ++u)
                    for (int j = jv; j < j1; ++j) {
                        const float d2 = dist2_chain(qb[u], soa + j, N, D);
                        if (d2 < r2) cand[b + u].push_back({d2, j});
                    }
            }
        }
        for (int t = 0; t < nt; ++t) emit(cand[t], K, r2, out_stride, t0 + t, idx_out, dist_out);
    }
}

// Core exact search over a query subset.  `include` (may be null) restricts the
// candidate set; `order` selects the distance arithmetic.
// Queries are read from qsoa (SoA, stride qstride): the points themselves
// (qsoa = soa, qstride = N) for a self-query, or a separate query set.
int search_core(const float* soa, int N, int D, int K, float r, int order,
                const int* qids, int nq, const unsigned char* include, int threads,
                int* idx_out, float* dist_out, int out_stride, long long* n_cand,
                const float* qsoa = nullptr, long long qstride = 0) {
    if (!qsoa) {
        qsoa = soa;
        qstride = N;
    }
    const float r2 = r * r;  // float r2 = radius * radius (find_nbrs.cu:550, :571)
    CpuGrid G;
    bool have_grid = build_grid(soa, N, D, r, include, G);
    long long total = 0;
    if (threads <= 0) threads = omp_get_max_threads();
    // D > 3 in the chain order over every point: the exhaustive SIMD search
    // when the grid (on at most 3 leading coordinates) would enumerate more
    // than 1/16 of the points per query (the SIMD loop is at least that much
    // faster per candidate).  Same candidates, same d2 bits, same ranking.
    const bool chain = order == ORDER_CHAIN || (order == ORDER_ENGINE && D != 3);
    if (chain && D > 3 && !include &&
        (!have_grid || grid_candidates(G, qsoa, qstride, qids, nq, D) * 16.0 > (double)N)) {
        brute_chain_search(soa, N, D, K, r2, qsoa, qstride, qids, nq, threads, idx_out, dist_out,
                           out_stride);
        if (n_cand) *n_cand = (long long)nq * N;
        return 0;
    }
#pragma omp parallel num_threads(threads) reduction(+ : total)
    {
        std::vector<float> q(D);
        std::vector<Cand> cand;
        cand.reserve(256);
#pragma omp for schedule(dynamic, 64)
        for (int t = 0; t < nq; ++t) {
            int qi = qids ? qids[t] : t;
            for (int d = 0; d < D; ++d) q[d] = qsoa[(long long)d * qstride + qi];
            cand.clear();
            auto consider = [&](int j) {
                ++total;
                float d2 = dist2(order, D, q.data(), soa + j, N);
                if (d2 < r2) cand.push_back({d2, j});
            };
            if (have_grid) {
                grid_visit(G, q.data(), consider);
            } else {
                for (int j = 0; j < N; ++j)
                    if (!include || include[j]) consider(j);
            }
            emit(cand, K, r2, out_stride, t, idx_out, dist_out);
        }
    }
    if (n_cand) *n_cand = total;
    return 0;
}

bool args_ok(const float* soa, int N, int D, int K, float r) {
    return soa && N > 0 && D >= 1 && D <= 128 && K >= 1 && K <= 128 && std::isfinite(r) && r > 0;
}

}  // namespace

extern "C" {

// Restatement of the reference dispatcher (frnn_engine.cu:195-250 with
// run_firstd_search :64-86).  Writes the path id, the grid dim used by the
// path (0 for brute force), the grid resolution and cell count.
int oracle_ref_plan(int N, int D, int K, float r, int* path, int* grid_dim, int* res_out,
                    long long* cells_out) {
    if (N <= 0 || D <= 0 || K <= 0 || !(r > 0)) return 1;
    int res = (int)std::ceil((1.0f - 0.0f) / r);           // frnn_engine.cu:207
    double total_d = std::pow((double)res, D);              // :210
    bool feasible = total_d <= 1000000.0;                   // :211
    long long total = feasible ? (long long)total_d : 0;    // :212
    const long long kBF = 2000000LL;                        // :215
    long long sel = std::max(1LL, (long long)(K + 7) / 8);
    long long db_dims = ((long long)N * D > kBF) ? (kBF + 1LL) : (long long)N * D;
    bool use_bf = (db_dims <= kBF / sel) && ((long long)N <= kBF / (db_dims * sel));
    long long shell = 1;
    for (int d = 0; d < D; ++d) shell = std::min(shell * 3, 1LL << 62);
    *grid_dim = 0; *res_out = res; *cells_out = total;
    if (use_bf) { *path = PATH_BF_SMALL; return 0; }
    if (res <= 1 || !feasible || shell >= total) {
        int g = (D > 4) ? 4 : std::min(D, 3);               // :65
        int gres = std::max(2, (int)std::ceil((1.0f - 0.0f) / r));  // :76-77
        double tc = std::pow((double)gres, g);              // :79
        long long gshell = 1;
        for (int d = 0; d < g; ++d) gshell *= 3;
        if (tc > 1000000.0 || gshell >= (long long)tc) {    // :80-86
            *path = PATH_BF_FALLBACK; *res_out = res; *cells_out = 0;
            return 0;
        }
        *path = PATH_FIRSTD; *grid_dim = g; *res_out = gres; *cells_out = (long long)tc;
        return 0;
    }
    *path = (D == 3) ? PATH_GRID_AOS3 : PATH_GRID_ND;
    *grid_dim = D;
    return 0;
}

// Exact search for every point as a query (self-query, the reference's only
// mode).  Output SoA idx_out/dist_out [k*N + q]; rows ascending by (d2, idx).
int oracle_search(const float* soa, int N, int D, int K, float r, int order, int threads,
                  int* idx_out, float* dist_out, long long* n_cand) {
    if (!args_ok(soa, N, D, K, r) || !idx_out || !dist_out) return 1;
    return search_core(soa, N, D, K, r, order, nullptr, N, nullptr, threads, idx_out,
                       dist_out, N, n_cand);
}

// Exact search for a subset of queries qids[0..nq) against all N points.
// Output SoA [k*nq + t] for query qids[t].
int oracle_search_subset(const float* soa, int N, int D, int K, float r, int order,
                         const int* qids, int nq, int threads, int* idx_out, float* dist_out,
                         long long* n_cand) {
    if (!args_ok(soa, N, D, K, r) || !qids || nq <= 0 || !idx_out || !dist_out) return 1;
    for (int t = 0; t < nq; ++t)
        if (qids[t] < 0 || qids[t] >= N) return 1;
    return search_core(soa, N, D, K, r, order, qids, nq, nullptr, threads, idx_out, dist_out,
                       nq, n_cand);
}

// Exact search for a separate query set (SoA qsoa[d*M + t], t < M) against the
// N points (no counterpart in the reference engine, which only self-queries).
// Output SoA [k*M + t].
int oracle_search_queries(const float* soa, int N, const float* qsoa, int M, int D, int K, float r,
                          int order, int threads, int* idx_out, float* dist_out, long long* n_cand) {
    if (!args_ok(soa, N, D, K, r) || !qsoa || M <= 0 || !idx_out || !dist_out) return 1;
    return search_core(soa, N, D, K, r, order, nullptr, M, nullptr, threads, idx_out, dist_out, M,
                       n_cand, qsoa, M);
}

// Reference mode: the path the reference dispatcher picks, with that path's
// distance order and domain rule (grid paths drop points whose reference cell
// lies outside [0,res); insert_points.cu:74-87).  valid_out[q] = 0 marks
// queries whose output the reference leaves undefined.
int oracle_ref_search(const float* soa, int N, int D, int K, float r, int threads, int* idx_out,
                      float* dist_out, unsigned char* valid_out, int* path_out) {
    if (!args_ok(soa, N, D, K, r) || !idx_out || !dist_out || !valid_out) return 1;
    int path, g, res;
    long long cells;
    oracle_ref_plan(N, D, K, r, &path, &g, &res, &cells);
    if (path_out) *path_out = path;
    int order = ORDER_CHAIN;
    if (path == PATH_GRID_AOS3) order = ORDER_AOS3;
    if (path == PATH_BF_SMALL || path == PATH_BF_FALLBACK) order = ORDER_BF4;
    std::vector<unsigned char> inc(N, 1);
    if (g > 0) {
        // insert_points.cu:64-87 with GridParams min=0, cell=r (frnn_engine.cu:201-208)
        const float inv_cell = 1.0f / r;
        for (int i = 0; i < N; ++i)
            for (int d = 0; d < g; ++d) {
                int gp = (int)std::floor((soa[(long long)d * N + i] - 0.0f) * inv_cell);
                if (gp < 0 || gp >= res) { inc[i] = 0; break; }
            }
    }
    for (int i = 0; i < N; ++i) valid_out[i] = inc[i];
    return search_core(soa, N, D, K, r, order, nullptr, N, g > 0 ? inc.data() : nullptr,
                       threads, idx_out, dist_out, N, nullptr);
}

// Float64 distances (the adjudicator used by the reference's own
// Tests/scripts/validate_correctness.py:118-126, computed directly as
// sum (q-p)^2 to avoid cancellation).  Writes d2 for the given (query, point)
// pairs.
int oracle_pair_d2_f64(const float* soa, int N, int D, const int* qi, const int* pj, long long n,
                       double* out) {
    if (!soa || N <= 0 || D <= 0 || !qi || !pj || !out) return 1;
    for (long long t = 0; t < n; ++t) {
        double s = 0.0;
        for (int d = 0; d < D; ++d) {
            double diff = (double)soa[(long long)d * N + qi[t]] - (double)soa[(long long)d * N + pj[t]];
            s += diff * diff;
        }
        out[t] = s;
    }
    return 0;
}

// fp32 distance of given pairs in a given order (for tie/boundary accounting).
int oracle_pair_d2_f32(const float* soa, int N, int D, int order, const int* qi, const int* pj,
                       long long n, float* out) {
    if (!soa || N <= 0 || D <= 0 || !qi || !pj || !out) return 1;
    std::vector<float> q(D);
    for (long long t = 0; t < n; ++t) {
        for (int d = 0; d < D; ++d) q[d] = soa[(long long)d * N + qi[t]];
        out[t] = dist2(order, D, q.data(), soa + pj[t], N);
    }
    return 0;
}

int oracle_max_threads(void) { return omp_get_max_threads(); }

}  // extern "C"
