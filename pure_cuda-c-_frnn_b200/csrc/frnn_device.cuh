// frnn_device.cuh -- types and device helpers shared by the engine's kernels.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace frnn {

constexpr int kMaxK = 128;           // grid.h:59 MAX_K_CAPACITY
constexpr int kMaxD = 128;           // grid.h:60 MAX_DIM_SUPPORTED
// Grid axes: the leading coordinates (at most 4, as the reference's first-d
// grid) or the data's principal axes (at most 6).
constexpr int kMaxGridAxes = 6;
// Floats per point of projected (principal-axis) coordinates: 6 used, padded.
constexpr int kProjStride = 8;
// Largest D for which principal axes are computed (the grid path's limit).
constexpr int kMaxPcaDim = 32;

// Grid description computed on the host from the data's bounding box.
// Replaces the reference's GridParams (grid.h:38-52): per-axis resolution and
// origin instead of a fixed [0,1] domain, and axis 0 varying fastest in the
// dense cell index so the three x-neighbours of a cell are one contiguous span.
struct GridPlan {
    int g;                       // grid axes (leading coordinates, or principal axes)
    int n;                       // number of points
    int dim;                     // full dimension D
    int row;                     // floats per sorted row (D rounded up to 4)
    float origin[kMaxGridAxes];  // cell (0,...,0) lower corner
    float cell;                  // cell edge (>= radius, so a 3^g shell covers r)
    float inv_cell;
    float eps;                   // absolute slack added to cell boxes (rounding)
    int res[kMaxGridAxes];       // cells per axis
    long long stride[kMaxGridAxes];
    long long cells;             // product of res
    // principal-axis grids: a candidate whose computed projected squared
    // distance to the query exceeds pre_r2 is not within r (0 on grids of the
    // data's own coordinates)
    float pre_r2;
};

// 64-bit ranking key: non-negative float bits are order-preserving as an
// unsigned integer, so (d2, index) lexicographic order is key order.
__device__ __forceinline__ unsigned long long make_key(float d2, int idx) {
    return ((unsigned long long)__float_as_uint(d2) << 32) | (unsigned int)idx;
}
__device__ __forceinline__ float key_d2(unsigned long long k) {
    return __uint_as_float((unsigned int)(k >> 32));
}
__device__ __forceinline__ int key_idx(unsigned long long k) { return (int)(unsigned int)k; }

// Ascending bitonic sorting network over a register array; every index is a
// compile-time constant after unrolling, so the array stays in registers.
template <int N>
__device__ __forceinline__ void bitonic_sort(unsigned long long (&a)[N]) {
#pragma unroll
    for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
#pragma unroll
            for (int i = 0; i < N; ++i) {
                const int l = i ^ j;
                if (l > i) {
                    const unsigned long long x = a[i], y = a[l];
                    const bool swap = ((i & k) == 0) ? (x > y) : (x < y);
                    a[i] = swap ? y : x;
                    a[l] = swap ? x : y;
                }
            }
        }
    }
}

// Canonical squared distances.  D = 3: fma(dx,dx,fma(dy,dy,dz*dz)), the
// reference's D=3 grid order (find_nbrs.cu:474-477).  Other D: the chain
// d2 = fma(diff, diff, d2) over d = 0..D-1 (find_nbrs.cu:193-199, :335-340).
// The chain is monotone (each step adds a non-negative term and rounding is
// monotone), so a prefix is a lower bound of the final value: early exit on a
// prefix above the acceptance threshold never changes a result.
__device__ __forceinline__ float dist2_d3(float qx, float qy, float qz, float px, float py,
                                          float pz) {
    float dx = qx - px, dy = qy - py, dz = qz - pz;
    return __fmaf_rn(dx, dx, __fmaf_rn(dy, dy, __fmul_rn(dz, dz)));
}

// Max-heap helpers over one shared-memory column (element i at col[i*S]).
// Kept out of line: they run only for queries with more than K candidates in
// radius and at the final heapsort, and inlining them into the candidate loop
// would raise the register count of the whole kernel.
static __device__ __noinline__ void heap_sift_down(unsigned long long* col, int S, int i, int size) {
    const unsigned long long v = col[(long long)i * S];
    while (true) {
        int l = 2 * i + 1;
        if (l >= size) break;
        unsigned long long lv = col[(long long)l * S];
        const int r = l + 1;
        if (r < size) {
            const unsigned long long rv = col[(long long)r * S];
            if (rv > lv) { l = r; lv = rv; }
        }
        if (lv <= v) break;
        col[(long long)i * S] = lv;
        i = l;
    }
    col[(long long)i * S] = v;
}

static __device__ __noinline__ void heap_build(unsigned long long* col, int S, int size) {
    for (int i = size / 2 - 1; i >= 0; --i) heap_sift_down(col, S, i, size);
}

// Turn slots 0..n-1 (n > K) of a column into a max-heap of the K smallest keys
// in slots 0..K-1 and return its root.  Slots 0..K-1 are already a heap when
// `heaped` is set.  A free function with value arguments (no object address),
// so the caller's state stays in registers.
static __device__ __noinline__ unsigned long long heap_fold(unsigned long long* col, int S, int K,
                                                            int n, bool heaped) {
    if (!heaped) heap_build(col, S, K);
    unsigned long long root = col[0];
    for (int i = K; i < n; ++i) {
        const unsigned long long v = col[(long long)i * S];
        if (v < root) {
            col[0] = v;
            heap_sift_down(col, S, 0, K);
            root = col[0];
        }
    }
    return root;
}

// Per-thread K-selection state kept in shared memory, one column per thread
// ([slot][thread] layout: every lane addresses its own bank whatever the slot).
//
// Accepted candidates are appended to a list of capacity C = K + B (a single
// predicated store per candidate, so a warp whose lanes accept at different
// times pays almost nothing for it).  Only when the list is full is it
// compacted: the first K slots become a max-heap of the K smallest keys seen
// so far, the B extra slots are folded into it, and the heap root becomes the
// acceptance bound.  A candidate is accepted iff d2 < r2 and its key is below
// the bound: the reference's rule (heap initialised to (r2,-1), strict
// d2 < root, find_nbrs.cu:77-97, :136-143) with ties broken by the smaller
// index.
//
// KMAX is the compile-time capacity class (16, 32, 64 or 128, K <= KMAX).
// For KMAX <= 32 the final ordering is a bitonic network over registers that
// every lane executes in lockstep; above that it is an in-place heapsort.
template <int KMAX, int B = 16>
struct TopK {
    unsigned long long* col;  // &smem[threadIdx.x]
    int S;                    // column stride (= blockDim.x)
    int K;
    int n;                    // keys held (slots 0..n-1)
    bool heaped;              // slots 0..K-1 form a max-heap
    unsigned long long thr;   // acceptance bound (exclusive)
    float lim;                // key_d2(thr): candidates with d2 > lim are rejected

    static constexpr int kExtra = B;
    __host__ __device__ static constexpr int slots(int k) { return k + B; }

    __device__ __forceinline__ void init(unsigned long long* base, int stride, int k, float r2) {
        col = base;
        S = stride;
        K = k;
        n = 0;
        heaped = false;
        thr = make_key(r2, 0);  // d2 < r2  <=>  key(d2, idx) < key(r2, 0)
        lim = r2;
    }
    __device__ __forceinline__ float thr_d2() const { return lim; }
    __device__ __forceinline__ unsigned long long at(int i) const { return col[(long long)i * S]; }
    __device__ __forceinline__ void put(int i, unsigned long long v) { col[(long long)i * S] = v; }

    // Offer a candidate: cheap float test first, full key only near the bound.
    __device__ __forceinline__ void offer(float d2, int idx) {
        if (d2 <= lim) {
            const unsigned long long key = make_key(d2, idx);
            if (key < thr) {
                put(n, key);
                if (++n == K + B) compact();
            }
        }
    }

    // Reduce the list to the K smallest keys (as a max-heap) and tighten the
    // bound.  Runs only when the list is full and once at the end.
    __device__ __forceinline__ void compact() {
        if (n <= K) return;
        thr = heap_fold(col, S, K, n, heaped);
        heaped = true;
        n = K;
        lim = key_d2(thr);
    }

    // Write the K smallest keys ascending to out rows 0..min(n,K)-1 and pad
    // the remaining rows with (-1, r2).  Output element k goes to
    // idx[k*ostride], dist[k*ostride].
    __device__ __forceinline__ void emit(int* __restrict__ oidx, float* __restrict__ odist,
                                         long long ostride, float r2) {
        if (n > K) compact();
        if constexpr (KMAX <= 32) {
            unsigned long long a[KMAX];
#pragma unroll
            for (int i = 0; i < KMAX; ++i) a[i] = i < n ? at(i) : ~0ull;
            bitonic_sort<KMAX>(a);
#pragma unroll
            for (int i = 0; i < KMAX; ++i) {
                if (i < K) {
                    const bool real = i < n;
                    oidx[i * ostride] = real ? key_idx(a[i]) : -1;
                    odist[i * ostride] = real ? key_d2(a[i]) : r2;
                }
            }
        } else {
            if (!heaped && n > 1) heap_build(col, S, n);
            for (int k = K - 1; k >= n; --k) {
                oidx[k * ostride] = -1;
                odist[k * ostride] = r2;
            }
            for (int m = n - 1; m >= 0; --m) {
                const unsigned long long top = at(0);
                oidx[m * ostride] = key_idx(top);
                odist[m * ostride] = key_d2(top);
                if (m > 0) {
                    put(0, at(m));
                    heap_sift_down(col, S, 0, m);
                }
            }
        }
    }
};

// Ascending bitonic network over n = 2^m keys of one shared-memory column
// (element i at col[i*S]).  Lanes of a warp run it in lockstep; registers
// stay few because the keys live in shared memory.
__device__ __forceinline__ void smem_bitonic_sort(unsigned long long* col, int S, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
#pragma unroll 4
            for (int i = 0; i < n; ++i) {
                const int l = i ^ j;
                if (l > i) {
                    const unsigned long long a = col[(long long)i * S], b = col[(long long)l * S];
                    const bool swap = ((i & k) == 0) ? (a > b) : (a < b);
                    if (swap) {
                        col[(long long)i * S] = b;
                        col[(long long)l * S] = a;
                    }
                }
            }
        }
    }
}

// K-selection for the grid searches: one shared-memory column of 8-byte keys
// per thread ([slot][thread] layout), `slots` entries long (>= K + extra).
//
//   * accepted candidates are appended (one predicated store);
//   * the first time the list holds K keys, their maximum becomes the
//     acceptance bound (any K candidates bound the K-th smallest from above),
//     which cuts later acceptances at no heap cost;
//   * only when the list is full is it compacted to the K smallest keys
//     (max-heap in slots 0..K-1, bound = root);
//   * the final order is a bitonic network over the column.
//
// Acceptance: d2 < r2 and key(d2, idx) below the bound -- the reference's
// rule (heap initialised to (r2,-1), strict d2 < root, find_nbrs.cu:77-97,
// :136-143) with ties broken by the smaller index.
struct SelK {
    unsigned long long* col;  // &smem[threadIdx.x]
    int S;                    // column stride (= blockDim.x)
    int K;
    int cap;                  // list slots
    int n;                    // keys held
    bool heaped;              // slots 0..K-1 form a max-heap
    unsigned long long thr;   // acceptance bound (exclusive)
    float lim;                // key_d2(thr)

    __device__ __forceinline__ void init(unsigned long long* base, int stride, int k, int slots,
                                         float r2) {
        col = base;
        S = stride;
        K = k;
        cap = slots;
        n = 0;
        heaped = false;
        thr = make_key(r2, 0);  // d2 < r2  <=>  key(d2, idx) < key(r2, 0)
        lim = r2;
    }
    __device__ __forceinline__ float thr_d2() const { return lim; }
    __device__ __forceinline__ unsigned long long at(int i) const { return col[(long long)i * S]; }
    __device__ __forceinline__ void put(int i, unsigned long long v) { col[(long long)i * S] = v; }

    __device__ __forceinline__ void offer(float d2, int idx) {
        if (d2 <= lim) {
            const unsigned long long key = make_key(d2, idx);
            if (key < thr) {
                // cap > K always (selk_slots): the store below stays inside the list
                put(n, key);
                ++n;
                if (n == cap) {
                    compact();
                } else if (n == K && !heaped) {
                    unsigned long long m = 0;
                    for (int i = 0; i < K; ++i) m = max(m, at(i));
                    set_bound(m);  // any K candidates bound the K-th smallest from above
                }
            }
        }
    }
    __device__ __forceinline__ void set_bound(unsigned long long b) {
        if (b < thr) {
            thr = b;
            lim = key_d2(b);
        }
    }
    __device__ __forceinline__ void compact() {
        if (n <= K) return;
        set_bound(heap_fold(col, S, K, n, heaped));
        heaped = true;
        n = K;
    }

    // K smallest keys ascending to out rows 0..min(n,K)-1, (-1, r2) padding
    // after.  `net` is the network size: a power of two >= min(n, K) for
    // every lane of the warp (warp-uniform), <= cap.
    __device__ __forceinline__ void emit(int* __restrict__ oidx, float* __restrict__ odist,
                                         long long ostride, float r2, int net) {
        if (n > K) compact();
        for (int i = n; i < net; ++i) put(i, ~0ull);
        smem_bitonic_sort(col, S, net);
        for (int i = 0; i < K; ++i) {
            const bool real = i < n;
            const unsigned long long v = real ? at(i) : 0ull;
            oidx[i * ostride] = real ? key_idx(v) : -1;
            odist[i * ostride] = real ? key_d2(v) : r2;
        }
    }
};

// List slots for a K: K plus room for a burst of acceptances, and at least
// the power-of-two network size the final sort may use.
__host__ __device__ constexpr int selk_slots(int K) {
    int p = 2;
    while (p < K) p <<= 1;
    return K + 16 > p ? K + 16 : p;
}

// Network size for a warp's emit: the next power of two >= the largest
// min(n, K) among the warp's active lanes (at least 2).
__device__ __forceinline__ int warp_net_size(int m) {
    int v = m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(__activemask(), v, o));
    int p = 2;
    while (p < v) p <<= 1;
    return p;
}

// Conservative lower bound of the squared distance from coordinate x to any
// point stored in cell c along one axis (box widened by eps for rounding in
// the cell assignment).
__device__ __forceinline__ float axis_gap(float x, int c, float origin, float cell, float eps) {
    float lo = origin + (float)c * cell - eps;
    float hi = lo + cell + 2.0f * eps;
    float g = x < lo ? lo - x : (x > hi ? x - hi : 0.0f);
    return g * g;
}

// Cell bounds are compared against the acceptance threshold after scaling by
// (1 - 2^-14): fp32 rounding of the bound and of d2 is far below that margin
// for D <= 128, so a pruned cell never holds an acceptable point.
constexpr float kPruneScale = 1.0f - 1.0f / 16384.0f;

__device__ __forceinline__ int cell_coord(float x, float origin, float inv_cell, int res) {
    int c = (int)floorf((x - origin) * inv_cell);
    return min(max(c, 0), res - 1);
}

}  // namespace frnn
