// frnn_device.cuh -- types and device helpers shared by the engine's kernels.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace frnn {

constexpr int kMaxK = 128;           // grid.h:59 MAX_K_CAPACITY
constexpr int kMaxD = 128;           // grid.h:60 MAX_DIM_SUPPORTED
constexpr int kMaxGridAxes = 4;

// Grid description computed on the host from the data's bounding box.
// Replaces the reference's GridParams (grid.h:38-52): per-axis resolution and
// origin instead of a fixed [0,1] domain, and axis 0 varying fastest in the
// dense cell index so the three x-neighbours of a cell are one contiguous span.
struct GridPlan {
    int g;                       // grid axes = leading coordinates used for cells
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

// Per-thread K-selection state kept in shared memory, one column per thread
// ([slot][thread] layout: every lane addresses its own bank whatever the slot).
// Holds up to K keys; while fewer than K are held it is an unsorted list, at K
// it becomes a max-heap whose root is the acceptance threshold.  A candidate
// is accepted iff d2 < r2 and its key is below the threshold, which is the
// reference's rule (heap initialised to (r2,-1), strict d2 < root,
// find_nbrs.cu:77-97, :136-143) with ties broken by the smaller index.
struct TopK {
    unsigned long long* col;  // &smem[threadIdx.x]
    int S;                    // column stride (= blockDim.x)
    int K;
    int n;
    unsigned long long thr;   // acceptance bound (exclusive)

    __device__ __forceinline__ void init(unsigned long long* base, int stride, int k, float r2) {
        col = base;
        S = stride;
        K = k;
        n = 0;
        thr = make_key(r2, 0);  // d2 < r2  <=>  key(d2, idx) < key(r2, 0)
    }
    __device__ __forceinline__ float thr_d2() const { return key_d2(thr); }
    __device__ __forceinline__ unsigned long long at(int i) const { return col[(long long)i * S]; }
    __device__ __forceinline__ void put(int i, unsigned long long v) { col[(long long)i * S] = v; }

    __device__ __forceinline__ void sift_down(int i, int size) {
        unsigned long long v = at(i);
        while (true) {
            int l = 2 * i + 1;
            if (l >= size) break;
            unsigned long long lv = at(l);
            int r = l + 1;
            if (r < size) {
                unsigned long long rv = at(r);
                if (rv > lv) { l = r; lv = rv; }
            }
            if (lv <= v) break;
            put(i, lv);
            i = l;
        }
        put(i, v);
    }
    __device__ __forceinline__ void heapify(int size) {
        for (int i = size / 2 - 1; i >= 0; --i) sift_down(i, size);
    }
    // Caller has checked key < thr.
    __device__ __forceinline__ void push(unsigned long long key) {
        if (n < K) {
            put(n, key);
            if (++n == K) {
                heapify(K);
                thr = at(0);
            }
        } else {
            put(0, key);
            sift_down(0, K);
            thr = at(0);
        }
    }
    // Write the held keys ascending to out rows 0..n-1 and pad rows n..K-1
    // with (-1, r2).  Output element k goes to idx[k*ostride], dist[k*ostride].
    __device__ __forceinline__ void emit(int* __restrict__ oidx, float* __restrict__ odist,
                                         long long ostride, float r2) {
        if (n < K && n > 1) heapify(n);
        for (int k = K - 1; k >= n; --k) {
            oidx[k * ostride] = -1;
            odist[k * ostride] = r2;
        }
        for (int m = n - 1; m >= 0; --m) {
            unsigned long long top = at(0);
            oidx[m * ostride] = key_idx(top);
            odist[m * ostride] = key_d2(top);
            if (m > 0) {
                put(0, at(m));
                sift_down(0, m);
            }
        }
    }
};

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
