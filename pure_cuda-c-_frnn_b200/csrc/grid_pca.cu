// grid_pca.cu -- a grid on the data's principal axes (D > 4).
//
// The reference grids D > 4 data on its first coordinates only
// (run_firstd_search, python_interface/frnn_engine.cu:64-102; the first-d
// kernel find_nbrs.cu:243-353): every query then scans every point whose
// first coordinates fall in its 3^g shell, whatever the other coordinates.
// For correlated or low-rank data most of those candidates are far away.
// Projecting onto orthonormal axes never lengthens a distance, so a grid on
// any orthonormal axes finds the same neighbours; on the principal axes the
// shell holds far fewer candidates (cfg3: 423 instead of 5,438 per query,
// cfg4: ~9.6K instead of ~195K, counted on the CPU).
//
// Kernels here:
//   moments   sums of x - x0 and (x - x0)(x - x0)^T over a strided sample, in
//             double, one partial per block, reduced in a fixed order (so every
//             engine given the same points builds the same grid -- the part
//             search relies on it);
//   project   y_k = sum_d P[k][d] (x_d - mu_d) for the top axes (fp32, one fixed
//             order), each point's max |x - mu|^2 and the bounding box of the
//             projected coordinates (last-block fold, as the bbox kernel);
//   estimate  for a sample of queries and points, how many points fall within
//             1.5 cells on every axis of a candidate grid, for the leading-
//             coordinate grid and for principal-axis grids of g = 1..6 axes:
//             the planner keeps the cheapest (isotropic data keeps the leading
//             coordinates, which a rotation would only make worse).
#include "frnn_device.cuh"
#include "frnn_internal.h"

namespace frnn {
namespace {

constexpr int kMomThreads = 256;
constexpr int kMomTile = 64;            // sample points staged per pass
constexpr int kProjThreads = 256;
constexpr int kProjSlots = 2 * kMaxGridAxes + 2;  // (min,max) per axis, max |x-mu|^2, non-finite

__global__ void __launch_bounds__(kMomThreads)
    moments_kernel(const float* __restrict__ pts, int n, int dim, int samples, double* __restrict__ partial,
                   int slots) {
    __shared__ float tile[kMomTile][kMaxPcaDim];
    __shared__ float x0[kMaxPcaDim];
    const int j0 = (int)((long long)samples * blockIdx.x / gridDim.x);
    const int j1 = (int)((long long)samples * (blockIdx.x + 1) / gridDim.x);
    if (threadIdx.x < dim) x0[threadIdx.x] = __ldg(&pts[(long long)threadIdx.x * n]);
    double acc[4] = {0.0, 0.0, 0.0, 0.0};   // slots t, t+256, t+512, t+768
    // slot s < dim: sum of (x_s - x0_s); then the upper triangle (a <= b) of
    // the sum of products, row by row
    int sa[4], sb[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        int s = threadIdx.x + k * kMomThreads;
        sa[k] = -1;
        sb[k] = -1;
        if (s < dim) {
            sa[k] = s;
        } else if (s < slots) {
            s -= dim;
            int a = 0;
            while (s >= dim - a) {
                s -= dim - a;
                ++a;
            }
            sa[k] = a;
            sb[k] = a + s;
        }
    }
    for (int base = j0; base < j1; base += kMomTile) {
        const int m = min(kMomTile, j1 - base);
        __syncthreads();
        for (int e = threadIdx.x; e < m * dim; e += kMomThreads) {
            const int j = base + e / dim, d = e % dim;
            const long long i = (long long)j * n / samples;
            tile[e / dim][d] = __ldg(&pts[(long long)d * n + i]) - x0[d];
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (sa[k] < 0) continue;
            // four chains over j mod 4, folded in a fixed order
            double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
            int j = 0;
            if (sb[k] < 0) {
                for (; j + 3 < m; j += 4) {
                    a0 += (double)tile[j][sa[k]];
                    a1 += (double)tile[j + 1][sa[k]];
                    a2 += (double)tile[j + 2][sa[k]];
                    a3 += (double)tile[j + 3][sa[k]];
                }
                for (; j < m; ++j) a0 += (double)tile[j][sa[k]];
            } else {
                for (; j + 3 < m; j += 4) {
                    a0 += (double)tile[j][sa[k]] * (double)tile[j][sb[k]];
                    a1 += (double)tile[j + 1][sa[k]] * (double)tile[j + 1][sb[k]];
                    a2 += (double)tile[j + 2][sa[k]] * (double)tile[j + 2][sb[k]];
                    a3 += (double)tile[j + 3][sa[k]] * (double)tile[j + 3][sb[k]];
                }
                for (; j < m; ++j) a0 += (double)tile[j][sa[k]] * (double)tile[j][sb[k]];
            }
            acc[k] += (a0 + a1) + (a2 + a3);
        }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int s = threadIdx.x + k * kMomThreads;
        if (s < slots) partial[(long long)blockIdx.x * slots + s] = acc[k];
    }
}

// out[s] = sum of the blocks' partials of slot s, one warp per slot: lane l
// sums blocks l, l + 32, ... and a fixed xor tree folds the lanes (the same
// order on every run); then out[slots + d] = x0_d (the shift the sums are
// taken about)
__global__ void moments_reduce_kernel(const double* __restrict__ partial, int blocks, int slots,
                                      double* __restrict__ out, const float* __restrict__ pts, int n,
                                      int dim) {
    const int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (s >= slots) {
        if (s < slots + dim && lane == 0) out[s] = (double)__ldg(&pts[(long long)(s - slots) * n]);
        return;
    }
    double a = 0.0;
    for (int b = lane; b < blocks; b += 32) a += __ldcg(&partial[(long long)b * slots + s]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) out[s] = a;
}

__global__ void __launch_bounds__(kProjThreads)
    project_kernel(const float* __restrict__ pts, int n, int dim, int axes, const float* __restrict__ mu,
                   const float* __restrict__ pm, float* __restrict__ proj, float* __restrict__ partial,
                   unsigned int* __restrict__ ticket, float* __restrict__ out) {
    __shared__ float smu[kMaxPcaDim];
    __shared__ float spm[kMaxGridAxes][kMaxPcaDim];
    for (int e = threadIdx.x; e < dim; e += blockDim.x) smu[e] = mu[e];
    for (int e = threadIdx.x; e < axes * dim; e += blockDim.x) spm[e / dim][e % dim] = pm[e];
    __syncthreads();
    float mn[kMaxGridAxes], mx[kMaxGridAxes], nmax = 0.0f;
    bool bad = false;
#pragma unroll
    for (int k = 0; k < kMaxGridAxes; ++k) {
        mn[k] = INFINITY;
        mx[k] = -INFINITY;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        float y[kMaxGridAxes];
#pragma unroll
        for (int k = 0; k < kMaxGridAxes; ++k) y[k] = 0.0f;
        float nrm = 0.0f;
        for (int d = 0; d < dim; ++d) {
            const float x = __ldg(&pts[(long long)d * n + i]);
            bad |= !isfinite(x);
            const float c = x - smu[d];
            nrm = __fmaf_rn(c, c, nrm);
#pragma unroll
            for (int k = 0; k < kMaxGridAxes; ++k)
                if (k < axes) y[k] = __fmaf_rn(spm[k][d], c, y[k]);
        }
        float4* dst = reinterpret_cast<float4*>(proj + (long long)i * kProjStride);
        dst[0] = make_float4(y[0], y[1], y[2], y[3]);
        dst[1] = make_float4(y[4], y[5], 0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < kMaxGridAxes; ++k) {
            mn[k] = fminf(mn[k], y[k]);
            mx[k] = fmaxf(mx[k], y[k]);
        }
        nmax = fmaxf(nmax, nrm);
    }
    __shared__ float sred[kProjSlots][kProjThreads / 32];
    __shared__ bool last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int k = 0; k < kMaxGridAxes; ++k) {
        float a = mn[k], b = mx[k];
        for (int o = 16; o > 0; o >>= 1) {
            a = fminf(a, __shfl_xor_sync(0xffffffffu, a, o));
            b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, o));
        }
        if (lane == 0) {
            sred[2 * k][warp] = a;
            sred[2 * k + 1][warp] = b;
        }
    }
    for (int o = 16; o > 0; o >>= 1) nmax = fmaxf(nmax, __shfl_xor_sync(0xffffffffu, nmax, o));
    const bool wbad = __any_sync(0xffffffffu, bad);
    if (lane == 0) {
        sred[kProjSlots - 2][warp] = nmax;
        sred[kProjSlots - 1][warp] = wbad ? 1.0f : 0.0f;
    }
    __syncthreads();
    if (threadIdx.x < kProjSlots) {
        const int t = threadIdx.x;
        const bool is_max = (t & 1) || t >= kProjSlots - 2;
        float acc = sred[t][0];
        for (int w = 1; w < kProjThreads / 32; ++w) acc = is_max ? fmaxf(acc, sred[t][w]) : fminf(acc, sred[t][w]);
        partial[(long long)blockIdx.x * kProjSlots + t] = acc;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (threadIdx.x < kProjSlots) {
        const int t = threadIdx.x;
        const bool is_max = (t & 1) || t >= kProjSlots - 2;
        float acc = is_max ? -INFINITY : INFINITY;
        for (int b = 0; b < (int)gridDim.x; ++b) {
            const float v = ((volatile float*)partial)[(long long)b * kProjSlots + t];
            acc = is_max ? fmaxf(acc, v) : fminf(acc, v);
        }
        out[t] = acc;
    }
    if (threadIdx.x == 0) *ticket = 0u;
}

// smp[c*m + j], column c = leading coordinate c (c < 8, zero past 6 or D)
// or projected coordinate c - 8, of sample point j (point j * n / m):
// column-major, so a warp's loads of one column are one 128-byte line.
__global__ void sample_kernel(const float* __restrict__ pts, int n, int dim, const float* __restrict__ proj,
                              int m, float* __restrict__ smp) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= m) return;
    const long long i = (long long)j * n / m;
#pragma unroll
    for (int d = 0; d < 8; ++d)
        smp[(long long)d * m + j] = d < dim && d < kMaxGridAxes ? __ldg(&pts[(long long)d * n + i]) : 0.0f;
#pragma unroll
    for (int d = 0; d < 8; ++d) smp[(long long)(8 + d) * m + j] = __ldg(&proj[i * kProjStride + d]);
}

// counts[q*16 + b*8 + g-1] += sample points within half-width h[b*8 + g-1] of
// sample query q (query q = sample point q * m / nq) on each of the first g
// axes of basis b (0 leading coordinates, 1 principal axes); block (q, y)
// scans the y-th of gridDim.y slices of the sample points (integer sums, so
// the total does not depend on the order).
__global__ void __launch_bounds__(256) estimate_kernel(const float* __restrict__ smp, int m, int nq,
                                                       const float* __restrict__ h, int* __restrict__ counts) {
    __shared__ float qv[16];
    __shared__ float hh[16];
    __shared__ int red[16][8];
    const int q = (int)((long long)blockIdx.x * m / nq);
    if (threadIdx.x < 16) {
        qv[threadIdx.x] = smp[(long long)threadIdx.x * m + q];
        hh[threadIdx.x] = h[threadIdx.x];
    }
    __syncthreads();
    int c[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) c[t] = 0;
    const int j0 = (int)((long long)m * blockIdx.y / gridDim.y), j1 = (int)((long long)m * (blockIdx.y + 1) / gridDim.y);
#pragma unroll 2
    for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            float run = 0.0f;
#pragma unroll
            for (int g = 0; g < kMaxGridAxes; ++g) {
                run = fmaxf(run, fabsf(__ldg(&smp[(long long)(8 * b + g) * m + j]) - qv[8 * b + g]));
                c[8 * b + g] += run < hh[8 * b + g] ? 1 : 0;
            }
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int t = 0; t < 16; ++t) {
        int v = c[t];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[t][warp] = v;
    }
    __syncthreads();
    if (threadIdx.x < 16) {
        int a = 0;
        for (int w = 0; w < 8; ++w) a += red[threadIdx.x][w];
        atomicAdd(&counts[(long long)blockIdx.x * 16 + threadIdx.x], a);
    }
}

}  // namespace

int pca_slots(int dim) { return dim + dim * (dim + 1) / 2; }

cudaError_t launch_pca_moments(const float* pts, int n, int dim, int samples, int blocks, double* partial,
                               double* out, cudaStream_t s) {
    if (dim > kMaxPcaDim || pca_slots(dim) > 4 * kMomThreads) return cudaErrorInvalidValue;
    const int slots = pca_slots(dim);
    moments_kernel<<<blocks, kMomThreads, 0, s>>>(pts, n, dim, samples, partial, slots);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    moments_reduce_kernel<<<(slots + dim + 3) / 4, 128, 0, s>>>(partial, blocks, slots, out, pts, n, dim);
    return cudaGetLastError();
}

int pca_project_slots() { return kProjSlots; }

cudaError_t launch_pca_project(const float* pts, int n, int dim, int axes, const float* mu, const float* pm,
                               float* proj, float* partial, unsigned int* ticket, float* out, int blocks,
                               cudaStream_t s) {
    if (dim > kMaxPcaDim || axes > kMaxGridAxes) return cudaErrorInvalidValue;
    project_kernel<<<blocks, kProjThreads, 0, s>>>(pts, n, dim, axes, mu, pm, proj, partial, ticket, out);
    return cudaGetLastError();
}

cudaError_t launch_pca_estimate(const float* pts, int n, int dim, const float* proj, int m, int nq, float* smp,
                                const float* h, int* counts, cudaStream_t s) {
    sample_kernel<<<(m + 255) / 256, 256, 0, s>>>(pts, n, dim, proj, m, smp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(counts, 0, (size_t)nq * 16 * sizeof(int), s);
    if (e != cudaSuccess) return e;
    estimate_kernel<<<dim3(nq, 8), 256, 0, s>>>(smp, m, nq, h, counts);
    return cudaGetLastError();
}

}  // namespace frnn
