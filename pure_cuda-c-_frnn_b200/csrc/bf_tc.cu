// bf_tc.cu -- brute force with a tcgen05 distance filter (D <= 128; the
// dispatcher takes it for D > 32).
//
// Replaces, for high D, the reference's TiledBruteforceNDKernel<128> and its
// launcher (frnn/csrc/no_grid_frnn/no_grid_frnn.cu:121-326): every query
// against every point, d2 < r2 accepted, the K smallest kept.  The all-pairs
// work is a dense contraction, so it runs on the tensor cores:
//
//   prep     one pass over the SoA input: per-dimension centre c and a power
//            of two s, then for every point H = s*(x - c) rounded to fp16 in
//            128-row tiles laid out exactly as the SW128 K-major shared-memory
//            operand (so a tile is one plain bulk copy), the point's fp32 row
//            (for the exact re-rank) and two per-point threshold terms.
//   filter   P = H_q . H_p for 128 x 128 tiles on tcgen05 (fp16 in, fp32
//            accumulators in TMEM).  A pair is a candidate when
//            n_q + n_p - 2P < s^2 r^2 + margin(q, p), written as
//            P - b_p > a_q; candidate point indices are appended to the
//            query's list.  Warp-specialised: one producer warp (bulk copies
//            into a 4- or 8-stage ring), one MMA warp (a single thread issues
//            the MMAs, commits release the ring stage and publish the
//            accumulator), sixteen epilogue warps (two groups alternating over
//            two TMEM accumulator buffers, so the next tile's MMAs overlap the
//            current tile's filter).  The epilogue tests 8-column group maxima
//            first and builds a bitmask only where a group passes, so the
//            per-candidate work stays off the common path.
//   rerank   one warp per query: every candidate's d2 is recomputed with the
//            engine's canonical fp32 order (the chain; the D = 3 order for
//            D = 3) from the fp32 rows, accepted when
//            d2 < r2, and the K smallest (d2, index) are emitted -- the same
//            results, bit for bit, as the SIMT brute force.
//
// Why the filter is exact (never drops a true neighbour).  With u = 2^-11 the
// fp16 unit roundoff and eta = 2^-25 its subnormal absolute roundoff, each
// fp16 coordinate h = H + delta with |delta| <= u|H| + eta.  Then
//   |2(h_q.h_p) - 2(H_q.H_p)| <= 4u|H_q||H_p| + 2 eta sqrt(D)(|H_q| + |H_p|) + 2 D eta^2,
// fp16 products are exact in fp32 and the accumulation adds at most
// gamma * sum|h_q h_p| (gamma well below 2^-12 for fp32 accumulators over
// D <= 128 terms), the centring and the fp32 norms add relative errors of
// order D 2^-24, and the chain d2 the engine accepts on differs from the real
// d2 by at most (D+1) 2^-24 d2.  With 2|H_q||H_p| <= n_q + n_p, alpha = 2^-8
// covers 2u + gamma + the fp32 terms with room to spare; the r^2 side takes a
// 2^-15 relative allowance and the eta terms are kept per point.  The margin
// only admits extra candidates, which the exact re-rank rejects.
//
// Every wait on an mbarrier is bounded (kWaitPolls polls and kWaitNs of
// global time); a wait that gives up sets the error flag, the other roles stop
// at their next wait, the MMA thread waits (bounded) for its own MMAs, the
// producer for its own copies in flight, and TMEM is freed before exit.
#include <cuda_fp16.h>
#include <cstdint>

#include "frnn_device.cuh"
#include "frnn_internal.h"
#include "grid_coop.cuh"

namespace frnn {
namespace tc {
namespace {

constexpr int kRows = 128;            // rows of a tile: M of the query block, N of a point tile
constexpr int kAtomBytes = 16384;     // 128 rows x 64 fp16 dims, SW128 K-major
// Epilogue warps: two groups (one per TMEM accumulator buffer) of 4 or 8
// warps; a warp reads the TMEM lanes of its subpartition (warp % 4) and
// 128 / (kEpiWarps / 8) of the tile's columns.  Build-time launch-policy knob;
// 16 measured 13% faster than 8 on B200 (cfg5: 290 against 332 ms).
#ifndef FRNN_TC_EPI_WARPS
#define FRNN_TC_EPI_WARPS 16
#endif
constexpr int kEpiWarps = FRNN_TC_EPI_WARPS;
static_assert(kEpiWarps == 8 || kEpiWarps == 16, "two groups of 4 or 8 warps");
constexpr int kChunksPerWarp = 4 / (kEpiWarps / 8);   // 32-column chunks per warp and block
constexpr int kThreads = (kEpiWarps + 2) * 32;
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;
constexpr int kTmemCols = 512;        // 2 query blocks x 2 buffers x 128 columns
constexpr uint32_t kWaitPolls = 1u << 26;
constexpr unsigned long long kWaitNs = 2000000000ull;

template <int KC>
struct Cfg {
    static constexpr int kStages = KC == 2 ? 4 : 8;
    static constexpr uint32_t kTileBytes = KC * kAtomBytes;
    static constexpr size_t kBarOffset = (size_t)(2 + kStages) * kTileBytes;
    // full[S], empty[S], tfull[2], tempty[2], afull, done
    static constexpr int kBars = 2 * kStages + 6;
    static constexpr size_t kSmem =
        1024 /* alignment slack */ + kBarOffset + kBars * 8 + 16 /* tmem slot, abort */ +
        2 * kRows * 4 /* per-query counters */ + 16 + kEpiWarps * kChunksPerWarp * 32 * 4 /* point terms */;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase of parity `parity`; false when it gave up (or
// another role already did).
__device__ __noinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (uint32_t i = 1; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort) return false;
            if (global_ns() - t0 > kWaitNs) return false;
        }
    }
    return false;
}
// Bounded wait that ignores the abort flag: used only to let this thread's own
// copies or MMAs finish before the CTA releases its memory.
__device__ __noinline__ void drain_wait(uint32_t bar, uint32_t parity) {
    const unsigned long long t0 = global_ns();
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return;
        if ((i & 255u) == 255u && global_ns() - t0 > kWaitNs) return;
    }
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// SW128 K-major shared-memory operand descriptor: 128-byte rows, 8-row groups
// 1024 bytes apart (stride byte offset), version 1, swizzle mode 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::f16 instruction descriptor: fp32 accumulate, fp16 A and B, both
// K-major, M = 128, N = 128.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kRows >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
          "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
          "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
          "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- prep -------------------------------------------------------------------

// Per-dimension min / max of the SoA input and a flag for non-finite
// coordinates.  box[2d] = min, box[2d+1] = max.  Blocks of 4,096 values of one
// dimension each (grid: chunks x dimensions) fold into the box with atomic
// min / max on an order-preserving unsigned encoding of the floats; the box
// words hold the encoding until box_final_kernel decodes them.
constexpr int kBoxChunk = 4096;

__device__ __forceinline__ unsigned order_key(float f) {
    const unsigned b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float order_value(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__global__ void box_init_kernel(unsigned* __restrict__ keys, int dim) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= dim) return;
    keys[2 * d] = 0xffffffffu;
    keys[2 * d + 1] = 0u;
}

__global__ void __launch_bounds__(256) dim_box_kernel(const float* __restrict__ pts, int n,
                                                      unsigned* __restrict__ keys, int* __restrict__ nonfinite) {
    const int d = blockIdx.y;
    const float* col = pts + (long long)d * n;
    const int i0 = blockIdx.x * kBoxChunk, i1 = min(n, i0 + kBoxChunk);
    float lo = __int_as_float(0x7f800000), hi = -__int_as_float(0x7f800000);
    bool bad = false;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const float x = __ldg(&col[i]);
        bad |= !isfinite(x);
        lo = fminf(lo, x);
        hi = fmaxf(hi, x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    bad = __any_sync(0xffffffffu, bad);
    __shared__ float slo[8], shi[8];
    __shared__ int sbad;
    if (threadIdx.x == 0) sbad = 0;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
        slo[threadIdx.x >> 5] = lo;
        shi[threadIdx.x >> 5] = hi;
        if (bad) sbad = 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
            lo = fminf(lo, slo[w]);
            hi = fmaxf(hi, shi[w]);
        }
        atomicMin(&keys[2 * d], order_key(lo));
        atomicMax(&keys[2 * d + 1], order_key(hi));
        if (sbad) atomicOr(nonfinite, 1);
    }
}

__global__ void box_final_kernel(unsigned* __restrict__ keys, int dim) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= 2 * dim) return;
    reinterpret_cast<float*>(keys)[i] = order_value(keys[i]);
}

// One thread per (padded) point: fp16 swizzled tile rows, fp32 rows, and the
// threshold terms qa (query side) and pb (point side).
__global__ void __launch_bounds__(128) prep_kernel(const float* __restrict__ pts, int n, int dim, int npad,
                                                   int kc_n, const float* __restrict__ center, float s,
                                                   float one_minus_alpha, float eta_c, float rc,
                                                   uint8_t* __restrict__ tiles, float* __restrict__ rows32,
                                                   int dp, float* __restrict__ qa, float* __restrict__ pb) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= npad) return;
    const bool real = i < n;
    const int t = i / kRows, r = i % kRows;
    float nsum = 0.0f;
    for (int kc = 0; kc < kc_n; ++kc) {
        uint8_t* atom = tiles + ((size_t)t * kc_n + kc) * kAtomBytes + (size_t)r * 128;
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
            const int d0 = kc * 64 + c * 8;
            float x[8];
            __align__(16) __half h[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int d = d0 + e;
                x[e] = (real && d < dim) ? __ldg(&pts[(long long)d * n + i]) : 0.0f;
                const float H = (real && d < dim) ? s * (x[e] - __ldg(&center[d])) : 0.0f;
                nsum = __fmaf_rn(H, H, nsum);
                h[e] = __float2half_rn(H);
            }
            *reinterpret_cast<uint4*>(atom + ((c ^ (r & 7)) * 16)) = *reinterpret_cast<const uint4*>(h);
            if (real) {
                float* row = rows32 + (size_t)i * dp;
                if (d0 + 4 <= dp) *reinterpret_cast<float4*>(row + d0) = make_float4(x[0], x[1], x[2], x[3]);
                if (d0 + 8 <= dp) *reinterpret_cast<float4*>(row + d0 + 4) = make_float4(x[4], x[5], x[6], x[7]);
            }
        }
    }
    if (real) {
        const float eta_term = eta_c * sqrtf(nsum);
        pb[i] = 0.5f * (one_minus_alpha * nsum - eta_term);
        qa[i] = 0.5f * (one_minus_alpha * nsum - eta_term - rc);
    } else {
        pb[i] = __int_as_float(0x7f800000);
        qa[i] = __int_as_float(0x7f800000);
    }
}

// ---- filter -----------------------------------------------------------------

// Group maxima of (acc[i] - b[i]) over the four 8-column groups of a chunk:
// packed fp32x2 subtractions (each lane rounded to nearest, as a scalar
// subtraction) and three-input maxima.  NaN differences are ignored, so they
// never pass.
__device__ __forceinline__ void group_max(const uint32_t (&acc)[32], const float (&b)[32], float (&m)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        m[j] = -__int_as_float(0x7f800000);
#pragma unroll
        for (int i = 8 * j; i < 8 * j + 8; i += 2) {
            float d0, d1;
            asm("{\n\t.reg .b64 x, y, z;\n\t"
                "mov.b64 x, {%2, %3};\n\t"
                "mov.b64 y, {%4, %5};\n\t"
                "sub.rn.f32x2 z, x, y;\n\t"
                "mov.b64 {%0, %1}, z;\n\t}"
                : "=f"(d0), "=f"(d1)
                : "f"(__uint_as_float(acc[i])), "f"(__uint_as_float(acc[i + 1])), "f"(b[i]), "f"(b[i + 1]));
            asm("max.f32 %0, %1, %2, %3;" : "=f"(m[j]) : "f"(m[j]), "f"(d0), "f"(d1));
        }
    }
}

// Filters one 32-column chunk for one query row: the cheap group maxima
// first; only groups whose maximum passes are tested column by column, then
// the passing columns are appended to query q's list with one shared-memory
// atomic for the lane's slots and independent stores.
__device__ __forceinline__ void filter_chunk(const uint32_t (&acc)[32], const float (&b)[32], float a, int* cnt,
                                             int* __restrict__ lists, int q, int cap, int col0) {
    float m[4];
    group_max(acc, b, m);
    if (fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])) > a) {
        uint32_t mask = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (m[j] > a) {
#pragma unroll
                for (int i = 8 * j; i < 8 * j + 8; ++i)
                    mask |= (__uint_as_float(acc[i]) - b[i] > a ? 1u : 0u) << i;
            }
        }
        int slot = atomicAdd(cnt, __popc(mask));
        int* dst = lists + (size_t)q * cap;
        while (mask) {
            const int i = __ffs(mask) - 1;
            mask &= mask - 1;
            if (slot < cap) dst[slot] = col0 + i;
            ++slot;
        }
    }
}

// The same for a symmetric search (a self-search that filters each pair of
// tiles once): the query's appends take their slots from the global counter
// counts[q], and with `both` (a tile off the diagonal) every passing column p
// also gets q appended to its own list, the pair seen from p's side.  The
// threshold test is symmetric in q and p (n_q + n_p - 2 q.p against margins
// that add a term of each), so one test decides both lists.  Padding rows and
// columns carry +inf terms and never pass.
__device__ __forceinline__ void filter_chunk_sym(const uint32_t (&acc)[32], const float (&b)[32], float a,
                                                 int* __restrict__ counts, int* __restrict__ lists, int q, int cap,
                                                 int col0, bool both) {
    float m[4];
    group_max(acc, b, m);
    if (fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])) > a) {
        uint32_t mask = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (m[j] > a) {
#pragma unroll
                for (int i = 8 * j; i < 8 * j + 8; ++i)
                    mask |= (__uint_as_float(acc[i]) - b[i] > a ? 1u : 0u) << i;
            }
        }
        if (mask == 0) return;
        int slot = atomicAdd(&counts[q], __popc(mask));
        int* dst = lists + (size_t)q * cap;
        while (mask) {
            const int i = __ffs(mask) - 1;
            mask &= mask - 1;
            if (slot < cap) dst[slot] = col0 + i;
            ++slot;
            if (both) {
                const int p = col0 + i;
                const int ps = atomicAdd(&counts[p], 1);
                if (ps < cap) lists[(size_t)p * cap + ps] = q;
            }
        }
    }
}

// sym (a whole self-search only): the CTA of query blocks qb0, qb0 + 1 filters
// point tiles t >= qb0 only -- each unordered pair of tiles once, so half the
// MMAs -- block qb0 + 1 skipping tile qb0 (its transpose, tile qb0 + 1 of
// block qb0, is filtered); tiles off a block's diagonal append each passing
// pair to both lists.  counts[] must be zero on entry and is final only when
// the kernel has finished (appends come from every CTA), so the overflow
// list is made afterwards by sym_overflow_kernel.  CTA 0 has the most tiles
// and starts first.  In a sharded search the CTAs cover this rank's query
// blocks [qb_begin, qb_end) and the pairs seen from points other ranks own
// stay in this rank's lists until those ranks pull them (tc_pull_kernel).
template <int KC>
__global__ void __launch_bounds__(kThreads, 1)
    filter_kernel(const uint8_t* __restrict__ tiles, const float* __restrict__ qa, const float* __restrict__ pb,
                  int n, int ntiles, int cap, int* __restrict__ lists, int* __restrict__ counts,
                  int* __restrict__ overflow, int* __restrict__ n_overflow, int* __restrict__ err,
                  int qb_begin, int qb_end, const uint8_t* __restrict__ qtiles, int skip_tile, int sym) {
    // qtiles: the query blocks' tiles (the points' own tiles for a self-query)
    using C = Cfg<KC>;
    constexpr int S = C::kStages;
    constexpr uint32_t TB = C::kTileBytes;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* base = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    const uint32_t sA = smem_u32(base);
    const uint32_t sB = sA + 2 * TB;
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + C::kBarOffset);
    const uint32_t bar0 = smem_u32(bars);
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (S + s); };
    auto tfull = [&](int b) { return bar0 + 8u * (2 * S + b); };
    auto tempty = [&](int b) { return bar0 + 8u * (2 * S + 2 + b); };
    const uint32_t afull = bar0 + 8u * (2 * S + 4);
    const uint32_t done = bar0 + 8u * (2 * S + 5);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kBars);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* qcnt = reinterpret_cast<int*>(tmem_slot + 4);
    // [kEpiWarps][kChunksPerWarp * 32], 16-byte aligned (read as float4)
    float* pbstage =
        reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(qcnt + 2 * kRows) + 15) & ~uintptr_t(15));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // this CTA's two query blocks (the second absent at an odd end); the point
    // tiles are all ntiles
    const int qb0 = qb_begin + 2 * blockIdx.x;
    const bool has1 = qb0 + 1 < qb_end;
    const int qb1 = has1 ? qb0 + 1 : qb0;
    // the point tiles filtered: t0 + i for i < ntl
    const int t0 = sym ? qb0 : 0;
    const int ntl = ntiles - t0;

    if (threadIdx.x < 2 * kRows) qcnt[threadIdx.x] = 0;
    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull(b), 1);
            mbar_init(tempty(b), kEpiWarps / 2);
        }
        mbar_init(afull, 1);
        mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kProducerWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;

    auto give_up = [&]() {
        *abort_flag = 1;
        atomicExch(err, 1);
    };

    if (warp == kProducerWarp) {
        if (lane == 0) {
            mbar_expect_tx(afull, (has1 ? 2u : 1u) * TB);
            bulk_g2s(sA, qtiles + (size_t)qb0 * TB, TB, afull);
            if (has1) bulk_g2s(sA + TB, qtiles + (size_t)qb1 * TB, TB, afull);
            int issued = 0;
            for (int i = 0; i < ntl; ++i) {
                const int t = t0 + i, s = i % S;
                const uint32_t u = (uint32_t)(i / S);
                if (!mbar_wait(empty(s), (u & 1u) ^ 1u, abort_flag)) {
                    give_up();
                    break;
                }
                // skip_tile (tests of the timeout path only): this stage is
                // never filled, so the MMA thread's wait for it gives up
                if (t != skip_tile) {
                    mbar_expect_tx(full(s), TB);
                    bulk_g2s(sB + (uint32_t)s * TB, tiles + (size_t)t * TB, TB, full(s));
                }
                issued = i + 1;
            }
            // copies still in flight land before the CTA may exit
            drain_wait(afull, 0);
            for (int i = issued - S < 0 ? 0 : issued - S; i < issued; ++i)
                if (t0 + i != skip_tile) drain_wait(full(i % S), (uint32_t)(i / S) & 1u);
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            bool ok = mbar_wait(afull, 0, abort_flag);
            if (!ok) give_up();
            for (int i = 0; ok && i < ntl; ++i) {
                const int t = t0 + i, s = i % S, b = i & 1;
                const uint32_t u = (uint32_t)(i / S), v = (uint32_t)(i >> 1);
                if (!mbar_wait(full(s), u & 1u, abort_flag) || !mbar_wait(tempty(b), (v & 1u) ^ 1u, abort_flag)) {
                    give_up();
                    break;
                }
                fence_after();
                const uint32_t bstage = sB + (uint32_t)s * TB;
                for (int a = 0; a < (has1 ? 2 : 1); ++a) {
                    if (sym && a == 1 && t < qb1) continue;  // the transpose of a pair filtered by block 0
                    const uint32_t d = tmem + (uint32_t)((a * 2 + b) * kRows);
                    const uint32_t astage = sA + (uint32_t)a * TB;
#pragma unroll
                    for (int k = 0; k < 4 * KC; ++k) {
                        const uint32_t off = (uint32_t)((k >> 2) * kAtomBytes + (k & 3) * 32);
                        mma_f16(d, sw128_desc(astage + off), sw128_desc(bstage + off), k > 0 ? 1u : 0u);
                    }
                }
                mma_commit(empty(s));
                mma_commit(tfull(b));
            }
            // every MMA issued above completes before TMEM is released
            mma_commit(done);
            drain_wait(done, 0);
        }
    } else {
        // epilogue: group g takes the tiles t = g (mod 2), TMEM buffer g
        const int sp = warp & 3, g = (warp >> 2) & 1, h = warp >> 3;
        const int row = sp * 32 + lane;
        const float aq0 = __ldg(&qa[(size_t)qb0 * kRows + row]);
        const float aq1 = has1 ? __ldg(&qa[(size_t)qb1 * kRows + row]) : __int_as_float(0x7f800000);
        const int q0 = qb0 * kRows + row, q1 = qb1 * kRows + row;
        const uint32_t lane_base = (uint32_t)(sp * 32) << 16;
        // the point-side terms of this warp's columns: loaded one tile ahead
        // into registers, staged in shared memory for the tile being filtered
        constexpr int kCols = kChunksPerWarp * 32;
        float* spb = pbstage + warp * kCols;
        static_assert(kCols == 64, "two terms per lane");
        auto load_terms = [&](int t) {
            const float* src = pb + (size_t)t * kRows + h * kCols + lane;
            return t < ntiles ? make_float2(__ldg(src), __ldg(src + 32)) : make_float2(0.0f, 0.0f);
        };
        float2 terms = load_terms(t0 + g);
        for (int i = g; i < ntl; i += 2) {
            const int t = t0 + i;
            const uint32_t v = (uint32_t)(i >> 1);
            // warp-uniform outcome: the TMEM loads below need the whole warp
            if (!__all_sync(0xffffffffu, mbar_wait(tfull(g), v & 1u, abort_flag))) {
                if (lane == 0) give_up();
                break;
            }
            fence_after();
            __syncwarp();
            spb[lane] = terms.x;
            spb[32 + lane] = terms.y;
            __syncwarp();
            terms = load_terms(t + 2);
#pragma unroll 1
            for (int c = h * kChunksPerWarp; c < (h + 1) * kChunksPerWarp; ++c) {
                // the point tile's threshold terms, shared by both query blocks
                float bq[32];
                const float4* b4 = reinterpret_cast<const float4*>(spb + (c - h * kChunksPerWarp) * 32);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 bb = b4[i];
                    bq[4 * i] = bb.x;
                    bq[4 * i + 1] = bb.y;
                    bq[4 * i + 2] = bb.z;
                    bq[4 * i + 3] = bb.w;
                }
                if (sym) {
#pragma unroll 1
                    for (int a = 0; a < (has1 ? 2 : 1); ++a) {
                        const int qb = a ? qb1 : qb0;
                        if (t < qb) continue;  // block 1 at tile qb0: filtered as its transpose
                        uint32_t acc[32];
                        __syncwarp();
                        tmem_ld32(tmem + lane_base + (uint32_t)((2 * a + g) * kRows + c * 32), acc);
                        tmem_wait_ld();
                        filter_chunk_sym(acc, bq, a ? aq1 : aq0, counts, lists, a ? q1 : q0, cap,
                                         t * kRows + c * 32, t != qb);
                    }
                } else if (kEpiWarps == 8) {
                    // both blocks' loads in flight before one wait
                    uint32_t acc0[32], acc1[32];
                    __syncwarp();
                    tmem_ld32(tmem + lane_base + (uint32_t)(g * kRows + c * 32), acc0);
                    if (has1) tmem_ld32(tmem + lane_base + (uint32_t)((2 + g) * kRows + c * 32), acc1);
                    tmem_wait_ld();
                    filter_chunk(acc0, bq, aq0, &qcnt[row], lists, q0, cap, t * kRows + c * 32);
                    if (has1) filter_chunk(acc1, bq, aq1, &qcnt[kRows + row], lists, q1, cap, t * kRows + c * 32);
                } else {
                    // one block at a time (register budget of 18 warps)
#pragma unroll 1
                    for (int a = 0; a < (has1 ? 2 : 1); ++a) {
                        uint32_t acc[32];
                        __syncwarp();
                        tmem_ld32(tmem + lane_base + (uint32_t)((2 * a + g) * kRows + c * 32), acc);
                        tmem_wait_ld();
                        filter_chunk(acc, bq, a ? aq1 : aq0, &qcnt[a * kRows + row], lists, a ? q1 : q0, cap,
                                     t * kRows + c * 32);
                    }
                }
            }
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty(g));
        }
    }

    fence_before();
    __syncthreads();
    if (!sym && threadIdx.x < 2 * kRows) {
        const int a = threadIdx.x / kRows, row = threadIdx.x % kRows;
        const int q = (a ? qb1 : qb0) * kRows + row;
        if ((a == 0 || has1) && q < n) {
            const int c = qcnt[threadIdx.x];
            counts[q] = c;
            if (c > cap) overflow[atomicAdd(n_overflow, 1)] = q;
        }
    }
    if (warp == kProducerWarp) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
    }
}

// A sharded symmetric filter leaves the pairs seen from a point in the lists
// of the rank that filtered them.  One warp per query q of this rank's range
// [q0, q1): from every other rank, its count for q and that many list entries
// (plain loads from memory mapped through CUDA IPC, a warp's entries
// contiguous), appended to q's own list.  A source list that overflowed its
// capacity carries a count above cap, so q's merged count does too and q
// goes to the overflow fallback.
__global__ void __launch_bounds__(256) tc_pull_kernel(const TcPeers peers, int self, int* __restrict__ counts,
                                                      int* __restrict__ lists, int q0, int q1, int cap) {
    const int lane = threadIdx.x & 31;
    const int q = q0 + (blockIdx.x * blockDim.x + threadIdx.x) / 32;
    if (q >= q1) return;
    for (int r = 0; r < peers.n; ++r) {
        if (r == self) continue;
        const int c = peers.counts[r][q];
        if (c == 0) continue;
        int base = 0;
        if (lane == 0) base = atomicAdd(&counts[q], c);
        base = __shfl_sync(0xffffffffu, base, 0);
        const int* src = peers.lists[r] + (size_t)q * cap;
        int* dst = lists + (size_t)q * cap;
        for (int j = lane; j < min(c, cap); j += 32)
            if (base + j < cap) dst[base + j] = src[j];
    }
}

// After a symmetric filter: the queries whose candidates overflowed their list.
__global__ void __launch_bounds__(256) sym_overflow_kernel(const int* __restrict__ counts, int q0, int q1, int cap,
                                                           int* __restrict__ overflow,
                                                           int* __restrict__ n_overflow) {
    const int q = q0 + blockIdx.x * blockDim.x + threadIdx.x;
    if (q < q1 && __ldg(&counts[q]) > cap) overflow[atomicAdd(n_overflow, 1)] = q;
}

// ---- exact re-rank ----------------------------------------------------------

constexpr int kRerankWarps = 4;

// Row stride of the staged candidate rows in shared memory, in floats: the
// row plus 4 or 8 floats so that stride / 4 is odd, and the eight lanes of a
// quarter warp, each reading 16 bytes at the same column of its own row, hit
// distinct banks.
__host__ __device__ inline int rerank_stride(int dp) { return dp + ((dp & 4) ? 8 : 4); }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}

// One warp per query, one lane per candidate.  The candidates' fp32 rows are
// random reads (512 bytes at D = 128); each pass of 32 candidates first
// stages all 32 rows in shared memory, every row copied by the warp as one
// coalesced run of 16-byte cp.async copies, so a warp has the whole pass's
// rows in flight at once and holds no registers for them; then each lane
// runs its candidate's chain from shared memory.
template <int LCAP>
__global__ void __launch_bounds__(kRerankWarps * 32)
    rerank_kernel(const float* __restrict__ rows32, int dim, int dp, const int* __restrict__ lists,
                  const int* __restrict__ counts, int cap, int K, float r2, int* __restrict__ oidx,
                  float* __restrict__ odist, int q0, int q1, const float* __restrict__ qrows32) {
    extern __shared__ unsigned long long rsmem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int stride = rerank_stride(dp);
    unsigned long long* keys = rsmem + (size_t)warp * LCAP;
    float* fbase = reinterpret_cast<float*>(rsmem + (size_t)kRerankWarps * LCAP);
    float* qrow = fbase + (size_t)warp * dp;
    float* stage = fbase + (size_t)kRerankWarps * dp + (size_t)warp * 32 * stride;
    const bool d3 = dp == 4 && dim == 3;
    const int q = q0 + blockIdx.x * kRerankWarps + warp;
    if (q >= q1) return;
    const int cnt = __ldg(&counts[q]);
    if (cnt > cap) return;  // searched by the fallback
    const float* qsrc = qrows32 + (size_t)q * dp;  // the query's own fp32 row
    for (int d = lane; d < dp; d += 32) qrow[d] = __ldg(&qsrc[d]);
    const int* mine = lists + (size_t)q * cap;
    const float4* q4 = reinterpret_cast<const float4*>(qrow);
    const int nv = dp / 4;
    unsigned long long thr = make_key(r2, 0);
    int nl = 0;
    for (int base = 0; base < cnt; base += 32) {
        const int j = base + lane;
        const int nrow = min(32, cnt - base);
        const int p = j < cnt ? __ldg(&mine[j]) : 0;
        for (int r = 0; r < nrow; ++r) {
            const int pr = __shfl_sync(0xffffffffu, p, r);
            for (int c = lane; c < nv; c += 32)
                cp_async16(stage + r * stride + 4 * c, rows32 + (size_t)pr * dp + 4 * c);
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncwarp();
        unsigned long long key = ~0ull;
        bool acc = false;
        if (j < cnt) {
            const float4* prow = reinterpret_cast<const float4*>(stage + lane * stride);
            float d2 = 0.0f;
            if (d3) {
                const float4 pv = prow[0];
                const float4 qv = q4[0];
                d2 = dist2_d3(qv.x, qv.y, qv.z, pv.x, pv.y, pv.z);
            } else {
                for (int v = 0; v < nv; ++v) {
                    const float4 pv = prow[v];
                    const float4 qv = q4[v];
                    float df = qv.x - pv.x;
                    d2 = __fmaf_rn(df, df, d2);
                    df = qv.y - pv.y;
                    d2 = __fmaf_rn(df, df, d2);
                    df = qv.z - pv.z;
                    d2 = __fmaf_rn(df, df, d2);
                    df = qv.w - pv.w;
                    d2 = __fmaf_rn(df, df, d2);
                }
            }
            key = make_key(d2, p);
            acc = d2 < r2 && key < thr;
        }
        const unsigned m = __ballot_sync(0xffffffffu, acc);
        if (acc) keys[nl + __popc(m & ((1u << lane) - 1u))] = key;
        nl += __popc(m);
        __syncwarp();  // every lane is done with the staged rows and the list
        if (nl > LCAP - 32) {
            thr = coop::compact_list(keys, nl, K);
            nl = K;
        }
    }
    __syncwarp();
    coop::emit_list(keys, nl, K, r2, oidx + (q - q0), odist + (q - q0), q1 - q0);
}

template <int LCAP>
cudaError_t launch_rerank(const float* rows32, int dim, int dp, const int* lists, const int* counts, int cap,
                          int K, float r2, int* oidx, float* odist, int q0, int q1, cudaStream_t s,
                          const float* qrows32) {
    const size_t smem = (size_t)kRerankWarps * (LCAP * 8 + dp * 4 + 32 * rerank_stride(dp) * 4);
    cudaError_t e = cudaFuncSetAttribute(rerank_kernel<LCAP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    if (q1 <= q0) return cudaSuccess;
    rerank_kernel<LCAP><<<(q1 - q0 + kRerankWarps - 1) / kRerankWarps, kRerankWarps * 32, smem, s>>>(
        rows32, dim, dp, lists, counts, cap, K, r2, oidx, odist, q0, q1, qrows32);
    return cudaGetLastError();
}

template <int KC>
cudaError_t launch_filter_kc(const uint8_t* tiles, const float* qa, const float* pb, int n, int ntiles,
                             int cap, int* lists, int* counts, int* overflow, int* n_overflow, int* err,
                             int qb_begin, int qb_end, cudaStream_t s, const uint8_t* qtiles, int skip_tile,
                             int sym, bool sym_part) {
    const size_t smem = Cfg<KC>::kSmem;
    cudaError_t e =
        cudaFuncSetAttribute(filter_kernel<KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (qb_end <= qb_begin) return cudaSuccess;
    filter_kernel<KC><<<(qb_end - qb_begin + 1) / 2, kThreads, smem, s>>>(
        tiles, qa, pb, n, ntiles, cap, lists, counts, overflow, n_overflow, err, qb_begin, qb_end, qtiles,
        skip_tile, sym);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // a whole symmetric search lists its overflows here; a sharded one only
    // once its queries' candidates from the other ranks are in (tc_pull)
    if (sym && !sym_part) sym_overflow_kernel<<<(n + 255) / 256, 256, 0, s>>>(counts, 0, n, cap, overflow, n_overflow);
    return cudaGetLastError();
}

}  // namespace
}  // namespace tc

int tc_kc(int dim) { return dim <= 64 ? 1 : 2; }
size_t tc_tile_bytes(int dim) { return (size_t)tc_kc(dim) * tc::kAtomBytes; }
int tc_row_floats(int dim) { return (dim + 3) / 4 * 4; }
int tc_list_cap(int K) { return 4 * K > 256 ? 4 * K : 256; }

cudaError_t launch_tc_box(const float* pts, int n, int dim, float* box, int* nonfinite, cudaStream_t s) {
    unsigned* keys = reinterpret_cast<unsigned*>(box);
    tc::box_init_kernel<<<1, 128, 0, s>>>(keys, dim);
    const dim3 grid((unsigned)((n + tc::kBoxChunk - 1) / tc::kBoxChunk), (unsigned)dim);
    tc::dim_box_kernel<<<grid, 256, 0, s>>>(pts, n, keys, nonfinite);
    tc::box_final_kernel<<<1, 256, 0, s>>>(keys, dim);
    return cudaGetLastError();
}

cudaError_t launch_tc_prep(const float* pts, int n, int dim, const float* center, float scale,
                           float one_minus_alpha, float eta_c, float rc, uint8_t* tiles, float* rows32,
                           float* qa, float* pb, cudaStream_t s) {
    const int npad = (n + tc::kRows - 1) / tc::kRows * tc::kRows;
    tc::prep_kernel<<<npad / 128, 128, 0, s>>>(pts, n, dim, npad, tc_kc(dim), center, scale, one_minus_alpha,
                                               eta_c, rc, tiles, rows32, tc_row_floats(dim), qa, pb);
    return cudaGetLastError();
}

cudaError_t launch_tc_filter(const uint8_t* tiles, const float* qa, const float* pb, int n, int dim,
                             int cap, int* lists, int* counts, int* overflow, int* n_overflow, int* err,
                             int qb_begin, int qb_end, cudaStream_t s, const uint8_t* qtiles, int m,
                             int skip_tile, bool sym, bool sym_part) {
    const int ntiles = (n + tc::kRows - 1) / tc::kRows;
    const int qtiles_n = qtiles ? (m + tc::kRows - 1) / tc::kRows : ntiles;
    if (qb_begin < 0 || qb_end > qtiles_n) return cudaErrorInvalidValue;
    // symmetric filtering: a self-search; a part of one only when sharded
    if (sym_part && !sym) return cudaErrorInvalidValue;
    if (sym && (qtiles || (!sym_part && (qb_begin != 0 || qb_end != ntiles)))) return cudaErrorInvalidValue;
    if (!qtiles) {
        qtiles = tiles;
        m = n;
    }
    if (tc_kc(dim) == 1)
        return tc::launch_filter_kc<1>(tiles, qa, pb, m, ntiles, cap, lists, counts, overflow, n_overflow, err,
                                       qb_begin, qb_end, s, qtiles, skip_tile, sym ? 1 : 0, sym_part);
    return tc::launch_filter_kc<2>(tiles, qa, pb, m, ntiles, cap, lists, counts, overflow, n_overflow, err,
                                   qb_begin, qb_end, s, qtiles, skip_tile, sym ? 1 : 0, sym_part);
}

cudaError_t launch_tc_pull(const TcPeers& peers, int self, int* counts, int* lists, int q0, int q1, int cap,
                           cudaStream_t s) {
    if (q1 <= q0) return cudaSuccess;
    if (peers.n < 1 || peers.n > kTcMaxPeers || self < 0 || self >= peers.n) return cudaErrorInvalidValue;
    const long long threads = (long long)(q1 - q0) * 32;
    tc::tc_pull_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(peers, self, counts, lists, q0, q1, cap);
    return cudaGetLastError();
}

cudaError_t launch_tc_sym_overflow(const int* counts, int q0, int q1, int cap, int* overflow, int* n_overflow,
                                   cudaStream_t s) {
    if (q1 <= q0) return cudaSuccess;
    tc::sym_overflow_kernel<<<(q1 - q0 + 255) / 256, 256, 0, s>>>(counts, q0, q1, cap, overflow, n_overflow);
    return cudaGetLastError();
}

cudaError_t launch_tc_rerank(const float* rows32, int dim, const int* lists, const int* counts, int cap,
                             int n, int K, float r2, int* oidx, float* odist, int q0, int q1,
                             cudaStream_t s, const float* qrows32) {
    if (q0 < 0 || q1 > n) return cudaErrorInvalidValue;
    if (!qrows32) qrows32 = rows32;
    const int dp = tc_row_floats(dim);
    const int lcap = coop::list_cap(K);
    if (lcap == 64) return tc::launch_rerank<64>(rows32, dim, dp, lists, counts, cap, K, r2, oidx, odist, q0, q1, s, qrows32);
    if (lcap == 128) return tc::launch_rerank<128>(rows32, dim, dp, lists, counts, cap, K, r2, oidx, odist, q0, q1, s, qrows32);
    return tc::launch_rerank<256>(rows32, dim, dp, lists, counts, cap, K, r2, oidx, odist, q0, q1, s, qrows32);
}

}  // namespace frnn
