// engine_noalloc.cu -- frnn_search_gpu_noalloc: a search that allocates nothing.
//
// Some callers cannot call cudaMalloc while they search: a framework that owns
// all device memory through its own pool and forbids allocations outside it,
// a real-time loop with a fixed memory budget, or a process that must not
// trigger the implicit synchronisation of cudaMalloc/cudaFree between frames.
// For them this entry point runs the engine's grid search (or, for small
// inputs, its brute force) with every piece of scratch taken from one
// file-scope device array instead of engine-owned allocations.  The caller
// passes the points and the two result buffers.
//
// Limits: N <= 65,536 points, 1 <= dim <= 16, 1 <= K <= 128, at most 2^19 grid
// cells (a coarser grid is chosen when the data would need more; the results
// are the same, only the work grows).  The array is 9,179,648 bytes (8.75 MiB) and every GPU
// on which the library is loaded holds it until the process exits.
//
// The array is shared by every call on a device and keeps what the last call
// left there; everything a call needs zeroed is cleared by that call.  Calls
// that overlap on a GPU (other host threads, or streams that run concurrently)
// race on it: issue them one after another.
//
// The first call on a device looks the array's device address up with
// cudaGetSymbolAddress (host code only sees a host-side stand-in under the
// array's name); make that first call before any stream capture begins.
#include <cmath>
#include <cstdint>
#include <mutex>

#include "frnn_b200.h"
#include "frnn_device.cuh"
#include "frnn_internal.h"
#include "grid_plan.cuh"

using namespace frnn;

namespace {

constexpr int kMaxPoints = 65536;
constexpr int kMaxDim = 16;
constexpr long long kMaxCells = 1LL << 19;
constexpr int kBoxBlocks = 64;           // bbox_blocks(kMaxPoints, ...) never exceeds this
constexpr int kMaxDevices = 64;
constexpr double kBruteSmallWork = 4.0e8;  // same small-input rule as the engine

constexpr size_t up256(size_t x) { return (x + 255) / 256 * 256; }

// Byte offsets of the scratch pieces inside the array.
struct Layout {
    size_t box_partial, box_out, box_ticket, scan_ticket, err, status, counts, starts, cellrank,
        rows, ids, total;
};
constexpr Layout make_layout() {
    Layout L{};
    size_t o = 0;
    L.box_partial = o; o += up256((size_t)kBoxBlocks * 9 * 4);
    L.box_out = o;     o += up256(16 * 4);
    L.box_ticket = o;  o += 256;
    L.scan_ticket = o; o += 256;
    L.err = o;         o += 256;
    L.status = o;      o += up256((size_t)((kMaxCells + 4095) / 4096) * 8);
    L.counts = o;      o += up256((size_t)kMaxCells * 4);
    L.starts = o;      o += up256((size_t)(kMaxCells + 1) * 4);
    L.cellrank = o;    o += up256((size_t)kMaxPoints * 8);
    L.rows = o;        o += up256((size_t)kMaxPoints * kMaxDim * 4);
    L.ids = o;         o += up256((size_t)kMaxPoints * 4);
    L.total = o;
    return L;
}
constexpr Layout kL = make_layout();
static_assert(kL.total == 9179648, "the documented scratch size");

// The scratch.  In host code this name is a host-side stand-in, not a device
// address: the device address is obtained with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kL.total];

std::mutex g_mu;
void* g_scratch[kMaxDevices] = {};

// Device address of the scratch on the current device (looked up once).
int scratch_on(int dev, unsigned char** out) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch[dev]) {
        void* p = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess || !p) {
            cudaGetLastError();
            return FRNN_ERR_CUDA;
        }
        g_scratch[dev] = p;
    }
    *out = static_cast<unsigned char*>(g_scratch[dev]);
    return FRNN_OK;
}

bool device_buffer(const void* p, int dev) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (a.type == cudaMemoryTypeManaged) return true;
    return a.type == cudaMemoryTypeDevice && a.device == dev;
}

// Grid on the leading min(dim, 4) axes over the bounding box: the engine's own
// planner (grid_plan.cuh) with the table capped at kMaxCells cells.
bool plan(const float* box, int N, int dim, float radius, GridPlan& P) {
    return plan_grid(box, dim <= 4 ? dim : 4, N, dim, radius, 0.0, kMaxCells, P);
}

#define NA_CHECK(call)                                  \
    do {                                                \
        if ((call) != cudaSuccess) {                    \
            cudaGetLastError();                         \
            return FRNN_ERR_CUDA;                       \
        }                                               \
    } while (0)

}  // namespace

extern "C" int frnn_search_gpu_noalloc(const float* d_points_soa, int N, int dim, int K,
                                       float radius, int* d_idx_out, float* d_dist_out,
                                       void* stream) {
    if (!d_points_soa || !d_idx_out || !d_dist_out) return FRNN_ERR_INVALID_ARG;
    if (N < 1 || N > kMaxPoints || dim < 1 || dim > kMaxDim || K < 1 || K > kMaxK)
        return FRNN_ERR_INVALID_ARG;
    if (!(radius > 0.0f) || !std::isfinite(radius) || !(radius * radius > 0.0f) ||
        !std::isfinite(radius * radius))
        return FRNN_ERR_INVALID_ARG;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return FRNN_ERR_NO_DEVICE;
    }
    if (!device_buffer(d_points_soa, dev) || !device_buffer(d_idx_out, dev) ||
        !device_buffer(d_dist_out, dev))
        return FRNN_ERR_INVALID_ARG;
    unsigned char* base = nullptr;
    int st = scratch_on(dev, &base);
    if (st != FRNN_OK) return st;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float r2 = radius * radius;
    const double work = (double)N * (double)N * dim;
    GridPlan P{};
    bool grid = work > kBruteSmallWork;
    if (grid) {
        float* box_partial = reinterpret_cast<float*>(base + kL.box_partial);
        float* box_out = reinterpret_cast<float*>(base + kL.box_out);
        unsigned* box_ticket = reinterpret_cast<unsigned*>(base + kL.box_ticket);
        NA_CHECK(cudaMemsetAsync(box_ticket, 0, 4, s));
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int blocks = bbox_blocks(N, sms) < kBoxBlocks ? bbox_blocks(N, sms) : kBoxBlocks;
        NA_CHECK(launch_bbox(d_points_soa, N, dim <= 4 ? dim : 4, box_partial, box_ticket, box_out,
                             blocks, s));
        float hbox[9];
        NA_CHECK(cudaMemcpyAsync(hbox, box_out, sizeof(hbox), cudaMemcpyDeviceToHost, s));
        NA_CHECK(cudaStreamSynchronize(s));
        if (hbox[8] != 0.0f) return FRNN_ERR_INVALID_ARG;  // NaN or Inf coordinates
        grid = plan(hbox, N, dim, radius, P);
    }
    if (grid) {
        int* counts = reinterpret_cast<int*>(base + kL.counts);
        int* starts = reinterpret_cast<int*>(base + kL.starts);
        unsigned long long* status = reinterpret_cast<unsigned long long*>(base + kL.status);
        int* scan_ticket = reinterpret_cast<int*>(base + kL.scan_ticket);
        int* err = reinterpret_cast<int*>(base + kL.err);
        int2* cellrank = reinterpret_cast<int2*>(base + kL.cellrank);
        float* rows = reinterpret_cast<float*>(base + kL.rows);
        int* ids = reinterpret_cast<int*>(base + kL.ids);
        // what this call needs zeroed (earlier calls leave their contents)
        NA_CHECK(cudaMemsetAsync(counts, 0, (size_t)P.cells * 4, s));
        NA_CHECK(cudaMemsetAsync(status, 0, (size_t)scan_tiles(P.cells) * 8, s));
        NA_CHECK(cudaMemsetAsync(scan_ticket, 0, 4, s));
        NA_CHECK(cudaMemsetAsync(err, 0, 4, s));
        NA_CHECK(launch_hash_count(d_points_soa, P, counts, cellrank, s));
        NA_CHECK(launch_scan(counts, starts, P.cells, status, scan_ticket, 1u, err, s));
        NA_CHECK(launch_scatter(d_points_soa, P, cellrank, starts, rows, ids, s));
        NA_CHECK(launch_grid_search(rows, ids, starts, P, K, r2, 0, N, d_idx_out, d_dist_out, N,
                                    ids, s));
        int herr = 0;
        NA_CHECK(cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, s));
        NA_CHECK(cudaStreamSynchronize(s));
        if (herr != 0) return FRNN_ERR_TIMEOUT;
        return FRNN_OK;
    }
    NA_CHECK(launch_bruteforce(d_points_soa, N, dim, K, r2, 0, N, d_idx_out, d_dist_out, N, s));
    NA_CHECK(cudaStreamSynchronize(s));
    return FRNN_OK;
}
