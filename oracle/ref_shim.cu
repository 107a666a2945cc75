// ref_shim.cu -- C-ABI wrapper around the reference's FRNNEngine class.
//
// TEST INFRASTRUCTURE ONLY.  Compiled together with the reference's own
// sources (python_interface/frnn_engine.cu, frnn/csrc/grid/insert_points.cu,
// frnn/csrc/grid/find_nbrs.cu, frnn/csrc/no_grid_frnn/no_grid_frnn.cu) into
// oracle/_ref/libfrnn_ref.so by oracle/Makefile.  It stands in for the
// reference's nanobind module (python_interface/nanobind_module.cu:8-21),
// exposing the same three methods with plain pointers so ctypes can call them.
//
// Only memory-safe uses are exposed: search_gpu takes a caller-owned device
// pointer (the reference's own search() overflows its 32-dim staging buffer
// for D > 32, frnn_engine.cu:26-27 and :117, so it is offered only for D <= 32).

#include <cstdint>
#include <cstring>
#include <vector>
#include <cuda_runtime.h>
#include "frnn_engine.h"

extern "C" {

void* ref_create(int max_points) {
    if (max_points <= 0) return nullptr;
    return new FRNNEngine(max_points);
}

void ref_destroy(void* e) { delete static_cast<FRNNEngine*>(e); }

// FRNNEngine::search_gpu (frnn_engine.cu:195-250).  Returns the engine-owned
// device pointers through idx_ptr / dist_ptr.
int ref_search_gpu(void* e, const float* d_points_soa, int N, int dim, int K, float radius,
                   uintptr_t* idx_ptr, uintptr_t* dist_ptr) {
    if (!e || !d_points_soa || N <= 0 || dim <= 0 || dim > 128 || K <= 0 || K > 128) return 1;
    auto r = static_cast<FRNNEngine*>(e)->search_gpu(reinterpret_cast<uintptr_t>(d_points_soa),
                                                     N, dim, K, radius);
    // The D=3 path returns before its last kernel finishes (frnn_engine.cu:240
    // launches ScatterToOrigKernel without a synchronize); wait for it here so
    // the caller reads finished results.
    cudaError_t err = cudaDeviceSynchronize();
    *idx_ptr = r.first;
    *dist_ptr = r.second;
    return err == cudaSuccess ? 0 : 3;
}

// FRNNEngine::get_results (frnn_engine.cu:252-258): SoA [k*N+q] copies.
int ref_get_results(void* e, int N, int K, int* h_idx, float* h_dist) {
    if (!e || !h_idx || !h_dist) return 1;
    auto r = static_cast<FRNNEngine*>(e)->get_results(N, K);
    std::memcpy(h_idx, r.first.data(), sizeof(int) * (size_t)N * K);
    std::memcpy(h_dist, r.second.data(), sizeof(float) * (size_t)N * K);
    return 0;
}

// FRNNEngine::search (frnn_engine.cu:104-193): flat AoS host array in,
// row-major [q*K+k] out.  N must be the engine's max_points (the reference
// derives dim = len/max_points, :108); dim > 32 is refused because the
// reference stages it in a 32-dim buffer.
int ref_search_host(void* e, const float* h_points_aos, int N, int dim, int K, float radius,
                    int* h_idx, float* h_dist) {
    if (!e || !h_points_aos || N <= 0 || dim <= 0 || dim > 32 || !h_idx || !h_dist) return 1;
    std::vector<float> pts(h_points_aos, h_points_aos + (size_t)N * dim);
    auto r = static_cast<FRNNEngine*>(e)->search(pts, K, radius);
    std::memcpy(h_idx, r.first.data(), sizeof(int) * r.first.size());
    std::memcpy(h_dist, r.second.data(), sizeof(float) * r.second.size());
    cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? 0 : 3;
}

}  // extern "C"
