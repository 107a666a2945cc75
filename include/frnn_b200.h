/*
 * frnn_b200.h -- C ABI of the B200 fixed-radius nearest-neighbour engine.
 *
 * Drop-in boundary for the reference engine DebuRatnam/Pure_CUDA-C-_FRNN:
 * its Python class frnn_cuda.FRNNEngine (python_interface/nanobind_module.cu:8-21)
 * is a thin binding over the C++ class FRNNEngine (python_interface/frnn_engine.h:9-55).
 * Each entry point below replaces one member of that class; the Python module
 * frnn_cuda in this repository binds these symbols with ctypes.
 *
 * Semantics kept from the reference:
 *   - input points are float32, SoA p[d*N + i] on the device path (grid.h:26-30),
 *     row-major AoS on the host path (frnn_engine.cu:108-116);
 *   - self-query: every point is a query against all points (self included);
 *   - a neighbour of q is any point with squared distance d2 < radius*radius
 *     (strict), at most K of them, the K smallest;
 *   - outputs are int32 indices padded with -1 and float32 squared distances
 *     padded with radius*radius; device results are SoA out[k*N + q]
 *     (find_nbrs.cu:206-213), host results of frnn_search row-major [q*K + k];
 *   - limits K <= 128 and D <= 128 (grid.h:59-60);
 *   - returned device pointers are engine-owned and stay valid until the next
 *     search call on the same engine (frnn_engine.cu:248-249).
 *
 * Differences from the reference:
 *   - the K slots of a query are returned in ascending (d2, index) order and
 *     ties at equal d2 are broken by the smaller index, so results are a
 *     deterministic function of the input (the reference returns heap order
 *     and breaks ties by nondeterministic visit order);
 *   - points need not lie in [0,1)^D: the grid is built on the data's bounding
 *     box (the reference drops points outside [0,1), insert_points.cu:74-87);
 *   - every entry returns an int status instead of failing silently.
 *
 * Threading: one engine is not re-entrant; use one engine per host thread.
 */
#ifndef FRNN_B200_H
#define FRNN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct frnn_engine frnn_engine;

/* Status codes returned by every entry point. */
enum frnn_status {
    FRNN_OK = 0,
    FRNN_ERR_INVALID_ARG = 1,  /* bad N / dim / K / radius / pointer            */
    FRNN_ERR_OOM = 2,          /* device or pinned-host allocation failed        */
    FRNN_ERR_CUDA = 3,         /* a CUDA runtime call or kernel launch failed    */
    FRNN_ERR_TIMEOUT = 4,      /* a bounded device wait gave up (scan lookback)  */
    FRNN_ERR_NO_DEVICE = 5,    /* no usable sm_100 device                        */
    FRNN_ERR_STATE = 6,        /* call order violated (e.g. results before search) */
    FRNN_ERR_COMM = 7          /* a collective of the sharded search failed       */
};

/* Search paths (frnn_engine.cu:215-246 chooses among the reference's three). */
enum frnn_path {
    FRNN_PATH_AUTO = 0,        /* dispatcher decides                              */
    FRNN_PATH_GRID = 1,        /* uniform grid on the leading min(D,4) axes,      *
                                * full-D ranking (full-D grid when D <= 3)         */
    FRNN_PATH_BRUTE = 2,       /* tiled brute force, SIMT fp32                    */
    FRNN_PATH_BRUTE_TC = 3     /* brute force with a tcgen05 fp16 distance filter *
                                * and exact fp32 re-rank; same results as         *
                                * FRNN_PATH_BRUTE.  The dispatcher takes it for   *
                                * D > 32 and N >= 1024                            */
};

/* Constructor.  Replaces FRNNEngine::FRNNEngine(int max_points)
 * (python_interface/frnn_engine.h:11, frnn_engine.cu:23-46).  device = -1
 * selects the current CUDA device.  Scratch grows lazily with N, D and K. */
int frnn_create(int max_points, int device, frnn_engine** out);

/* Destructor.  Replaces FRNNEngine::~FRNNEngine (frnn_engine.cu:48-55). */
int frnn_destroy(frnn_engine* e);

/* Device path.  Replaces FRNNEngine::search_gpu(uintptr_t dev_ptr, int N,
 * int dim, int K, float radius) (frnn_engine.h:24-26, frnn_engine.cu:195-250).
 * d_points_soa: caller-owned device memory, SoA [d*N + i], N <= max_points.
 * On return *d_idxs / *d_dists point at engine-owned SoA results [k*N + q];
 * the call is blocking like the reference's (its launchers synchronise). */
int frnn_search_gpu(frnn_engine* e, const float* d_points_soa, int N, int dim, int K,
                    float radius, int** d_idxs, float** d_dists);

/* Host path.  Replaces FRNNEngine::search(std::vector<float> points_raw, int K,
 * float radius) (frnn_engine.h:15-19, frnn_engine.cu:104-193).
 * h_points_aos holds count floats, row-major (N, dim) with N = max_points and
 * dim = count / max_points (frnn_engine.cu:108).  h_idxs / h_dists receive
 * N*K values row-major [q*K + k]. */
int frnn_search(frnn_engine* e, const float* h_points_aos, int64_t count, int K, float radius,
                int* h_idxs, float* h_dists);

/* Replaces FRNNEngine::get_results(int N, int K) (frnn_engine.h:30,
 * frnn_engine.cu:252-258): copies the last results device->host in SoA order
 * [k*N + q].  N and K must match the last search. */
int frnn_get_results(frnn_engine* e, int N, int K, int* h_idxs, float* h_dists);

/* ---- additions with no reference counterpart ---------------------------- */

/* Human-readable text for a status code / the engine's last error. */
const char* frnn_status_string(int status);
const char* frnn_last_error(const frnn_engine* e);

/* Run the engine's work on a caller stream (cudaStream_t; 0 = legacy default
 * stream, the reference's behaviour and the default). */
int frnn_set_stream(frnn_engine* e, void* stream);

/* Force a search path (FRNN_PATH_*); FRNN_PATH_AUTO restores the dispatcher. */
int frnn_set_path(frnn_engine* e, int path);

/* Path taken by the last search and the grid it used (grid_dims = 0 for brute
 * force; cells = number of dense cells). */
int frnn_last_plan(const frnn_engine* e, int* path, int* grid_dims, int64_t* cells);

/* Same as frnn_search_gpu but does not wait for the device: results are
 * ready when the engine's stream reaches this point. */
int frnn_search_gpu_async(frnn_engine* e, const float* d_points_soa, int N, int dim, int K,
                          float radius, int** d_idxs, float** d_dists);

/* Search a separate query set: every one of the M queries (SoA
 * d_queries_soa[d*M + q]) against the N points (SoA, N <= max_points), the
 * same acceptance, ordering, padding and arithmetic as frnn_search_gpu, with
 * no self-match (a query is not one of the points).  Results SoA
 * [k*M + q] in engine-owned buffers; frnn_get_results(e, M, K) copies them.
 * No counterpart in the reference engine, which self-queries only
 * (python_interface/frnn_engine.cu:195-250); its kernels assume the query set
 * is the point set (find_nbrs.cu:197,325,338).  Blocking. */
int frnn_search_gpu_queries(frnn_engine* e, const float* d_points_soa, int N, const float* d_queries_soa, int M,
                            int dim, int K, float radius, int** d_idxs, float** d_dists);

/* Grid reuse: build once, query many.  frnn_build_grid plans and builds the
 * search structure for N points and a radius (on the grid path: the cell
 * plan, principal axes if chosen, and the cell-sorted points); every
 * frnn_query_grid call then searches a query set (SoA d_queries_soa[d*M + q],
 * the points' dim) against it with its own K, exactly like
 * frnn_search_gpu_queries, without rebuilding.  On the brute-force paths
 * nothing is built and each query call reads the points again, so they must
 * stay valid; the grid path does not read them after the build.  Any other
 * search on the engine (frnn_search_gpu, _queries, _part, frnn_search)
 * discards the built grid; frnn_query_grid then returns FRNN_ERR_STATE.  Results
 * SoA [k*M + q] in engine-owned buffers; frnn_get_results(e, M, K) copies them.
 * No counterpart in the reference engine, which rebuilds its grid on every
 * search (python_interface/frnn_engine.cu:195-250).  Blocking. */
int frnn_build_grid(frnn_engine* e, const float* d_points_soa, int N, int dim, float radius);
int frnn_query_grid(frnn_engine* e, const float* d_queries_soa, int M, int K, int** d_idxs, float** d_dists);

/* Part of a search, for sharding the queries of one cloud over several
 * engines (one per GPU).  No counterpart in the reference, whose engine only
 * searches whole clouds (python_interface/frnn_engine.cu:195-250); queries
 * are independent, so its search splits over GPUs by query.  Every part
 * sees all N points; part `part` of `nparts` searches one contiguous slice of
 * the engine's query order (cell order on the grid path, input order on brute
 * force, whole 128-query tiles on the tensor-core path), and the slices of
 * parts 0..nparts-1 cover every query exactly once when every part is given
 * the same points, N, dim, K, radius and path.  On return *n_rows is the
 * slice's size and the engine-owned device arrays hold
 *   d_row_ids[j]                original index of the query of row j,
 *   d_idxs[k*n_rows + j],       its k-th neighbour (ascending (d2, index),
 *   d_dists[k*n_rows + j]       padding (-1, r^2)), exactly as the whole
 *                               search would report it.
 * Blocking, like frnn_search_gpu.  frnn_get_results does not read parts. */
int frnn_search_gpu_part(frnn_engine* e, const float* d_points_soa, int N, int dim, int K, float radius,
                         int part, int nparts, int* n_rows, int** d_row_ids, int** d_idxs,
                         float** d_dists);

/* Host path with caller-provided pinned or pageable buffers in the device
 * layouts: h_points_soa [d*N + i] in, SoA results [k*N + q] out.  The copies
 * run on the engine stream; used for end-to-end timing. */
int frnn_search_host_soa(frnn_engine* e, const float* h_points_soa, int N, int dim, int K,
                         float radius, int* h_idxs, float* h_dists);

/* Tuning options (frnn_set_option). */
enum frnn_option {
    /* D = 3 searches with K > 32: result sets up to this many bytes (N*K*8)
     * are written straight to original query order from the search kernel;
     * larger ones are written in cell order and unpermuted one output row at
     * a time.  Default 48 MiB.  Other searches always write directly. */
    FRNN_OPT_DIRECT_OUTPUT_MAX_BYTES = 1,
    /* Grid axes for D > 4 (FRNN_GRID_AXES_*).  The reference grids the first
     * coordinates (python_interface/frnn_engine.cu:64-102); the engine may
     * instead grid the data's principal axes (up to 6), which finds the same
     * neighbours with fewer candidates on correlated data.  Default AUTO: a
     * sampled estimate of candidates per query decides. */
    FRNN_OPT_GRID_AXES = 2,
    /* Grid searches with D != 3 and K <= 32 (FRNN_LIST_SEARCH_*): the list
     * search (one thread per query appends every in-radius key to its own
     * list, then a register sort emits the K smallest in original order, as
     * for D = 3) or the warp-cooperative search.  Default AUTO: the list
     * search for D <= 12.  No reference counterpart. */
    FRNN_OPT_LIST_SEARCH = 3,
    /* Tests of the timeout path only (FRNN_TEST_STALL_*): make one bounded
     * device wait run out on purpose, so a test can check that the search
     * returns FRNN_ERR_TIMEOUT and that the engine's next search succeeds.
     * SCAN: one tile of the grid's prefix scan (the cell-count scan that
     * replaces the reference's thrust::exclusive_scan, frnn_engine.cu:91-94)
     * never publishes its status, so the next tile's look-back gives up
     * after its poll limit.  TC_FILTER: the tensor-core filter's producer
     * never copies one point tile, so the MMA thread's wait for it gives up
     * after 2 s.  Results of a stalled search are undefined; nothing is
     * written outside the engine's buffers.  Default OFF. */
    FRNN_OPT_TEST_STALL = 4,
    /* Blocking self-searches with D <= 4 on the grid (frnn_search_gpu and the
     * host entry points): 1 (default) plans the grid on the GPU -- the
     * bounding-box kernel runs the host planner's own code and every later
     * kernel reads the plan from device memory, so no host round trip
     * separates the box from the build and the search; 0 reads the box back
     * and plans on the host, as the reference does (frnn_engine.cu:64-86,
     * 142-156).  Results are the same either way.  No reference counterpart. */
    FRNN_OPT_DEVICE_PLAN = 5,
    /* Whole self-searches on the tensor-core path: 1 (default) filters each
     * unordered pair of 128-point tiles once and appends every passing pair
     * to both points' candidate lists (the distance is symmetric), half the
     * MMAs of the all-pairs filter; 0 filters every (query tile, point tile)
     * pair, as the reference's brute force visits every pair
     * (no_grid_frnn.cu:121-326).  Results are the same either way.  No
     * reference counterpart. */
    FRNN_OPT_TC_SYMMETRIC = 6
};
enum frnn_test_stall {
    FRNN_TEST_STALL_OFF = 0,
    FRNN_TEST_STALL_SCAN = 1,      /* needs a grid of more than 8,192 cells   */
    FRNN_TEST_STALL_TC_FILTER = 2  /* needs more than 128 points              */
};
enum frnn_list_search {
    FRNN_LIST_SEARCH_AUTO = 0,     /* list search for D <= 12               */
    FRNN_LIST_SEARCH_ALWAYS = 1,   /* list search for every D != 3          */
    FRNN_LIST_SEARCH_NEVER = 2     /* warp-cooperative search for D != 3    */
};
enum frnn_grid_axes {
    FRNN_GRID_AXES_AUTO = 0,       /* cheaper of the two by the estimate    */
    FRNN_GRID_AXES_LEADING = 1,    /* leading min(D, 4) coordinates only     */
    FRNN_GRID_AXES_PRINCIPAL = 2   /* principal axes whenever D > 4          */
};
int frnn_set_option(frnn_engine* e, int option, int64_t value);

/* Axes of the last search's grid: FRNN_GRID_AXES_LEADING (also for searches
 * that used no grid) or FRNN_GRID_AXES_PRINCIPAL.  No reference counterpart. */
int frnn_last_grid_axes(const frnn_engine* e, int* axes);

/* Per-stage device timing.  When enabled, each search records CUDA events
 * around its stages on the engine stream; frnn_last_stage_times writes the
 * last search's milliseconds for stages 0..n-1 (0 bounding box, 1 cell
 * histogram, 2 prefix scan, 3 scatter, 4 neighbour search, 5 unpermute,
 * 6 brute force, 7 candidate collection and 8 list emit -- stages 7 and 8
 * replace 4 and 5 for D = 3 with K <= 32 -- and, on FRNN_PATH_BRUTE_TC,
 * 0 the per-dimension box, 9 prep, 10 tensor-core filter, 11 exact re-rank, with 6 timing the
 * brute-force pass over queries whose candidate list overflowed), -1 for
 * stages that did not run. */
int frnn_set_timing(frnn_engine* e, int enable);
int frnn_last_stage_times(frnn_engine* e, float* ms, int n);

/* Number of kernels this engine has launched since it was created. */
int frnn_launch_count(const frnn_engine* e, int64_t* n);

/* Queries of the last whole search (frnn_search_gpu, _async once finished,
 * _queries, frnn_query_grid, frnn_search, frnn_search_host_soa) whose
 * candidate list overflowed its capacity and which a fallback pass searched
 * again (the grid list search keeps up to 64 or 128 in-radius keys per query;
 * the tensor-core filter up to max(4K, 256) candidates).  *count receives
 * their number; the first min(*count, max_ids) original query indices go to
 * h_query_ids (any order).  Searches without candidate lists report 0.
 * FRNN_ERR_STATE when no whole search has finished.  No reference
 * counterpart (its heaps never overflow: they keep K entries). */
int frnn_last_overflow(frnn_engine* e, int* count, int* h_query_ids, int max_ids);

/* ---- query-sharded search over the GPUs of a node ----------------------
 *
 * One cloud, searched by several engines (one process per GPU), each taking
 * a slice of the queries; results gathered on one rank.  No counterpart in the
 * reference, whose engine searches a cloud on one GPU
 * (python_interface/frnn_engine.cu:195-250): queries are independent and the
 * point set is read-only, so that search splits by query.  The ranks are
 * joined by an NCCL communicator (NVLink / NVSwitch); NCCL is loaded at the
 * first call of frnn_shard_unique_id or frnn_shard_create (the process's own
 * libnccl.so.2 when one is already loaded).
 *
 * Per call of frnn_search_sharded (every rank calls it, with the same root,
 * N, dim, K and radius): the root plans and builds the search structure once
 * (on the grid path the cell-sorted rows, their ids and the cell starts),
 * gives every rank one range of original query indices of equal estimated
 * work, and broadcasts the plan and the structure (the cloud itself on the
 * brute-force paths); every rank searches its queries in cell order and
 * copies its rows -- one contiguous column block -- into the root's result
 * buffers over NVLink with the copy engines (CUDA IPC mappings); the root's
 * results -- [k*N + q], the same values as frnn_search_gpu on the whole cloud
 * -- are returned in shard-owned device buffers valid until the next call.  Host waits are bounded by the shard's timeout (default 120 s):
 * FRNN_ERR_TIMEOUT when a rank does not take part, FRNN_ERR_COMM when NCCL
 * reports an error; after either the shard is unusable (FRNN_ERR_STATE).  An
 * error on one rank before the data exchange (bad arguments, allocation) is
 * returned by every rank.  Blocking. */
typedef struct frnn_shard frnn_shard;
#define FRNN_SHARD_ID_BYTES 128

/* A new id for one shard group (an NCCL unique id): call on one rank and pass
 * the FRNN_SHARD_ID_BYTES bytes to every rank over any host channel. */
int frnn_shard_unique_id(unsigned char* id_out);

/* Join rank `rank` of `nranks` (collective: every rank calls it with the same
 * id).  The engine (on this process's GPU) does the rank's work; it stays
 * usable for ordinary searches, which discard nothing the shard needs. */
int frnn_shard_create(frnn_engine* e, int nranks, int rank, const unsigned char* id, frnn_shard** out);
int frnn_shard_destroy(frnn_shard* sh);
int frnn_shard_set_timeout(frnn_shard* sh, double seconds);

/* Tuning of the gather (frnn_shard_set_option). */
enum frnn_shard_option {
    /* Chunks a rank's queries are searched in (1..8, default 1): each
     * finished chunk is copied into the root's results while the next one is
     * searched.  Chunks are at least 65,536 queries. */
    FRNN_SHARD_OPT_CHUNKS = 1,
    /* 1: the gather's stream gets the device's highest priority; 0 (default)
     * normal priority. */
    FRNN_SHARD_OPT_COMM_PRIORITY = 2,
    /* Tensor-core path with 2..8 ranks: 1 (default) shares the symmetric
     * filter (each unordered pair of tiles once; rank r filters its query
     * blocks against the tiles at or above them and keeps every passing
     * pair, then pulls the entries the other ranks listed for its own
     * queries over NVLink); 0 filters each rank's query tiles against every
     * point tile.  Results are the same either way.  No reference
     * counterpart. */
    FRNN_SHARD_OPT_TC_SYMMETRIC = 3
};
int frnn_shard_set_option(frnn_shard* sh, int option, int64_t value);

/* The sharded search.  d_points_soa: the root's cloud (SoA [d*N + i], device
 * memory on the root's GPU); ignored on the other ranks.  On the root
 * *d_idxs / *d_dists receive the [K, N] results; elsewhere NULL. */
int frnn_search_sharded(frnn_shard* sh, int root, const float* d_points_soa, int N, int dim, int K,
                        float radius, int** d_idxs, float** d_dists);

/* The last sharded call on this rank: device milliseconds of its stages
 * (0 root plan and build, 1 header and status exchange, 2 data broadcast,
 * 3 the rank's search, chunk by chunk, 4 its copies into the root's results,
 * which overlap stage 3 when there are several chunks; -1 when not run or
 * timing is off, see frnn_set_timing on the engine), the bytes this rank
 * broadcast or received and copied or gathered, and its number of queries. */
int frnn_shard_last_stats(frnn_shard* sh, float* stage_ms, int n, int64_t* bcast_bytes, int64_t* gather_bytes,
                          int* rows);

/* The partition the root applies (host code, no GPU): bucket t of the
 * original query indices starts at index tile_start[t] (ascending) and
 * carries tile_work[t] units of estimated work; bounds[0..nparts] receive the
 * cut points, each a bucket start (or N) nearest to the r/nparts quantile of
 * the cumulative work; rank r owns [bounds[r], bounds[r+1]), possibly empty. */
int frnn_shard_partition(const uint64_t* tile_work, const int* tile_start, int64_t tiles, int N, int nparts,
                         int* bounds);

/* The partition of a sharded tensor-core search that shares the symmetric
 * filter (FRNN_SHARD_OPT_TC_SYMMETRIC, host code, no GPU): query block b
 * (128 queries) filters the ceil(N/128) - b point tiles at or above it, plus
 * about 0.35 tile's worth of re-rank, and bounds[0..nparts] cut the blocks,
 * in pairs (multiples of 256 queries, or N), into equal shares of that work;
 * rank r owns [bounds[r], bounds[r+1]).  The reference's brute force runs
 * on one GPU (no_grid_frnn.cu:121-326); no counterpart. */
int frnn_shard_tc_partition(int N, int nparts, int* bounds);

/* Allocation-free search.  No counterpart in the reference: it is for callers
 * that cannot allocate device memory while they search (a framework whose own
 * pool owns all device memory, a real-time loop with a fixed budget, code that
 * must avoid the implicit synchronisation of cudaMalloc/cudaFree).  No engine
 * object: the caller passes SoA points d_points_soa [d*N + i] and two
 * caller-owned device buffers of K*N elements that receive the same SoA
 * results [k*N + q] as frnn_search_gpu.  Scratch comes from one fixed device
 * array inside the library (8.75 MiB, held on every GPU that loads the library
 * until exit); nothing is allocated.  Limits: N <= 65,536, 1 <= dim <= 16,
 * K <= 128; larger inputs return FRNN_ERR_INVALID_ARG.  All calls on a device
 * share that array, so calls that overlap on the GPU race: serialise them.
 * The first call on a device looks up the array's address; make it before any
 * stream capture.  Runs on `stream` (0 = legacy default) and waits for it. */
int frnn_search_gpu_noalloc(const float* d_points_soa, int N, int dim, int K, float radius,
                            int* d_idx_out, float* d_dist_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FRNN_B200_H */
