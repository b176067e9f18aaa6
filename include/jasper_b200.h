/*
 * jasper_b200.h -- C ABI of the jasper_b200 graph index (B200 / sm_100a).
 *
 * Drop-in boundary for Jasper's batched Vamana beam-search path.  Each entry
 * point replaces one op of the reference's tvm_ffi module
 * (ffi/jasper_ffi_common.cuh, ffi/jasper_ffi_plain.cu); the reference config
 * id (f16_r{8,16,32,64}_{l2,ip}) becomes the (n_neighbors, metric) argument
 * pair.  All pointers are plain C pointers; no framework types cross the ABI.
 *
 * Conventions
 *   - Every function returns JB_OK (0) or a JB_ERR_* code; jb_last_error()
 *     returns the message of the calling thread's last failure.  Where the
 *     reference raised (TVM_FFI_ICHECK, std::runtime_error) or called exit(),
 *     these functions return an error instead.
 *   - Vectors are IEEE fp16 values passed as uint16_t bit patterns, row-major,
 *     `row_stride` elements between rows (>= dim).
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream).  Device
 *     calls are asynchronous on that stream unless stated otherwise.
 *   - Handles are process-wide and thread-safe to look up; one handle must not
 *     be built and searched concurrently (as in the reference).
 */
#ifndef JASPER_B200_H_
#define JASPER_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define JB_OK 0
#define JB_ERR_INVALID_ARGUMENT 1
#define JB_ERR_INVALID_HANDLE 2
#define JB_ERR_IO 3
#define JB_ERR_CUDA 4
#define JB_ERR_RUNTIME 5

#define JB_METRIC_L2 0
#define JB_METRIC_IP 1

typedef struct jb_graph_info {
  uint64_t n_vectors;
  uint64_t n_deleted;
  uint64_t next_id;
  uint32_t dim;
  uint32_t n_neighbors;
  int32_t metric;
  uint32_t medoid;
  uint32_t global_offset;
  int32_t on_host;
  int32_t device;
} jb_graph_info;

/* Message of this thread's last failing call ("" if none). */
const char* jb_last_error(void);

/* ABI revision of this header (bumped on incompatible changes). */
int jb_abi_version(void);

/* Process-wide choice of the query-search kernel (no reference counterpart;
 * results are identical either way): 0 = automatic -- one CTA of 2 warps per
 * query when a launch has fewer than 8 queries per SM (small batches, where
 * a query's latency decides the time), else one warp per query; 1 = always a
 * warp per query; 2 or more = always a CTA of 2 warps per query.  For tests
 * and tuning.  Negative values are rejected. */
int jb_search_set_warps_per_query(int32_t warps_per_query);

/* Build a graph (reference: ConstructGraph_##id, ffi/jasper_ffi_common.cuh:
 * 232-261 -> jasper::construct_graph, include/jasper/index/construct.cuh:
 * 992-1160).  `vectors` may be host (pageable or pinned) or device memory.
 * The batch cap is min(budget-derived cap, n / 50) exactly as the reference
 * computes it; where that is 0 (n < 50) one row per batch is used (the
 * reference loops forever there).  Synchronous. */
int jb_graph_construct(const uint16_t* vectors, uint64_t n, uint32_t dim, uint32_t row_stride,
                       uint32_t n_neighbors, int32_t metric, double alpha,
                       uint64_t workspace_budget_bytes, int32_t on_host, void* stream,
                       int64_t* out_handle);

/* Load a graph file written by the reference or by jb_graph_save (reference:
 * LoadGraph_##id, ffi/jasper_ffi_common.cuh:210-219 -> load_graph_from_file,
 * include/jasper/index/graph.cuh:1425-1651).  Synchronous. */
int jb_graph_load(const char* path, uint32_t dim, uint32_t n_neighbors, int32_t metric,
                  int32_t on_host, int64_t* out_handle);

/* Write the reference's on-disk layout (reference: SaveGraph_##id,
 * ffi/jasper_ffi_common.cuh:221-230 -> save_graph_to_file, graph.cuh:
 * 1653-1788).  Synchronous. */
int jb_graph_save(int64_t handle, const char* path);

/* Beam search (reference: Search_##id, ffi/jasper_ffi_common.cuh:302-369 ->
 * jasper::search, include/jasper/beam_search/api.cuh:57-73).  `queries`,
 * `out_idx` ([nq][k] int32 stable ids, -1 when fewer than k results) and
 * `out_dist` ([nq][k] f32, 1e30 when unfilled) are device pointers.
 * Asynchronous on `stream`. */
int jb_graph_search(int64_t handle, const uint16_t* queries, uint64_t n_queries,
                    uint32_t row_stride, int32_t* out_idx, float* out_dist, uint32_t k,
                    uint32_t beam_width, uint32_t limit, void* stream);

/* Same search with per-query counters (instrumentation): stats[q][0..4] =
 * expansions, sum of expanded degrees, distance evaluations, visited-table
 * resets, distinct rows evaluated (device pointer, [n_queries][5] uint32).
 * The last needs `seen_scratch`: zeroed device memory of
 * n_queries * ceil(n_vectors / 32) uint32 words (else it repeats field 2).
 * Asynchronous. */
int jb_graph_search_stats(int64_t handle, const uint16_t* queries, uint64_t n_queries,
                          uint32_t row_stride, int32_t* out_idx, float* out_dist, uint32_t k,
                          uint32_t beam_width, uint32_t limit, uint32_t* stats,
                          uint32_t* seen_scratch, void* stream);

/* End-to-end search from host buffers.  Page-locked (pinned) buffers are
 * used in place: the search kernel reads each query row from host memory
 * once and writes the results into host memory.  Pageable buffers, and
 * query rows not at the padded stride (or not 16-byte aligned), go through
 * device buffers with copies before and after the search.  Synchronous (the
 * reference's Search_ also synchronises, beam_search.cuh:330). */
int jb_graph_search_host(int64_t handle, const uint16_t* queries, uint64_t n_queries,
                         uint32_t row_stride, int32_t* out_idx, float* out_dist, uint32_t k,
                         uint32_t beam_width, uint32_t limit, void* stream);

/* Search without any device allocation.  No counterpart in the reference.
 * For callers that cannot allocate device memory while they search: code
 * that runs under a fixed, pre-reserved memory budget, code whose process
 * owns an allocator this library must not bypass, or code that may not touch
 * the CUDA allocator while other work is in flight.  Same arguments and
 * results as jb_graph_search (device pointers, asynchronous on `stream`).
 * Its scratch is a fixed 4 MiB device array inside this library, held on
 * every GPU that loads it until the process exits: the work counter, plus a
 * repacked copy of the queries when their rows are not at stride
 * ceil(dim/8)*8 with a 16-byte aligned base; a call that would need more than
 * that is rejected with JB_ERR_INVALID_ARGUMENT.  All calls share the array,
 * so calls that overlap on the GPU race.  The first call on each device looks
 * up the array's device address: make it before any stream capture. */
int jb_graph_search_noalloc(int64_t handle, const uint16_t* queries, uint64_t n_queries,
                            uint32_t row_stride, int32_t* out_idx, float* out_dist, uint32_t k,
                            uint32_t beam_width, uint32_t limit, void* stream);

/* Release a graph (reference: FreeGraph, ffi/jasper_ffi_plain.cu:15-47). */
int jb_graph_free(int64_t handle);

/* Metadata (reference: GetNumVectors / GetNumTombstoned / GetNumLive / GetDim,
 * ffi/jasper_ffi_plain.cu:49-124). */
int jb_graph_get_info(int64_t handle, jb_graph_info* out);

/* Copy the row with this stable id into `out` (dim fp16; host or device)
 * (reference: GetVector_##id, ffi/jasper_ffi_common.cuh:263-300). */
int jb_graph_get_vector(int64_t handle, int64_t stable_id, uint16_t* out);

/* Hand out `count` fresh stable ids into a host int32 array (reference:
 * ReserveIds, ffi/jasper_ffi_plain.cu:75-93). */
int jb_graph_reserve_ids(int64_t handle, int64_t count, int32_t* out_ids);

/* Soft-delete rows by id (host int32 array; out-of-range ids ignored); search
 * never returns them (reference: MarkDeleted_##id ->
 * include/jasper/index/graph_ops.cuh:93-134). */
int jb_graph_mark_deleted(int64_t handle, const int32_t* ids, uint64_t n_ids);

/* Live append (reference: Append_##id, ffi/jasper_ffi_common.cuh:411-432 ->
 * jasper::append_batch, include/jasper/index/construct.cuh:1169-1265): the
 * n rows (host or device memory, row stride `row_stride` elements) take the
 * next slots, are wired into the graph by the construction's batched search
 * and RobustPrune(alpha) in batches of min(n, 100000) rows, and receive the
 * stable ids next_id .. next_id + n - 1, written to the host int32 array
 * `out_ids` (may be NULL).  Device-resident plain graphs with global offset 0
 * only (directional, RaBitQ or prerotated graphs are rejected, as the
 * reference exports no directional append).  Synchronous on `stream`. */
int jb_graph_append(int64_t handle, const uint16_t* vectors, uint64_t n, uint32_t row_stride,
                    double alpha, int32_t* out_ids, void* stream);

/* Create a graph from rows with no edges (host or device rows). */
int jb_graph_create(const uint16_t* vectors, uint64_t n, uint32_t dim, uint32_t row_stride,
                    uint32_t n_neighbors, int32_t metric, int32_t on_host, int64_t* out_handle);

/* Replace all adjacency (host arrays [n][R] ids, [n][R] bf16 bit patterns,
 * [n] counts) and the medoid. */
int jb_graph_set_edges(int64_t handle, const uint32_t* edges, const uint16_t* edge_dists,
                       const uint8_t* counts, uint32_t medoid);

/* Read all adjacency into host arrays (same shapes as jb_graph_set_edges). */
int jb_graph_get_edges(int64_t handle, uint32_t* edges, uint16_t* edge_dists, uint8_t* counts);

/* Make this graph the id range [offset, offset + n) of a larger index: adds
 * `offset` to every stored neighbour id and to the medoid (reference:
 * graph::apply_global_offset, include/jasper/index/graph.cuh:801-827). */
int jb_graph_apply_global_offset(int64_t handle, uint32_t offset);

/* ── directional (LSH / PQ) ──────────────────────────────────────────── */

#define JB_DIR_LSH 0
#define JB_DIR_PQ 1
#define JB_DIR_RABITQ 2

/* Attach cross-polytope LSH edge payloads (host arrays): packed [n][R *
 * k_ranks] words of packed_bytes (1: 7-bit coord, 2: 15-bit coord; sign in
 * the top bit), mag_sq [n][R] bf16 bit patterns, c [k_ranks] and norm_denom
 * (reference: edge_lsh_list + lsh_globals, include/jasper/lsh/edge_lsh.cuh:
 * 9-80, lsh_globals.cuh:12-15; state kept per handle like dir_meta,
 * ffi/jasper_ffi_common.cuh:135-149). */
int jb_graph_set_lsh(int64_t handle, uint32_t k_ranks, uint32_t packed_bytes, const void* packed,
                     const uint16_t* mag_sq, const float* c, float norm_denom);

/* Attach PQ payloads (host arrays): centroids [m][256][dsub] f32, codes [n][m
 * * R] (edge e of subspace j at j * R + e), exact norms [n] f32 (reference:
 * pq_codebooks / edge_pq_list / graph::d_vector_norms,
 * include/jasper/pq/pq_codebooks.cuh, edge_pq.cuh:23-50). */
int jb_graph_set_pq(int64_t handle, uint32_t m, uint32_t dsub, const float* centroids,
                    const uint8_t* codes, const float* norms);

/* Which payloads a graph carries: bit 0 LSH, bit 1 PQ, bit 2 RaBitQ (reference:
 * jasper_get_directional_flags_<cfg>, ffi/jasper_ffi_common.cuh:760-775). */
int jb_graph_get_directional_flags(int64_t handle, int32_t* out_flags);

/* The d x d random orthogonal prerotation for `seed` as float32, column-major
 * (host memory, no GPU needed) -- the reference's set_rotation_matrix
 * (include/jasper/rotation/rotation.cuh:74-110). */
int jb_rotation_matrix(uint32_t dim, uint64_t seed, float* out);

/* Rotate n rows by the prerotation of (dim, seed): out[r] = P^T rows[r]
 * (reference: rotate_data_vec / the prerotation GEMM, rotation/rotation.cuh:
 * 122-151, index/construct.cuh:1077-1089).  `rows` and `out` are device
 * arrays [n][ceil(dim/8)*8] fp16, 16-byte aligned, pad lanes of `rows` zero.
 * use_tensor_cores = 1 runs the tcgen05 GEMM (the one builds and queries
 * use), 0 the SIMT reference GEMM.  Synchronous. */
int jb_rotate_rows(uint32_t dim, uint64_t seed, const uint16_t* rows, uint16_t* out, uint64_t n,
                   int32_t use_tensor_cores, void* stream);

/* Directional search: kind JB_DIR_LSH (reference: DirectionalSearch_##id ->
 * directional_search, ffi/jasper_ffi_common.cuh:530-609, beam_search/
 * api.cuh:118-138) or JB_DIR_PQ (PqSearch_##id -> pq_search, :611-688,
 * api.cuh:185-205).  Queries are rotated first when the graph was built with
 * prerotation.  Device pointers; unfilled slots are (0x7FFFFFFF, FLT_MAX) as
 * in the reference.  Asynchronous on `stream`. */
int jb_graph_directional_search(int64_t handle, int32_t kind, const uint16_t* queries,
                                uint64_t n_queries, uint32_t row_stride, int32_t* out_idx,
                                float* out_dist, uint32_t k, uint32_t beam_width, uint32_t limit,
                                void* stream);

/* Build a graph for directional search (reference: ConstructDirectionalGraph_
 * ##id, ffi/jasper_ffi_common.cuh:382-424).  With `prerotate` every row is
 * first rotated by the prerotation of `prerotate_seed` (construct.cuh:
 * 1019-1111) and the graph keeps the matrix to rotate queries; the caller's
 * `vectors` are left unchanged (the reference rotates them in place).
 * Synchronous. */
int jb_graph_construct_directional(const uint16_t* vectors, uint64_t n, uint32_t dim,
                                   uint32_t row_stride, uint32_t n_neighbors, int32_t metric,
                                   double alpha, uint64_t workspace_budget_bytes, int32_t on_host,
                                   int32_t prerotate, uint64_t prerotate_seed, void* stream,
                                   int64_t* out_handle);

/* Build the LSH payloads: k_ranks-rank cross-polytope sketch of every edge
 * and the per-rank calibration from `n_samples` random edges (reference:
 * BuildLsh_##id, ffi/jasper_ffi_common.cuh:426-444 -> generate_lsh_globals +
 * populate_edge_lsh, graph.cuh:1153-1198, 1322-1370).  Synchronous. */
int jb_graph_build_lsh(int64_t handle, uint32_t k_ranks, uint64_t n_samples, uint64_t seed);

/* Build the PQ payloads: m x 256 codebooks by k-means on `n_train` sampled
 * edge residuals, every edge's m-byte code and exact row norms (reference:
 * BuildPq_##id, ffi/jasper_ffi_common.cuh:446-467 -> generate_pq_codebooks,
 * populate_edge_pq, compute_vector_norms, graph.cuh:1142-1320).
 * Synchronous. */
int jb_graph_build_pq(int64_t handle, uint32_t m, uint64_t n_train, uint32_t kmeans_iter,
                      uint64_t seed);

/* Save the base graph plus the directional trailer (reference:
 * SaveDirectionalGraph_##id -> save_directional_graph_to_file, graph.cuh:
 * 1834-1937).  Synchronous. */
int jb_graph_save_directional(int64_t handle, const char* path);

/* Load a graph and its directional trailer, if any (reference:
 * LoadDirectionalGraph_##id -> load_directional_graph_from_file, graph.cuh:
 * 1939-2090).  `k_ranks` must match the file's LSH rank count / PQ
 * subquantizer count; `prerotate` / `prerotate_seed` must match the build,
 * as in the reference (they are not stored in the file).  Synchronous. */
int jb_graph_load_directional(const char* path, uint32_t dim, uint32_t n_neighbors,
                              int32_t metric, uint32_t k_ranks, int32_t on_host,
                              int32_t prerotate, uint64_t prerotate_seed, int64_t* out_handle);

/* Read the LSH payloads back into host arrays (shapes of jb_graph_set_lsh;
 * c gets k_ranks floats).  The reference's counterpart is its debug dump
 * (graph::dump_edge_lsh, graph.cuh:1372-1423).  Synchronous. */
int jb_graph_get_lsh(int64_t handle, uint32_t* out_k_ranks, uint32_t* out_packed_bytes,
                     void* packed, uint16_t* mag_sq, float* c, float* norm_denom);

/* Read the PQ payloads back into host arrays (shapes of jb_graph_set_pq).
 * Any output pointer may be NULL to skip it.  Synchronous. */
int jb_graph_get_pq(int64_t handle, uint32_t* out_m, uint32_t* out_dsub, float* centroids,
                    uint8_t* codes, float* norms);

/* ── RaBitQ (1 bit per dimension) ────────────────────────────────────── */

/* The reference's quantizer rabitq_quantize<1> (include/jasper/rabitq/
 * quantize.cuh:296-353): rows [n][dim] f32, rotation (dim x dim f32
 * column-major; NULL = identity; rows are rotated by P^T and the centroid by
 * P, as the reference does), centroid [dim] f32, metric -> out: n nodes of
 * ceil(dim/8) code bytes padded to 4, then f_add and f_rescale (f32)
 * (rabitq/layout.cuh:42-116).  Device pointers; asynchronous on `stream`. */
int jb_rabitq_quantize(const float* rows, uint64_t n, uint32_t dim, const float* rotation,
                       const float* centroid, int32_t metric, uint8_t* out, void* stream);

/* RaBitQ codes of the graph's own rows (prerotated when the graph was built
 * with prerotation) around their column mean, plus each row's estimate error
 * scale; enables jb_graph_search_rabitq.  No reference counterpart: the
 * reference quantizes but has no RaBitQ search.  Synchronous. */
int jb_graph_build_rabitq(int64_t handle);

/* The beam search with exact distances (as jb_graph_search; queries are
 * prerotated when the graph is) plus a RaBitQ candidate filter: while the
 * beam is full, a new neighbour whose estimate minus margin * |q - c| *
 * err(v) exceeds the beam's worst exact distance is skipped without reading
 * its row.  margin = 1 keeps the exact search's recall in our tests; larger
 * is more conservative.  Device pointers; unfilled slots (-1, 1e30); stats as
 * jb_graph_search_stats (NULL for none).  jb_graph_directional_search with
 * kind JB_DIR_RABITQ runs this with margin 1.  Asynchronous. */
int jb_graph_search_rabitq(int64_t handle, const uint16_t* queries, uint64_t n_queries,
                           uint32_t row_stride, int32_t* out_idx, float* out_dist, uint32_t k,
                           uint32_t beam_width, uint32_t limit, float margin, uint32_t* stats,
                           void* stream);

/* Each row's estimate error scale [n] f32 (host or device). */
int jb_graph_get_rabitq_err(int64_t handle, float* err);

/* Attach / read RaBitQ payloads (host arrays): store [n][node_bytes] as
 * jb_rabitq_quantize writes it, centroid [dim] f32.  Either output pointer
 * of the getter may be NULL. */
int jb_graph_set_rabitq(int64_t handle, uint32_t node_bytes, const uint8_t* store,
                        const float* centroid);
int jb_graph_get_rabitq(int64_t handle, uint32_t* out_node_bytes, uint8_t* store, float* centroid);

/* Merge per-shard top-k lists (device pointers, [n_shards][n_queries][k])
 * into the global top-k by (distance, id), on `stream`.  Used after the shards
 * of a range-sharded index are gathered on one GPU; no reference counterpart
 * (the reference has no multi-GPU path). */
int jb_merge_topk(const int32_t* shard_idx, const float* shard_dist, uint32_t n_shards,
                  uint64_t n_queries, uint32_t k, int32_t* out_idx, float* out_dist, void* stream);

/* jb_merge_topk with shard s's lists starting shard_stride elements after
 * shard s-1's (shard_stride >= n_queries * k): the layout of one gathered
 * buffer [n_shards][2][n_queries][k] in which each shard sends its ids and
 * distance bits together (shard_stride = 2 * n_queries * k).  No reference
 * counterpart. */
int jb_merge_topk_strided(const int32_t* shard_idx, const float* shard_dist, uint64_t shard_stride,
                          uint32_t n_shards, uint64_t n_queries, uint32_t k, int32_t* out_idx,
                          float* out_dist, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* JASPER_B200_H_ */
