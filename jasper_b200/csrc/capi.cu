// capi.cu -- extern "C" entry points of libjasper_b200.so (include/jasper_b200.h).
//
// The handle table mirrors the reference's (ffi/jasper_ffi_plain.cu:10-13):
// a process-wide map from int64 handle to graph, guarded by one mutex that is
// held only for lookups; the op bodies run unlocked.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstring>
#include <functional>
#include <memory>
#include <tuple>
#include <map>
#include <mutex>
#include <set>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>
#include "../../include/jasper_b200.h"
#include "builders.cuh"
#include "rabitq.cuh"
#include "construct.cuh"
#include "dirsearch.cuh"
#include "rotate.cuh"
#include "jb_graph.h"
#include "merge.cuh"
#include "search.cuh"

namespace {

thread_local std::string g_last_error;
std::unordered_map<int64_t, std::shared_ptr<jb::Graph>> g_graphs;
int64_t g_next_handle = 0;
std::mutex g_mutex;

struct InvalidHandle : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct IoError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

template <typename F>
int guarded(F&& f) {
  try {
    f();
    g_last_error.clear();
    return JB_OK;
  } catch (const InvalidHandle& e) {
    return fail(JB_ERR_INVALID_HANDLE, e.what());
  } catch (const std::invalid_argument& e) {
    return fail(JB_ERR_INVALID_ARGUMENT, e.what());
  } catch (const IoError& e) {
    return fail(JB_ERR_IO, e.what());
  } catch (const std::exception& e) {
    std::string m = e.what();
    if (m.find("Failed to open") != std::string::npos || m.find("Short read") != std::string::npos ||
        m.find("graph file") != std::string::npos)
      return fail(JB_ERR_IO, m);
    return fail(JB_ERR_RUNTIME, m);
  } catch (...) {
    return fail(JB_ERR_RUNTIME, "unknown error");
  }
}

std::shared_ptr<jb::Graph> lookup(int64_t h) {
  std::lock_guard<std::mutex> lock(g_mutex);
  auto it = g_graphs.find(h);
  if (it == g_graphs.end()) throw InvalidHandle("Invalid handle: " + std::to_string(h));
  return it->second;
}

int64_t insert(std::shared_ptr<jb::Graph> g) {
  std::lock_guard<std::mutex> lock(g_mutex);
  int64_t h = g_next_handle++;
  g_graphs[h] = std::move(g);
  return h;
}

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
  }
}

// Runs with the graph's device current, restoring the caller's afterwards.
struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceScope() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

void check_metric(int32_t metric) {
  if (metric != JB_METRIC_L2 && metric != JB_METRIC_IP)
    throw std::invalid_argument("metric must be JB_METRIC_L2 or JB_METRIC_IP");
}

// Device search over queries with any row stride: rows whose stride is not
// the padded dim are first packed into a padded scratch copy.
// rq_margin >= 0 turns on the RaBitQ candidate filter; `rotate` applies the
// graph's prerotation to the queries first.
// Per-call search buffers (repacked queries, results, work counter) come from
// a stream-ordered pool of the library's own, one per device, that keeps up to
// 256 MiB reserved between calls: a pool with the default release threshold of
// 0 hands its memory back to the driver at every synchronisation, so each call
// would map it afresh.  The device's default pool, which other libraries in
// the process share, is left as it is.
cudaMemPool_t search_pool() {
  static std::mutex m;
  static std::map<int, cudaMemPool_t> pools;
  int dev = 0;
  cuda_check(cudaGetDevice(&dev), "get device");
  std::lock_guard<std::mutex> lock(m);
  auto it = pools.find(dev);
  if (it != pools.end()) return it->second;
  cudaMemPoolProps props{};
  props.allocType = cudaMemAllocationTypePinned;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = dev;
  cudaMemPool_t pool;
  cuda_check(cudaMemPoolCreate(&pool, &props), "create search pool");
  uint64_t keep = uint64_t(256) << 20;
  cuda_check(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep),
             "set search pool threshold");
  pools[dev] = pool;
  return pool;
}

void pool_alloc(void** p, size_t bytes, cudaStream_t st, const char* what) {
  cuda_check(cudaMallocFromPoolAsync(p, bytes, search_pool(), st), what);
}

// Device address of page-locked host memory mapped into the current
// device's address space; null for pageable or device memory.
void* mapped_host(const void* p) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return at.type == cudaMemoryTypeHost ? at.devicePointer : nullptr;
}

void search_impl(const jb::Graph& g, const uint16_t* queries, uint64_t nq, uint32_t row_stride,
                 int32_t* out_idx, float* out_dist, uint32_t k, uint32_t bw, uint32_t limit,
                 uint32_t* stats, uint32_t* seen, cudaStream_t st, float rq_margin = -1.0f,
                 bool rotate = false, bool host_queries = false) {
  if (nq == 0) return;
  if (nq > 0x7FFFFFFFull) throw std::invalid_argument("too many queries");
  if (k == 0) throw std::invalid_argument("k must be > 0");
  if (row_stride < g.dim) throw std::invalid_argument("row_stride < dim");
  if (out_idx == nullptr || out_dist == nullptr || queries == nullptr)
    throw std::invalid_argument("null pointer argument");
  const uint16_t* q = queries;
  void* packed = nullptr;
  void* counter = nullptr;
  const bool aligned = (reinterpret_cast<uintptr_t>(queries) % 16) == 0;
  // Prerotated graphs rotate the queries in the search kernel's prologue; a
  // separate GEMM pass over packed queries is left only for very wide rows.
  const bool fused_rotation = rotate && g.dpad <= jb::kFusedRotationMaxDpad;
  if (fused_rotation) rotate = false;
  if (row_stride != g.dpad || !aligned || rotate) {
    pool_alloc(reinterpret_cast<void**>(&packed), size_t(nq) * g.dpad * 2, st, "alloc packed queries");
    cuda_check(cudaMemsetAsync(packed, 0, size_t(nq) * g.dpad * 2, st), "clear packed queries");
    cuda_check(cudaMemcpy2DAsync(packed, size_t(g.dpad) * 2, queries, size_t(row_stride) * 2,
                                 size_t(g.dim) * 2, nq, cudaMemcpyDefault, st),
               "pack queries");
    if (rotate) {
      try {
        jb::rotate_rows_inplace(g, static_cast<uint16_t*>(packed), nq, st);
      } catch (...) {
        cudaFreeAsync(packed, st);
        throw;
      }
    }
    q = static_cast<const uint16_t*>(packed);
  }
  pool_alloc(reinterpret_cast<void**>(&counter), jb::kSearchScratchBytes, st, "alloc search scratch");
  cuda_check(cudaMemsetAsync(counter, 0, jb::kSearchScratchBytes, st), "clear search scratch");
  jb::SearchArgs a{};
  a.g = g.view();
  a.queries = q;
  a.nq = uint32_t(nq);
  a.k = k;
  a.bw = bw;
  a.limit = limit;
  a.max_result_size = 2048;  // jasper::search_params default (beam_search/api.cuh:17)
  a.out_idx = out_idx;
  a.out_dist = out_dist;
  a.work_counter = static_cast<uint32_t*>(counter);
  a.stats = stats;
  a.seen_bits = seen;
  a.rot_pad = fused_rotation ? g.dir.rotation_pad : nullptr;
  // queries still in page-locked host memory (not repacked): staged per row
  a.stage_query = (host_queries && q == queries) ? 1 : 0;
  if (a.stage_query && a.rot_pad != nullptr) throw std::logic_error("host queries on a prerotated graph");
  if (rq_margin >= 0.0f) {
    if (!g.dir.has_rabitq) throw std::runtime_error("graph has no RaBitQ codes built");
    if (!g.dir.rq_err)
      throw std::runtime_error("graph has RaBitQ codes but no error scales (build them with "
                               "jb_graph_build_rabitq)");
    a.rq_on = 1;
    a.rq_store = g.dir.rq_store;
    a.rq_node_bytes = g.dir.rq_node_bytes;
    a.rq_code_bytes = g.dir.rq_code_bytes;
    a.rq_centroid = g.dir.rq_centroid;
    a.rq_err = g.dir.rq_err;
    a.rq_margin = rq_margin;
  }
  try {
    jb::launch_search(a, st);
  } catch (...) {
    cudaFreeAsync(counter, st);
    if (packed) cudaFreeAsync(packed, st);
    throw;
  }
  cuda_check(cudaFreeAsync(counter, st), "free search scratch");
  if (packed) cuda_check(cudaFreeAsync(packed, st), "free packed queries");
}

}  // namespace

// Handle lookup and error reporting for entry points defined in other files
// of this library (noalloc.cu).
namespace jb {
std::shared_ptr<Graph> capi_lookup(int64_t h) { return lookup(h); }
int capi_guarded(const std::function<void()>& f) { return guarded(f); }
}  // namespace jb

extern "C" {

const char* jb_last_error(void) { return g_last_error.c_str(); }

int jb_abi_version(void) { return 1; }

int jb_search_set_warps_per_query(int32_t warps_per_query) {
  return guarded([&] { jb::set_search_mode(warps_per_query); });
}

int jb_graph_create(const uint16_t* vectors, uint64_t n, uint32_t dim, uint32_t row_stride,
                    uint32_t n_neighbors, int32_t metric, int32_t on_host, int64_t* out_handle) {
  return guarded([&] {
    check_metric(metric);
    if (out_handle == nullptr) throw std::invalid_argument("out_handle is null");
    if (n > 0 && vectors == nullptr) throw std::invalid_argument("vectors is null");
    if (row_stride < dim) throw std::invalid_argument("row_stride < dim");
    if (n >= 0x7FFFFFFFull) throw std::invalid_argument("too many vectors");
    auto g = std::make_shared<jb::Graph>();
    jb::graph_allocate(*g, dim, n_neighbors, metric, uint32_t(n), on_host != 0);
    try {
      jb::graph_upload_rows(*g, vectors, row_stride);
    } catch (...) {
      jb::graph_free(*g);
      throw;
    }
    *out_handle = insert(g);
  });
}

int jb_graph_construct(const uint16_t* vectors, uint64_t n, uint32_t dim, uint32_t row_stride,
                       uint32_t n_neighbors, int32_t metric, double alpha,
                       uint64_t workspace_budget_bytes, int32_t on_host, void* stream,
                       int64_t* out_handle) {
  return guarded([&] {
    check_metric(metric);
    if (out_handle == nullptr) throw std::invalid_argument("out_handle is null");
    if (n > 0 && vectors == nullptr) throw std::invalid_argument("vectors is null");
    if (row_stride < dim) throw std::invalid_argument("row_stride < dim");
    if (n >= 0x7FFFFFFFull) throw std::invalid_argument("too many vectors");
    auto g = std::make_shared<jb::Graph>();
    jb::graph_allocate(*g, dim, n_neighbors, metric, uint32_t(n), on_host != 0);
    try {
      jb::graph_upload_rows(*g, vectors, row_stride);
      uint32_t mb = jb::reference_max_batch_size(workspace_budget_bytes, uint32_t(n), n_neighbors);
      jb::construct_graph(*g, float(alpha), mb, static_cast<cudaStream_t>(stream));
    } catch (...) {
      jb::graph_free(*g);
      throw;
    }
    *out_handle = insert(g);
  });
}

int jb_graph_load(const char* path, uint32_t dim, uint32_t n_neighbors, int32_t metric,
                  int32_t on_host, int64_t* out_handle) {
  return guarded([&] {
    check_metric(metric);
    if (path == nullptr || out_handle == nullptr) throw std::invalid_argument("null argument");
    auto g = std::make_shared<jb::Graph>();
    jb::graph_load_file(*g, path, dim, n_neighbors, metric, on_host != 0);
    *out_handle = insert(g);
  });
}

int jb_graph_save(int64_t handle, const char* path) {
  return guarded([&] {
    if (path == nullptr) throw std::invalid_argument("path is null");
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    cuda_check(cudaDeviceSynchronize(), "sync before save");
    jb::graph_save_file(*g, path);
  });
}

int jb_graph_search(int64_t handle, const uint16_t* queries, uint64_t n_queries,
                    uint32_t row_stride, int32_t* out_idx, float* out_dist, uint32_t k,
                    uint32_t beam_width, uint32_t limit, void* stream) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    search_impl(*g, queries, n_queries, row_stride, out_idx, out_dist, k, beam_width, limit,
                nullptr, nullptr, static_cast<cudaStream_t>(stream));
  });
}

int jb_graph_search_stats(int64_t handle, const uint16_t* queries, uint64_t n_queries,
                          uint32_t row_stride, int32_t* out_idx, float* out_dist, uint32_t k,
                          uint32_t beam_width, uint32_t limit, uint32_t* stats,
                          uint32_t* seen_scratch, void* stream) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    search_impl(*g, queries, n_queries, row_stride, out_idx, out_dist, k, beam_width, limit, stats,
                seen_scratch, static_cast<cudaStream_t>(stream));
  });
}

int jb_graph_search_host(int64_t handle, const uint16_t* queries, uint64_t n_queries,
                         uint32_t row_stride, int32_t* out_idx, float* out_dist, uint32_t k,
                         uint32_t beam_width, uint32_t limit, void* stream) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (n_queries == 0) return;
    if (queries == nullptr || out_idx == nullptr || out_dist == nullptr)
      throw std::invalid_argument("null pointer argument");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t qbytes = size_t(n_queries) * g->dpad * 2;
    const size_t obytes = size_t(n_queries) * k * 4;
    // Page-locked buffers are used in place: the search kernel reads each
    // query row over the host link once (16-byte loads staged in shared
    // memory) and writes the results straight into host memory, so no copy
    // sits before or after the search.  Pageable buffers (and query rows
    // that are not at the padded stride, 16-byte aligned) go through device
    // buffers and stream-ordered copies.
    void* mq = mapped_host(queries);
    void* mi = mapped_host(out_idx);
    void* md = mapped_host(out_dist);
    const bool q_direct = mq != nullptr && row_stride == g->dpad &&
                          (reinterpret_cast<uintptr_t>(mq) % 16) == 0;
    void *dq = nullptr, *di = nullptr, *dd = nullptr;
    try {
      if (!q_direct) {
        pool_alloc(&dq, qbytes, st, "alloc queries");
        if (row_stride == g->dpad) {
          cuda_check(cudaMemcpyAsync(dq, queries, qbytes, cudaMemcpyHostToDevice, st), "copy queries");
        } else {
          cuda_check(cudaMemsetAsync(dq, 0, qbytes, st), "clear queries");
          cuda_check(cudaMemcpy2DAsync(dq, size_t(g->dpad) * 2, queries, size_t(row_stride) * 2,
                                       size_t(g->dim) * 2, n_queries, cudaMemcpyHostToDevice, st),
                     "copy queries");
        }
      }
      if (mi == nullptr) pool_alloc(&di, obytes, st, "alloc out idx");
      if (md == nullptr) pool_alloc(&dd, obytes, st, "alloc out dist");
      search_impl(*g, q_direct ? static_cast<const uint16_t*>(mq) : static_cast<uint16_t*>(dq),
                  n_queries, g->dpad, static_cast<int32_t*>(mi ? mi : di),
                  static_cast<float*>(md ? md : dd), k, beam_width, limit, nullptr, nullptr, st,
                  -1.0f, false, q_direct);
      if (di) cuda_check(cudaMemcpyAsync(out_idx, di, obytes, cudaMemcpyDeviceToHost, st), "copy idx");
      if (dd) cuda_check(cudaMemcpyAsync(out_dist, dd, obytes, cudaMemcpyDeviceToHost, st), "copy dist");
    } catch (...) {
      for (void* p : {dq, di, dd})
        if (p) cudaFreeAsync(p, st);
      cudaStreamSynchronize(st);
      throw;
    }
    for (void* p : {dq, di, dd})
      if (p) cudaFreeAsync(p, st);
    cuda_check(cudaStreamSynchronize(st), "search");
  });
}

int jb_graph_free(int64_t handle) {
  return guarded([&] {
    std::shared_ptr<jb::Graph> g;
    {
      std::lock_guard<std::mutex> lock(g_mutex);
      auto it = g_graphs.find(handle);
      if (it == g_graphs.end()) throw InvalidHandle("Invalid handle: " + std::to_string(handle));
      g = it->second;
      g_graphs.erase(it);
    }
    DeviceScope ds(g->device);
    cudaDeviceSynchronize();
    jb::graph_free(*g);
  });
}

int jb_graph_get_info(int64_t handle, jb_graph_info* out) {
  return guarded([&] {
    if (out == nullptr) throw std::invalid_argument("out is null");
    auto g = lookup(handle);
    out->n_vectors = g->n;
    out->n_deleted = g->n_deleted;
    out->next_id = g->next_id;
    out->dim = g->dim;
    out->n_neighbors = g->R;
    out->metric = g->metric;
    out->medoid = g->medoid;
    out->global_offset = g->global_offset;
    out->on_host = g->on_host ? 1 : 0;
    out->device = g->device;
  });
}

int jb_graph_get_vector(int64_t handle, int64_t stable_id, uint16_t* out) {
  return guarded([&] {
    if (out == nullptr) throw std::invalid_argument("out is null");
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (stable_id < 0) throw std::invalid_argument("stable id must be non-negative");
    int64_t slot = -1;
    if (g->ids_identity) {
      if (uint64_t(stable_id) < g->n) slot = stable_id;
    } else {
      std::vector<uint32_t> ids(g->n);
      cuda_check(cudaMemcpy(ids.data(), g->slot_to_id, size_t(g->n) * 4, cudaMemcpyDefault), "ids");
      for (uint32_t i = 0; i < g->n; i++)
        if (ids[i] == uint32_t(stable_id)) { slot = i; break; }
    }
    if (slot < 0) throw std::invalid_argument("Stable id " + std::to_string(stable_id) + " not found");
    cuda_check(cudaMemcpy(out, g->vec + size_t(slot) * g->dpad, size_t(g->dim) * 2, cudaMemcpyDefault),
               "copy vector");
  });
}

int jb_graph_reserve_ids(int64_t handle, int64_t count, int32_t* out_ids) {
  return guarded([&] {
    auto g = lookup(handle);
    if (count < 0) throw std::invalid_argument("count must be >= 0");
    if (count > 0 && out_ids == nullptr) throw std::invalid_argument("out_ids is null");
    const uint64_t start = g->next_id;
    g->next_id += uint64_t(count);
    for (int64_t i = 0; i < count; i++) out_ids[i] = int32_t(start + uint64_t(i));
  });
}

int jb_graph_mark_deleted(int64_t handle, const int32_t* ids, uint64_t n_ids) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (n_ids > 0 && ids == nullptr) throw std::invalid_argument("ids is null");
    std::vector<uint32_t> words((size_t(g->n) + 31) / 32);
    cuda_check(cudaDeviceSynchronize(), "sync");
    cuda_check(cudaMemcpy(words.data(), g->deleted, words.size() * 4, cudaMemcpyDefault), "bits");
    for (uint64_t i = 0; i < n_ids; i++) {
      const int64_t id = ids[i];
      if (id < 0 || uint64_t(id) >= g->n) continue;  // ids are slots while ids are identity
      uint32_t& w = words[size_t(id) >> 5];
      const uint32_t bit = 1u << (id & 31);
      if (!(w & bit)) { w |= bit; g->n_deleted++; }
    }
    cuda_check(cudaMemcpy(g->deleted, words.data(), words.size() * 4, cudaMemcpyDefault), "bits");
  });
}

int jb_graph_append(int64_t handle, const uint16_t* vectors, uint64_t n, uint32_t row_stride,
                    double alpha, int32_t* out_ids, void* stream) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (n > 0 && vectors == nullptr) throw std::invalid_argument("vectors is null");
    auto ids = jb::graph_append(*g, vectors, n, row_stride, float(alpha),
                                static_cast<cudaStream_t>(stream));
    if (out_ids != nullptr)
      for (size_t i = 0; i < ids.size(); i++) out_ids[i] = int32_t(ids[i]);
  });
}

int jb_graph_set_edges(int64_t handle, const uint32_t* edges, const uint16_t* edge_dists,
                       const uint8_t* counts, uint32_t medoid) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (!edges || !edge_dists || !counts) throw std::invalid_argument("null argument");
    if (medoid - g->global_offset >= g->n && g->n > 0) throw std::invalid_argument("medoid out of range");
    const size_t nr = size_t(g->n) * g->R;
    cuda_check(cudaMemcpy(g->edges, edges, nr * 4, cudaMemcpyDefault), "set edges");
    cuda_check(cudaMemcpy(g->edist, edge_dists, nr * 2, cudaMemcpyDefault), "set dists");
    cuda_check(cudaMemcpy(g->counts, counts, g->n, cudaMemcpyDefault), "set counts");
    g->medoid = medoid;
    if (g->eflag) {  // edges set from outside: no prune of them is known
      cudaFree(g->eflag);
      g->eflag = nullptr;
    }
  });
}

int jb_graph_get_edges(int64_t handle, uint32_t* edges, uint16_t* edge_dists, uint8_t* counts) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (!edges || !edge_dists || !counts) throw std::invalid_argument("null argument");
    cuda_check(cudaDeviceSynchronize(), "sync");
    const size_t nr = size_t(g->n) * g->R;
    cuda_check(cudaMemcpy(edges, g->edges, nr * 4, cudaMemcpyDefault), "get edges");
    cuda_check(cudaMemcpy(edge_dists, g->edist, nr * 2, cudaMemcpyDefault), "get dists");
    cuda_check(cudaMemcpy(counts, g->counts, g->n, cudaMemcpyDefault), "get counts");
  });
}

int jb_graph_apply_global_offset(int64_t handle, uint32_t offset) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (uint64_t(offset) + g->n >= 0x7FFFFFFFull) throw std::invalid_argument("offset too large");
    cuda_check(cudaDeviceSynchronize(), "sync");
    const size_t nr = size_t(g->n) * g->R;
    std::vector<uint32_t> e(nr);
    std::vector<uint8_t> c(g->n);
    cuda_check(cudaMemcpy(e.data(), g->edges, nr * 4, cudaMemcpyDefault), "edges");
    cuda_check(cudaMemcpy(c.data(), g->counts, g->n, cudaMemcpyDefault), "counts");
    const uint32_t delta = offset - g->global_offset;
    for (uint32_t i = 0; i < g->n; i++)
      for (uint32_t j = 0; j < c[i]; j++) {
        uint32_t& v = e[size_t(i) * g->R + j];
        if (v != 0xFFFFFFFFu) v += delta;
      }
    cuda_check(cudaMemcpy(g->edges, e.data(), nr * 4, cudaMemcpyDefault), "edges");
    g->medoid += delta;
    g->global_offset = offset;
  });
}

int jb_rotation_matrix(uint32_t dim, uint64_t seed, float* out) {
  return guarded([&] {
    if (dim == 0 || !out) throw std::invalid_argument("dim must be > 0 and out non-null");
    std::vector<float> P = jb::rotation_matrix_f32(int(dim), seed);
    std::memcpy(out, P.data(), P.size() * sizeof(float));
  });
}

int jb_graph_set_lsh(int64_t handle, uint32_t k_ranks, uint32_t packed_bytes, const void* packed,
                     const uint16_t* mag_sq, const float* c, float norm_denom) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (k_ranks == 0 || k_ranks > 16) throw std::invalid_argument("k_ranks must be in [1, 16]");
    if (packed_bytes != 1 && packed_bytes != 2) throw std::invalid_argument("packed_bytes must be 1 or 2");
    if (packed_bytes == 1 && g->dpad > 128)
      throw std::invalid_argument("1-byte LSH words address at most 128 coordinates");
    if (!packed || !mag_sq || !c) throw std::invalid_argument("null argument");
    jb::DirArtifacts& d = g->dir;
    if (d.lsh_packed) { cudaFree(d.lsh_packed); d.lsh_packed = nullptr; }
    if (d.lsh_mag) { cudaFree(d.lsh_mag); d.lsh_mag = nullptr; }
    const size_t nw = size_t(g->n) * g->R * k_ranks;
    cuda_check(cudaMalloc(&d.lsh_packed, nw * packed_bytes + 16), "alloc lsh words");
    cuda_check(cudaMalloc(&d.lsh_mag, size_t(g->n) * g->R * 2 + 16), "alloc lsh magnitudes");
    cuda_check(cudaMemcpy(d.lsh_packed, packed, nw * packed_bytes, cudaMemcpyDefault), "lsh words");
    cuda_check(cudaMemcpy(d.lsh_mag, mag_sq, size_t(g->n) * g->R * 2, cudaMemcpyDefault), "lsh mags");
    d.k_ranks = k_ranks;
    d.packed_bytes = packed_bytes;
    for (uint32_t r = 0; r < 16; r++) d.lsh_c[r] = r < k_ranks ? c[r] : 0.f;
    d.norm_denom = norm_denom;
    d.has_lsh = true;
  });
}

int jb_graph_set_pq(int64_t handle, uint32_t m, uint32_t dsub, const float* centroids,
                    const uint8_t* codes, const float* norms) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (m == 0 || dsub == 0 || m * dsub != g->dpad)
      throw std::invalid_argument("PQ needs m * dsub == padded dim");
    if (!centroids || !codes || !norms) throw std::invalid_argument("null argument");
    jb::DirArtifacts& d = g->dir;
    if (d.pq_centroids) { cudaFree(d.pq_centroids); d.pq_centroids = nullptr; }
    if (d.pq_codes) { cudaFree(d.pq_codes); d.pq_codes = nullptr; }
    if (d.norms) { cudaFree(d.norms); d.norms = nullptr; }
    const size_t nc = size_t(m) * 256 * dsub, ncode = size_t(g->n) * g->R * m;
    cuda_check(cudaMalloc(&d.pq_centroids, nc * 4), "alloc centroids");
    cuda_check(cudaMalloc(&d.pq_codes, ncode + 16), "alloc codes");
    cuda_check(cudaMalloc(&d.norms, size_t(g->n) * 4 + 16), "alloc norms");
    cuda_check(cudaMemcpy(d.pq_centroids, centroids, nc * 4, cudaMemcpyDefault), "centroids");
    cuda_check(cudaMemcpy(d.pq_codes, codes, ncode, cudaMemcpyDefault), "codes");
    cuda_check(cudaMemcpy(d.norms, norms, size_t(g->n) * 4, cudaMemcpyDefault), "norms");
    d.pq_m = m;
    d.pq_dsub = dsub;
    d.has_pq = true;
  });
}

int jb_graph_get_directional_flags(int64_t handle, int32_t* out_flags) {
  return guarded([&] {
    if (!out_flags) throw std::invalid_argument("out_flags is null");
    auto g = lookup(handle);
    *out_flags = (g->dir.has_lsh ? 1 : 0) | (g->dir.has_pq ? 2 : 0) | (g->dir.has_rabitq ? 4 : 0);
  });
}

int jb_graph_directional_search(int64_t handle, int32_t kind, const uint16_t* queries,
                                uint64_t n_queries, uint32_t row_stride, int32_t* out_idx,
                                float* out_dist, uint32_t k, uint32_t beam_width, uint32_t limit,
                                void* stream) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (kind != JB_DIR_LSH && kind != JB_DIR_PQ && kind != JB_DIR_RABITQ)
      throw std::invalid_argument("kind must be LSH, PQ or RaBitQ");
    const jb::DirArtifacts& d = g->dir;
    if (kind == JB_DIR_LSH && !d.has_lsh)
      throw std::runtime_error("Graph " + std::to_string(handle) + " has no LSH artifacts built");
    if (kind == JB_DIR_PQ && !d.has_pq)
      throw std::runtime_error("Graph " + std::to_string(handle) + " has no PQ artifacts built");
    if (kind == JB_DIR_RABITQ && !d.has_rabitq)
      throw std::runtime_error("Graph " + std::to_string(handle) + " has no RaBitQ codes built");
    if (kind == JB_DIR_RABITQ) {  // the exact search with the RaBitQ filter, margin 1
      search_impl(*g, queries, n_queries, row_stride, out_idx, out_dist, k, beam_width, limit,
                  nullptr, nullptr, static_cast<cudaStream_t>(stream), 1.0f, d.prerotate);
      return;
    }
    if (n_queries == 0) return;
    if (!queries || !out_idx || !out_dist) throw std::invalid_argument("null pointer argument");
    if (row_stride < g->dim) throw std::invalid_argument("row_stride < dim");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    void* packed = nullptr;
    void* counter = nullptr;
    const uint16_t* q = queries;
    const size_t qbytes = size_t(n_queries) * g->dpad * 2;
    const bool aligned = (reinterpret_cast<uintptr_t>(queries) % 16) == 0;
    const bool fused_rotation = d.prerotate && g->dpad <= jb::kFusedRotationMaxDpad;
    if (row_stride != g->dpad || !aligned || (d.prerotate && !fused_rotation)) {
      pool_alloc(reinterpret_cast<void**>(&packed), qbytes, st, "alloc queries");
      cuda_check(cudaMemsetAsync(packed, 0, qbytes, st), "clear queries");
      cuda_check(cudaMemcpy2DAsync(packed, size_t(g->dpad) * 2, queries, size_t(row_stride) * 2,
                                   size_t(g->dim) * 2, n_queries, cudaMemcpyDefault, st),
                 "pack queries");
      if (d.prerotate && !fused_rotation)
        jb::rotate_rows_inplace(*g, static_cast<uint16_t*>(packed), n_queries, st);
      q = static_cast<const uint16_t*>(packed);
    }
    pool_alloc(reinterpret_cast<void**>(&counter), 256, st, "alloc counter");
    cuda_check(cudaMemsetAsync(counter, 0, 256, st), "clear counter");
    jb::DirSearchArgs a{};
    a.g = g->view();
    a.kind = kind;
    a.k_ranks = d.k_ranks;
    a.packed_bytes = d.packed_bytes;
    a.packed = d.lsh_packed;
    a.mag = d.lsh_mag;
    for (int r = 0; r < 16; r++) a.c[r] = d.lsh_c[r];
    a.inv_norm_denom = d.has_lsh ? 1.0f / d.norm_denom : 0.f;
    a.pq_m = d.pq_m;
    a.pq_dsub = d.pq_dsub;
    a.centroids = d.pq_centroids;
    a.codes = d.pq_codes;
    a.norms = d.norms;
    a.queries = q;
    a.nq = uint32_t(n_queries);
    a.k = k;
    a.bw = beam_width;
    a.limit = limit;
    a.max_result_size = 2048;
    a.out_idx = out_idx;
    a.out_dist = out_dist;
    a.work_counter = static_cast<uint32_t*>(counter);
    a.rot_pad = fused_rotation ? d.rotation_pad : nullptr;
    try {
      jb::launch_dir_search(a, st);
    } catch (...) {
      cudaFreeAsync(counter, st);
      if (packed) cudaFreeAsync(packed, st);
      throw;
    }
    cudaFreeAsync(counter, st);
    if (packed) cudaFreeAsync(packed, st);
  });
}

int jb_merge_topk(const int32_t* shard_idx, const float* shard_dist, uint32_t n_shards,
                  uint64_t n_queries, uint32_t k, int32_t* out_idx, float* out_dist, void* stream) {
  return guarded([&] {
    if (n_queries == 0) return;
    if (!shard_idx || !shard_dist || !out_idx || !out_dist) throw std::invalid_argument("null argument");
    jb::launch_merge_topk(shard_idx, shard_dist, n_shards, n_queries, k, n_queries * k, out_idx,
                          out_dist, static_cast<cudaStream_t>(stream));
  });
}

int jb_merge_topk_strided(const int32_t* shard_idx, const float* shard_dist, uint64_t shard_stride,
                          uint32_t n_shards, uint64_t n_queries, uint32_t k, int32_t* out_idx,
                          float* out_dist, void* stream) {
  return guarded([&] {
    if (n_queries == 0) return;
    if (!shard_idx || !shard_dist || !out_idx || !out_dist) throw std::invalid_argument("null argument");
    jb::launch_merge_topk(shard_idx, shard_dist, n_shards, n_queries, k, shard_stride, out_idx,
                          out_dist, static_cast<cudaStream_t>(stream));
  });
}

int jb_graph_construct_directional(const uint16_t* vectors, uint64_t n, uint32_t dim,
                                   uint32_t row_stride, uint32_t n_neighbors, int32_t metric,
                                   double alpha, uint64_t workspace_budget_bytes, int32_t on_host,
                                   int32_t prerotate, uint64_t prerotate_seed, void* stream,
                                   int64_t* out_handle) {
  return guarded([&] {
    check_metric(metric);
    if (out_handle == nullptr) throw std::invalid_argument("out_handle is null");
    if (n > 0 && vectors == nullptr) throw std::invalid_argument("vectors is null");
    if (row_stride < dim) throw std::invalid_argument("row_stride < dim");
    if (n >= 0x7FFFFFFFull) throw std::invalid_argument("too many vectors");
    auto g = std::make_shared<jb::Graph>();
    jb::graph_allocate(*g, dim, n_neighbors, metric, uint32_t(n), on_host != 0);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    try {
      jb::graph_upload_rows(*g, vectors, row_stride);
      if (prerotate) {
        jb::set_rotation(*g, prerotate_seed);
        jb::rotate_rows_inplace(*g, g->vec, n, st);
        cuda_check(cudaStreamSynchronize(st), "prerotate");
      }
      uint32_t mb = jb::reference_max_batch_size(workspace_budget_bytes, uint32_t(n), n_neighbors);
      jb::construct_graph(*g, float(alpha), mb, st);
    } catch (...) {
      jb::graph_free(*g);
      throw;
    }
    *out_handle = insert(g);
  });
}

int jb_graph_build_lsh(int64_t handle, uint32_t k_ranks, uint64_t n_samples, uint64_t seed) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (n_samples == 0 || n_samples > 0xFFFFFFFFull)
      throw std::invalid_argument("n_samples must be in [1, 2^32)");
    cuda_check(cudaDeviceSynchronize(), "sync before build_lsh");
    jb::build_lsh(*g, k_ranks, uint32_t(n_samples), seed, nullptr);
  });
}

int jb_graph_build_pq(int64_t handle, uint32_t m, uint64_t n_train, uint32_t kmeans_iter,
                      uint64_t seed) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (n_train > 0xFFFFFFFFull) throw std::invalid_argument("n_train must be below 2^32");
    cuda_check(cudaDeviceSynchronize(), "sync before build_pq");
    jb::build_pq(*g, m, uint32_t(n_train), kmeans_iter, seed, nullptr);
  });
}

int jb_graph_save_directional(int64_t handle, const char* path) {
  return guarded([&] {
    if (path == nullptr) throw std::invalid_argument("path is null");
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    cuda_check(cudaDeviceSynchronize(), "sync before save");
    jb::graph_save_directional(*g, path);
  });
}

int jb_graph_load_directional(const char* path, uint32_t dim, uint32_t n_neighbors,
                              int32_t metric, uint32_t k_ranks, int32_t on_host,
                              int32_t prerotate, uint64_t prerotate_seed, int64_t* out_handle) {
  return guarded([&] {
    check_metric(metric);
    if (path == nullptr || out_handle == nullptr) throw std::invalid_argument("null argument");
    if (k_ranks == 0 || k_ranks > 16) throw std::invalid_argument("k_ranks must be in [1, 16]");
    auto g = std::make_shared<jb::Graph>();
    jb::graph_load_file(*g, path, dim, n_neighbors, metric, on_host != 0);
    try {
      jb::graph_load_directional(*g, path, k_ranks);
      if (prerotate) jb::set_rotation(*g, prerotate_seed);
    } catch (...) {
      jb::graph_free(*g);
      throw;
    }
    *out_handle = insert(g);
  });
}

int jb_graph_get_lsh(int64_t handle, uint32_t* out_k_ranks, uint32_t* out_packed_bytes,
                     void* packed, uint16_t* mag_sq, float* c, float* norm_denom) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    const jb::DirArtifacts& d = g->dir;
    if (!d.has_lsh) throw std::runtime_error("Graph " + std::to_string(handle) + " has no LSH artifacts built");
    cuda_check(cudaDeviceSynchronize(), "sync");
    if (out_k_ranks) *out_k_ranks = d.k_ranks;
    if (out_packed_bytes) *out_packed_bytes = d.packed_bytes;
    const size_t ne = size_t(g->n) * g->R;
    if (packed) cuda_check(cudaMemcpy(packed, d.lsh_packed, ne * d.k_ranks * d.packed_bytes, cudaMemcpyDefault), "lsh words");
    if (mag_sq) cuda_check(cudaMemcpy(mag_sq, d.lsh_mag, ne * 2, cudaMemcpyDefault), "lsh mags");
    if (c) std::memcpy(c, d.lsh_c, 4 * d.k_ranks);
    if (norm_denom) *norm_denom = d.norm_denom;
  });
}

int jb_graph_get_pq(int64_t handle, uint32_t* out_m, uint32_t* out_dsub, float* centroids,
                    uint8_t* codes, float* norms) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    const jb::DirArtifacts& d = g->dir;
    if (!d.has_pq) throw std::runtime_error("Graph " + std::to_string(handle) + " has no PQ artifacts built");
    cuda_check(cudaDeviceSynchronize(), "sync");
    if (out_m) *out_m = d.pq_m;
    if (out_dsub) *out_dsub = d.pq_dsub;
    if (centroids) cuda_check(cudaMemcpy(centroids, d.pq_centroids, size_t(d.pq_m) * 256 * d.pq_dsub * 4, cudaMemcpyDefault), "centroids");
    if (codes) cuda_check(cudaMemcpy(codes, d.pq_codes, size_t(g->n) * g->R * d.pq_m, cudaMemcpyDefault), "codes");
    if (norms && d.norms) cuda_check(cudaMemcpy(norms, d.norms, size_t(g->n) * 4, cudaMemcpyDefault), "norms");
  });
}

int jb_rotate_rows(uint32_t dim, uint64_t seed, const uint16_t* rows, uint16_t* out, uint64_t n,
                   int32_t use_tensor_cores, void* stream) {
  return guarded([&] {
    if (dim == 0) throw std::invalid_argument("dim must be > 0");
    if (n > 0 && (!rows || !out)) throw std::invalid_argument("null argument");
    if (n == 0) return;
    const uint32_t dpad = jb::pad_dim(dim);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The matrix for (device, dim, seed, layout) is built once and kept for
    // the life of the process (a few hundred KB at most per key).
    static std::mutex mu;
    static std::map<std::tuple<int, uint32_t, uint64_t, int>, void*> cache;
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    void* dm = nullptr;
    {
      std::lock_guard<std::mutex> lock(mu);
      auto key = std::make_tuple(dev, dim, seed, use_tensor_cores ? 1 : 0);
      auto it = cache.find(key);
      if (it != cache.end()) {
        dm = it->second;
      } else {
        std::vector<float> P = jb::rotation_matrix_f32(int(dim), seed);
        std::vector<uint16_t> Ph(P.size());
        for (size_t i = 0; i < P.size(); i++) {
          const __half h = __float2half_rn(P[i]);
          Ph[i] = *reinterpret_cast<const uint16_t*>(&h);
        }
        const std::vector<uint16_t> M = use_tensor_cores ? jb::pad_rotation(Ph, dim, dpad) : Ph;
        cuda_check(cudaMalloc(&dm, M.size() * 2), "alloc rotation");
        cuda_check(cudaMemcpy(dm, M.data(), M.size() * 2, cudaMemcpyHostToDevice), "rotation");
        cache[key] = dm;
      }
    }
    if (use_tensor_cores)
      jb::rotate_rows_tc(static_cast<uint16_t*>(dm), dpad, rows, out, n, st);
    else
      jb::rotate_rows(static_cast<uint16_t*>(dm), dim, dpad, rows, out, n, st);
    cuda_check(cudaStreamSynchronize(st), "rotate");
    if (use_tensor_cores)
      if (const int e = jb::rotate_tc_error(true))
        throw std::runtime_error("rotation GEMM gave up waiting (code " + std::to_string(e) + ")");
  });
}

int jb_rabitq_quantize(const float* rows, uint64_t n, uint32_t dim, const float* rotation,
                       const float* centroid, int32_t metric, uint8_t* out, void* stream) {
  return guarded([&] {
    check_metric(metric);
    if (n > 0 && (!rows || !centroid || !out)) throw std::invalid_argument("null argument");
    jb::rabitq_quantize_rows(rows, n, dim, rotation, centroid, metric == JB_METRIC_IP ? 1 : 0, out,
                             static_cast<cudaStream_t>(stream));
  });
}

int jb_graph_build_rabitq(int64_t handle) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    cuda_check(cudaDeviceSynchronize(), "sync before build_rabitq");
    jb::build_rabitq(*g, nullptr);
  });
}

int jb_graph_set_rabitq(int64_t handle, uint32_t node_bytes, const uint8_t* store,
                        const float* centroid) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    const uint32_t cb = jb::rabitq_code_bytes(g->dim);
    if (node_bytes != cb + 8)
      throw std::invalid_argument("node_bytes must be " + std::to_string(cb + 8) + " for dim " +
                                  std::to_string(g->dim));
    if (!store || !centroid) throw std::invalid_argument("null argument");
    jb::DirArtifacts& d = g->dir;
    if (d.rq_store) { cudaFree(d.rq_store); d.rq_store = nullptr; }
    if (d.rq_centroid) { cudaFree(d.rq_centroid); d.rq_centroid = nullptr; }
    cuda_check(cudaMalloc(&d.rq_store, size_t(g->n) * node_bytes + 16), "alloc rabitq codes");
    cuda_check(cudaMalloc(&d.rq_centroid, size_t(g->dim) * 4 + 16), "alloc rabitq centroid");
    cuda_check(cudaMemcpy(d.rq_store, store, size_t(g->n) * node_bytes, cudaMemcpyDefault), "codes");
    cuda_check(cudaMemcpy(d.rq_centroid, centroid, size_t(g->dim) * 4, cudaMemcpyDefault), "centroid");
    d.rq_code_bytes = cb;
    d.rq_node_bytes = node_bytes;
    d.has_rabitq = true;
  });
}

int jb_graph_get_rabitq(int64_t handle, uint32_t* out_node_bytes, uint8_t* store, float* centroid) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    const jb::DirArtifacts& d = g->dir;
    if (!d.has_rabitq) throw std::runtime_error("Graph " + std::to_string(handle) + " has no RaBitQ codes built");
    cuda_check(cudaDeviceSynchronize(), "sync");
    if (out_node_bytes) *out_node_bytes = d.rq_node_bytes;
    if (store) cuda_check(cudaMemcpy(store, d.rq_store, size_t(g->n) * d.rq_node_bytes, cudaMemcpyDefault), "codes");
    if (centroid) cuda_check(cudaMemcpy(centroid, d.rq_centroid, size_t(g->dim) * 4, cudaMemcpyDefault), "centroid");
  });
}

int jb_graph_search_rabitq(int64_t handle, const uint16_t* queries, uint64_t n_queries,
                           uint32_t row_stride, int32_t* out_idx, float* out_dist, uint32_t k,
                           uint32_t beam_width, uint32_t limit, float margin, uint32_t* stats,
                           void* stream) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (!(margin >= 0.0f)) throw std::invalid_argument("margin must be >= 0");
    search_impl(*g, queries, n_queries, row_stride, out_idx, out_dist, k, beam_width, limit, stats,
                nullptr, static_cast<cudaStream_t>(stream), margin, g->dir.prerotate);
  });
}

int jb_graph_get_rabitq_err(int64_t handle, float* err) {
  return guarded([&] {
    auto g = lookup(handle);
    DeviceScope ds(g->device);
    if (!g->dir.has_rabitq || !g->dir.rq_err) throw std::runtime_error("graph has no RaBitQ codes built");
    if (!err) throw std::invalid_argument("err is null");
    cuda_check(cudaMemcpy(err, g->dir.rq_err, size_t(g->n) * 4, cudaMemcpyDefault), "rabitq errors");
  });
}

}  // extern "C"
