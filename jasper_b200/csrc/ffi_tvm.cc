// ffi_tvm.cc -- tvm_ffi module with the reference's op names over libjasper_b200.
//
// Exports the functions the reference's Python package looks up by name
// (python/jasper/__init__.py:117-149): jasper_{load,construct,search,save,
// get_vector,mark_deleted,consolidate,compact,append}_<config> for the eight
// plain configs f16_r{8,16,32,64}_{l2,ip} (ffi/jasper_ffi_common.cuh:39-47,
// 787-796) and the config-agnostic jasper_free_graph / get_n_vectors /
// get_n_tombstoned / get_n_live / reserve_ids / get_dim
// (ffi/jasper_ffi_plain.cu:126-131), with the same argument lists, and the
// nine directional ops jasper_{construct_directional,build_lsh,build_pq,
// directional_search,pq_search,save_directional,load_directional,
// get_vector_directional,get_directional_flags}_<config> for the sixteen
// directional configs f16_r{32,64}_{l2,ip}_k{4,16}_d{128,32678}
// (ffi/jasper_ffi_common.cuh:72-104, 798-807).  Every
// body is a thin call into the C ABI of include/jasper_b200.h, so the
// reference's own `jasper` package runs on these kernels when this module is
// installed as its lib/libjasper_ffi.so.
//
// Streams: the reference's search runs on the legacy default stream and then
// synchronises (beam_search.cuh:330); this module launches on the stream
// tvm_ffi reports for the query tensor's device (TVMFFIEnvGetStream) -- the
// stream torch is using -- and does not synchronise.
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/tvm_ffi.h>

#include <cuda_runtime.h>
#include <string>
#include <vector>

#include "jasper_b200.h"

namespace jasper_b200_ffi {

namespace ffi = tvm::ffi;

void check(int rc) {
  if (rc == JB_OK) return;
  const std::string m = jb_last_error();
  if (rc == JB_ERR_INVALID_ARGUMENT) TVM_FFI_THROW(ValueError) << m;
  if (rc == JB_ERR_INVALID_HANDLE) TVM_FFI_THROW(InternalError) << m;
  TVM_FFI_THROW(RuntimeError) << m;
}

void* stream_of(const ffi::TensorView& t) {
  DLDevice d = t.device();
  if (d.device_type != kDLCUDA) return nullptr;
  return TVMFFIEnvGetStream(d.device_type, d.device_id);
}

uint32_t row_stride(const ffi::TensorView& t) {
  return t.ndim() == 2 ? static_cast<uint32_t>(t.stride(0)) : 0u;
}

template <int R, int METRIC>
struct Ops {
  static int64_t Load(ffi::String path, int64_t dim, bool on_host) {
    int64_t h = -1;
    check(jb_graph_load(std::string(path).c_str(), uint32_t(dim), R, METRIC, on_host, &h));
    return h;
  }
  static void Save(int64_t handle, ffi::String path) {
    check(jb_graph_save(handle, std::string(path).c_str()));
  }
  static int64_t Construct(ffi::TensorView vectors, int64_t dim, double alpha,
                           int64_t workspace_budget_bytes, bool on_host) {
    int64_t h = -1;
    check(jb_graph_construct(static_cast<const uint16_t*>(vectors.data_ptr()),
                             uint64_t(vectors.size(0)), uint32_t(dim), row_stride(vectors), R,
                             METRIC, alpha, uint64_t(workspace_budget_bytes), on_host,
                             stream_of(vectors), &h));
    return h;
  }
  static void Search(int64_t handle, ffi::TensorView queries, ffi::TensorView out_indices,
                     ffi::TensorView out_distances, int64_t k, int64_t beam_width, int64_t limit,
                     bool print_throughput) {
    (void)print_throughput;
    check(jb_graph_search(handle, static_cast<const uint16_t*>(queries.data_ptr()),
                          uint64_t(queries.size(0)), row_stride(queries),
                          static_cast<int32_t*>(out_indices.data_ptr()),
                          static_cast<float*>(out_distances.data_ptr()), uint32_t(k),
                          uint32_t(beam_width), uint32_t(limit), stream_of(queries)));
  }
  static void GetVector(int64_t handle, int64_t index, ffi::TensorView out) {
    check(jb_graph_get_vector(handle, index, static_cast<uint16_t*>(out.data_ptr())));
  }
  static void MarkDeleted(int64_t handle, ffi::TensorView ids) {
    check(jb_graph_mark_deleted(handle, static_cast<const int32_t*>(ids.data_ptr()),
                                uint64_t(ids.size(0))));
  }
  static void Consolidate(int64_t, double) {
    TVM_FFI_THROW(RuntimeError) << "consolidate is not part of jasper_b200";
  }
  static void Compact(int64_t) { TVM_FFI_THROW(RuntimeError) << "compact is not part of jasper_b200"; }
  // out_ids: host int32 [n] (the reference copies its ids there with
  // cudaMemcpyDefault, ffi/jasper_ffi_common.cuh:428-431).
  static void Append(int64_t handle, ffi::TensorView vectors, double alpha,
                     ffi::TensorView out_ids) {
    const uint64_t n = uint64_t(vectors.size(0));
    std::vector<int32_t> ids(n);
    check(jb_graph_append(handle, static_cast<const uint16_t*>(vectors.data_ptr()), n,
                          row_stride(vectors), alpha, ids.data(), stream_of(vectors)));
    if (n > 0) cudaMemcpy(out_ids.data_ptr(), ids.data(), n * 4, cudaMemcpyDefault);
  }
};

// Directional configs: k_ranks is both the LSH rank count and the PQ
// subquantizer count; LE128 selects 1-byte (dim <= 128) LSH words.
template <int R, int METRIC, int KR, bool LE128>
struct DirOps {
  static void check_dim(int64_t dim) {
    if ((dim <= 128) != LE128)
      TVM_FFI_THROW(ValueError) << "dim " << dim << " does not belong to this config's dim bucket";
  }
  static int64_t Construct(ffi::TensorView vectors, int64_t dim, double alpha,
                           int64_t workspace_budget_bytes, bool on_host, bool prerotate,
                           int64_t prerotate_seed) {
    check_dim(dim);
    int64_t h = -1;
    check(jb_graph_construct_directional(
        static_cast<const uint16_t*>(vectors.data_ptr()), uint64_t(vectors.size(0)),
        uint32_t(dim), row_stride(vectors), R, METRIC, alpha, uint64_t(workspace_budget_bytes),
        on_host, prerotate, uint64_t(prerotate_seed), stream_of(vectors), &h));
    return h;
  }
  static void BuildLsh(int64_t handle, int64_t n_samples, int64_t seed) {
    check(jb_graph_build_lsh(handle, KR, uint64_t(n_samples), uint64_t(seed)));
  }
  static void BuildPq(int64_t handle, int64_t n_train, int64_t kmeans_iter, int64_t seed) {
    check(jb_graph_build_pq(handle, KR, uint64_t(n_train), uint32_t(kmeans_iter), uint64_t(seed)));
  }
  static void Run(int32_t kind, int64_t handle, ffi::TensorView queries,
                  ffi::TensorView out_indices, ffi::TensorView out_distances, int64_t k,
                  int64_t beam_width, int64_t limit) {
    check(jb_graph_directional_search(handle, kind,
                                      static_cast<const uint16_t*>(queries.data_ptr()),
                                      uint64_t(queries.size(0)), row_stride(queries),
                                      static_cast<int32_t*>(out_indices.data_ptr()),
                                      static_cast<float*>(out_distances.data_ptr()), uint32_t(k),
                                      uint32_t(beam_width), uint32_t(limit), stream_of(queries)));
  }
  static void DirectionalSearch(int64_t handle, ffi::TensorView queries,
                                ffi::TensorView out_indices, ffi::TensorView out_distances,
                                int64_t k, int64_t beam_width, int64_t limit,
                                bool print_throughput) {
    (void)print_throughput;
    Run(JB_DIR_LSH, handle, queries, out_indices, out_distances, k, beam_width, limit);
  }
  static void PqSearch(int64_t handle, ffi::TensorView queries, ffi::TensorView out_indices,
                       ffi::TensorView out_distances, int64_t k, int64_t beam_width,
                       int64_t limit, bool print_throughput) {
    (void)print_throughput;
    Run(JB_DIR_PQ, handle, queries, out_indices, out_distances, k, beam_width, limit);
  }
  static void Save(int64_t handle, ffi::String path) {
    check(jb_graph_save_directional(handle, std::string(path).c_str()));
  }
  static int64_t Load(ffi::String path, int64_t dim, bool on_host, bool prerotate,
                      int64_t prerotate_seed) {
    check_dim(dim);
    int64_t h = -1;
    check(jb_graph_load_directional(std::string(path).c_str(), uint32_t(dim), R, METRIC, KR,
                                    on_host, prerotate, uint64_t(prerotate_seed), &h));
    return h;
  }
  static void GetVector(int64_t handle, int64_t index, ffi::TensorView out) {
    check(jb_graph_get_vector(handle, index, static_cast<uint16_t*>(out.data_ptr())));
  }
  static int64_t GetFlags(int64_t handle) {
    int32_t f = 0;
    if (jb_graph_get_directional_flags(handle, &f) != JB_OK) return 0;
    return f;
  }
};

void FreeGraph(int64_t handle) { check(jb_graph_free(handle)); }

jb_graph_info Info(int64_t handle) {
  jb_graph_info info{};
  check(jb_graph_get_info(handle, &info));
  return info;
}

int64_t GetNumVectors(int64_t h) { return int64_t(Info(h).n_vectors); }
int64_t GetNumTombstoned(int64_t h) { return int64_t(Info(h).n_deleted); }
int64_t GetNumLive(int64_t h) {
  jb_graph_info i = Info(h);
  return int64_t(i.n_vectors - i.n_deleted);
}
int64_t GetDim(int64_t h) { return int64_t(Info(h).dim); }
void ReserveIds(int64_t h, ffi::TensorView out_ids, int64_t count) {
  check(jb_graph_reserve_ids(h, count, static_cast<int32_t*>(out_ids.data_ptr())));
}

}  // namespace jasper_b200_ffi

#define JB_EXPORT_CONFIG(id, R, M)                                                        \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_load_##id, (jasper_b200_ffi::Ops<R, M>::Load));         \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_construct_##id, (jasper_b200_ffi::Ops<R, M>::Construct)); \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_search_##id, (jasper_b200_ffi::Ops<R, M>::Search));     \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_save_##id, (jasper_b200_ffi::Ops<R, M>::Save));         \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_get_vector_##id, (jasper_b200_ffi::Ops<R, M>::GetVector)); \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_mark_deleted_##id,                                 \
                                (jasper_b200_ffi::Ops<R, M>::MarkDeleted));                \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_consolidate_##id,                                  \
                                (jasper_b200_ffi::Ops<R, M>::Consolidate));                \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_compact_##id, (jasper_b200_ffi::Ops<R, M>::Compact));   \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_append_##id, (jasper_b200_ffi::Ops<R, M>::Append));

JB_EXPORT_CONFIG(f16_r8_l2, 8, JB_METRIC_L2)
JB_EXPORT_CONFIG(f16_r16_l2, 16, JB_METRIC_L2)
JB_EXPORT_CONFIG(f16_r32_l2, 32, JB_METRIC_L2)
JB_EXPORT_CONFIG(f16_r64_l2, 64, JB_METRIC_L2)
JB_EXPORT_CONFIG(f16_r8_ip, 8, JB_METRIC_IP)
JB_EXPORT_CONFIG(f16_r16_ip, 16, JB_METRIC_IP)
JB_EXPORT_CONFIG(f16_r32_ip, 32, JB_METRIC_IP)
JB_EXPORT_CONFIG(f16_r64_ip, 64, JB_METRIC_IP)

TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_free_graph, jasper_b200_ffi::FreeGraph);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_get_n_vectors, jasper_b200_ffi::GetNumVectors);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_get_n_tombstoned, jasper_b200_ffi::GetNumTombstoned);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_get_n_live, jasper_b200_ffi::GetNumLive);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_reserve_ids, jasper_b200_ffi::ReserveIds);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_get_dim, jasper_b200_ffi::GetDim);

#define JB_EXPORT_DIR(id, R, M, KR, LE)                                                   \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_construct_directional_##id,                        \
                                (jasper_b200_ffi::DirOps<R, M, KR, LE>::Construct));        \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_build_lsh_##id,                                    \
                                (jasper_b200_ffi::DirOps<R, M, KR, LE>::BuildLsh));         \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_build_pq_##id,                                     \
                                (jasper_b200_ffi::DirOps<R, M, KR, LE>::BuildPq));          \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_directional_search_##id,                           \
                                (jasper_b200_ffi::DirOps<R, M, KR, LE>::DirectionalSearch)); \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_pq_search_##id,                                    \
                                (jasper_b200_ffi::DirOps<R, M, KR, LE>::PqSearch));         \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_save_directional_##id,                             \
                                (jasper_b200_ffi::DirOps<R, M, KR, LE>::Save));             \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_load_directional_##id,                             \
                                (jasper_b200_ffi::DirOps<R, M, KR, LE>::Load));             \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_get_vector_directional_##id,                       \
                                (jasper_b200_ffi::DirOps<R, M, KR, LE>::GetVector));        \
  TVM_FFI_DLL_EXPORT_TYPED_FUNC(jasper_get_directional_flags_##id,                        \
                                (jasper_b200_ffi::DirOps<R, M, KR, LE>::GetFlags));

JB_EXPORT_DIR(f16_r32_l2_k4_d128, 32, JB_METRIC_L2, 4, true)
JB_EXPORT_DIR(f16_r32_l2_k4_d32678, 32, JB_METRIC_L2, 4, false)
JB_EXPORT_DIR(f16_r64_l2_k4_d128, 64, JB_METRIC_L2, 4, true)
JB_EXPORT_DIR(f16_r64_l2_k4_d32678, 64, JB_METRIC_L2, 4, false)
JB_EXPORT_DIR(f16_r32_l2_k16_d128, 32, JB_METRIC_L2, 16, true)
JB_EXPORT_DIR(f16_r32_l2_k16_d32678, 32, JB_METRIC_L2, 16, false)
JB_EXPORT_DIR(f16_r64_l2_k16_d128, 64, JB_METRIC_L2, 16, true)
JB_EXPORT_DIR(f16_r64_l2_k16_d32678, 64, JB_METRIC_L2, 16, false)
JB_EXPORT_DIR(f16_r32_ip_k4_d128, 32, JB_METRIC_IP, 4, true)
JB_EXPORT_DIR(f16_r32_ip_k4_d32678, 32, JB_METRIC_IP, 4, false)
JB_EXPORT_DIR(f16_r64_ip_k4_d128, 64, JB_METRIC_IP, 4, true)
JB_EXPORT_DIR(f16_r64_ip_k4_d32678, 64, JB_METRIC_IP, 4, false)
JB_EXPORT_DIR(f16_r32_ip_k16_d128, 32, JB_METRIC_IP, 16, true)
JB_EXPORT_DIR(f16_r32_ip_k16_d32678, 32, JB_METRIC_IP, 16, false)
JB_EXPORT_DIR(f16_r64_ip_k16_d128, 64, JB_METRIC_IP, 16, true)
JB_EXPORT_DIR(f16_r64_ip_k16_d32678, 64, JB_METRIC_IP, 16, false)
