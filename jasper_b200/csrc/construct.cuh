// construct.cuh -- batched Vamana construction driver.
#pragma once
#include <cuda_runtime.h>
#include <vector>
#include "jb_graph.h"

namespace jb {

// Construction constants of the reference (construct.cuh:57-62 with the FFI's
// graph_construct_config<cfg, 64, 4, R, 64>, ffi/jasper_ffi_common.cuh:56-62).
constexpr uint32_t kBuildL = 64;
constexpr uint32_t kBuildLimit = 256;
constexpr uint32_t kBuildMaxResult = 256;

struct BuildWorkspace {
  uint32_t max_batch = 0;
  uint32_t* vis_idx = nullptr;     // [max_batch][256]
  float* vis_dist = nullptr;       // [max_batch][256]
  uint32_t* vis_cnt = nullptr;     // [max_batch]
  uint64_t* rev_keys = nullptr;    // [max_batch * R]
  uint64_t* rev_sorted = nullptr;  // [max_batch * R]
  uint32_t* group_starts = nullptr;
  uint32_t* deferred = nullptr;    // reverse groups left to the Gram pass
  uint32_t* counters = nullptr;    // [0] search work counter, [1] reverse group count,
                                   // [2] deferred group count
  void* sort_tmp = nullptr;        // semisort counts: [256][blocks of 4096 pairs], then 256 totals
  size_t sort_tmp_bytes = 0;
};

// The batch cap ConstructGraph derives from the workspace budget.
uint32_t reference_max_batch_size(uint64_t budget_bytes, uint32_t n, uint32_t R);

void workspace_allocate(BuildWorkspace& ws, uint32_t max_batch, uint32_t R);
void workspace_free(BuildWorkspace& ws);

// One batch: rows [off, off + bs) (global ids), stream-ordered.
void process_batch(Graph& g, BuildWorkspace& ws, uint32_t off, uint32_t bs, float alpha,
                   cudaStream_t stream);

// Live append of `count` rows (host or device, row stride `stride` elements):
// returns their stable ids.  Synchronises `stream`.
std::vector<uint32_t> graph_append(Graph& g, const uint16_t* rows, uint64_t count,
                                   uint32_t stride, float alpha, cudaStream_t stream);

// Whole build over the rows already uploaded to g (edge counts zero).
void construct_graph(Graph& g, float alpha, uint32_t max_batch, cudaStream_t stream);

}  // namespace jb
