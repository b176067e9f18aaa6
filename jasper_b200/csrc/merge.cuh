// merge.cuh -- merge of per-shard top-k lists (range-sharded search).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace jb {

// shard lists: [n_shards][nq][k]; unfilled slots carry id -1 / dist 1e30 and
// sort last.  Output: the k smallest by (distance, id) per query.
void launch_merge_topk(const int32_t* shard_idx, const float* shard_dist, uint32_t n_shards,
                       uint64_t nq, uint32_t k, int32_t* out_idx, float* out_dist,
                       cudaStream_t stream);

}  // namespace jb
