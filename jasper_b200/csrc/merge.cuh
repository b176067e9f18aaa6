// merge.cuh -- merge of per-shard top-k lists (range-sharded search).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace jb {

// shard lists: shard s, query q at s * shard_stride + q * k (k entries);
// unfilled slots carry id -1 / dist 1e30 and sort last.  Output: the k
// smallest by (distance, id) per query.
void launch_merge_topk(const int32_t* shard_idx, const float* shard_dist, uint32_t n_shards,
                       uint64_t nq, uint32_t k, uint64_t shard_stride, int32_t* out_idx,
                       float* out_dist, cudaStream_t stream);

}  // namespace jb
