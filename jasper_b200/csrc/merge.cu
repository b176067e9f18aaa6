// merge.cu -- k-way merge of per-shard top-k lists, one warp per query.
//
// Shard s's list for query q starts at s * shard_stride + q * k (stride
// n_queries * k when the shards are stacked; larger when each shard's ids and
// distances travel interleaved in one gathered buffer).
// Each range shard returns its own top-k with global ids (shards own disjoint
// id ranges, so no id repeats).  The warp loads the n_shards * k candidates
// as (distance, id) keys, sorts them with a bitonic network in shared memory
// and writes the first k.  Empty slots (id -1, distance 1e30) sort last.
#include <stdexcept>
#include <string>
#include "jb_common.cuh"
#include "merge.cuh"

namespace jb {
namespace {

constexpr int kMergeCap = 1024;

__global__ void __launch_bounds__(128) merge_topk_kernel(const int32_t* sidx, const float* sdist,
                                                         uint32_t ns, uint64_t nq, uint32_t k,
                                                         uint64_t stride, int32_t* oidx,
                                                         float* odist) {
  __shared__ uint64_t buf[4][kMergeCap];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint64_t* a = buf[wid];
  const uint64_t nw = uint64_t(gridDim.x) * 4;
  for (uint64_t q = uint64_t(blockIdx.x) * 4 + wid; q < nq; q += nw) {
    const int total = int(ns * k);
    for (int i = lane; i < total; i += 32) {
      const uint32_t s = uint32_t(i) / k, j = uint32_t(i) % k;
      const size_t off = size_t(s) * stride + q * k + j;
      const int32_t id = sidx[off];
      a[i] = id < 0 ? kKeyMax : make_pair_key(sdist[off], uint32_t(id));
    }
    int n = 32;
    while (n < total) n <<= 1;
    for (int i = total + lane; i < n; i += 32) a[i] = kKeyMax;
    __syncwarp();
    warp_sort_smem(a, n, lane);
    for (uint32_t j = lane; j < k; j += 32) {
      const uint64_t key = a[j];
      oidx[q * k + j] = key == kKeyMax ? -1 : int32_t(pair_id(key));
      odist[q * k + j] = key == kKeyMax ? 1e30f : key_dist(key);
    }
    __syncwarp();
  }
}

}  // namespace

void launch_merge_topk(const int32_t* sidx, const float* sdist, uint32_t ns, uint64_t nq,
                       uint32_t k, uint64_t shard_stride, int32_t* oidx, float* odist,
                       cudaStream_t st) {
  if (ns == 0 || k == 0) throw std::invalid_argument("n_shards and k must be > 0");
  if (shard_stride < nq * k) throw std::invalid_argument("shard stride must be >= n_queries * k");
  if (uint64_t(ns) * k > kMergeCap) throw std::invalid_argument("n_shards * k must be <= 1024");
  uint64_t blocks = (nq + 3) / 4;
  if (blocks > 148 * 16) blocks = 148 * 16;
  merge_topk_kernel<<<uint32_t(blocks), 128, 0, st>>>(sidx, sdist, ns, nq, k, shard_stride, oidx,
                                                              odist);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("merge launch: ") + cudaGetErrorString(e));
}

}  // namespace jb
