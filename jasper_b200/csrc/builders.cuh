// builders.cuh -- directional payload builders (LSH sketches + calibration,
// PQ codebooks + codes + exact norms).
#pragma once
#include <cuda_runtime.h>
#include "jb_graph.h"

namespace jb {

// Fill g.dir's LSH words, magnitudes and globals (reference BuildLsh_##id:
// generate_lsh_globals + populate_edge_lsh).  Synchronous on `st`.
void build_lsh(Graph& g, uint32_t k_ranks, uint32_t n_samples, uint64_t seed, cudaStream_t st);

// Train M x 256 codebooks on sampled edge residuals, encode every edge and
// compute exact row norms (reference BuildPq_##id).  Synchronous on `st`.
void build_pq(Graph& g, uint32_t M, uint32_t n_train, uint32_t kmeans_iter, uint64_t seed,
              cudaStream_t st);

}  // namespace jb
