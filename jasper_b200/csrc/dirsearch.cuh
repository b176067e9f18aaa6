// dirsearch.cuh -- directional (LSH / PQ estimated) beam search.
#pragma once
#include <cuda_runtime.h>
#include "jb_graph.h"

namespace jb {

enum DirKind : int { kDirLsh = 0, kDirPq = 1 };

struct DirSearchArgs {
  GraphView g;
  int kind;
  // LSH
  uint32_t k_ranks;
  uint32_t packed_bytes;
  const void* packed;
  const uint16_t* mag;
  float c[16];
  float inv_norm_denom;
  // PQ
  uint32_t pq_m;
  uint32_t pq_dsub;
  const float* centroids;
  const uint8_t* codes;
  const float* norms;
  // queries / outputs
  const uint16_t* queries;  // [nq][dpad]
  uint32_t nq, k, bw, limit, max_result_size;
  int32_t* out_idx;
  float* out_dist;
  uint32_t* work_counter;   // zeroed
  // Optional prerotation of the queries in the kernel prologue (dpad x dpad
  // fp16, row i = column i of P), as in SearchArgs::rot_pad.
  const uint16_t* rot_pad;
};

void launch_dir_search(const DirSearchArgs& a, cudaStream_t stream);

}  // namespace jb
