// search.cuh -- launch interface of the warp-per-query beam search.
#pragma once
#include <cuda_runtime.h>
#include "jb_graph.h"

namespace jb {

struct SearchArgs {
  GraphView g;
  // Query rows: either `queries` ([nq][g.dpad] fp16, 16-byte aligned rows) or,
  // when use_range, graph rows [query_start, query_start + nq) (the build).
  const uint16_t* queries;
  int use_range;
  uint32_t query_start;
  uint32_t nq;
  uint32_t k;
  uint32_t bw;
  uint32_t limit;
  uint32_t max_result_size;
  int32_t* out_idx;   // [nq][k] or null
  float* out_dist;    // [nq][k] or null
  uint32_t* vis_idx;  // [nq][max_result_size] expansion order, or null
  float* vis_dist;
  uint32_t* vis_cnt;  // [nq]
  uint32_t* work_counter;  // one zeroed uint32 per launch (dynamic query scheduling)
  uint32_t* stats;         // optional [nq][5]: expansions, sum of degrees, distance evals,
                           // visited-table resets, first-time distance evals
  uint32_t* seen_bits;     // optional zeroed [nq][ceil(n / 32)] bitmap; with it stats[4]
                           // counts each distinct row once (the roofline's numerator)
  // Optional RaBitQ candidate filter (rq_on): with the beam full, a new
  // neighbour whose estimate minus rq_margin * |q - c| * rq_err[v] exceeds
  // the beam's worst exact distance is skipped without reading its row.
  int rq_on;
  const uint8_t* rq_store;   // [n][rq_node_bytes]: code bits, f_add, f_rescale
  uint32_t rq_node_bytes, rq_code_bytes;
  const float* rq_centroid;  // [dim]
  const float* rq_err;       // [n]
  float rq_margin;
  // Optional prerotation of the queries (not of the use_range rows): dpad x
  // dpad fp16, row i = column i of P; the kernel rotates each query in its
  // prologue.  Needs dpad <= kFusedRotationMaxDpad.
  const uint16_t* rot_pad;
  // Queries in page-locked host memory (read over the host link): each row
  // is read once, with 16-byte loads, into shared memory before any use.
  // Not combined with rot_pad.
  int stage_query;
};

// Largest padded dimension whose query rotation fits the prologue's scratch.
constexpr uint32_t kFusedRotationMaxDpad = 1024;

// Bytes of device scratch a search launch needs (the work counter).
constexpr size_t kSearchScratchBytes = 256;

// Enqueue the search on `stream`.  `work_counter` must point at zeroed device
// memory (the caller clears it on the same stream).  Throws on bad arguments.
void launch_search(const SearchArgs& a, cudaStream_t stream);

// Process-wide kernel choice for query searches: 0 = automatic (a CTA of 2
// warps per query when a launch has fewer than 8 queries per SM, else a warp
// per query), 1 = always a warp per query, 2 or more = always a CTA per query.
void set_search_mode(int warps_per_query);

// Number of kernel launches launch_search issues (for launch accounting).
constexpr int kSearchLaunches = 1;

}  // namespace jb
