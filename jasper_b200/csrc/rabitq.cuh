// rabitq.cuh -- RaBitQ 1-bit codes (rabitq.cu).
#pragma once
#include <cuda_runtime.h>
#include "jb_graph.h"

namespace jb {

// Code bytes of one node: ceil(dim / 8) rounded up to 4 (layout.cuh:58-63).
uint32_t rabitq_code_bytes(uint32_t dim);

// The reference's rabitq_quantize<1>: rows [n][dim] f32 (device), optional
// column-major dim x dim rotation (nullptr = none), centroid [dim] (device)
// -> out [n][code_bytes + 8] (device).  Asynchronous on st.
void rabitq_quantize_rows(const float* rows, uint64_t n, uint32_t dim, const float* rotation,
                          const float* centroid, int ip, uint8_t* out, cudaStream_t st);

// Codes of g's own rows (already prerotated when the graph was built so)
// around their column mean; fills g.dir's RaBitQ fields.  Synchronous.
void build_rabitq(Graph& g, cudaStream_t st);

}  // namespace jb
