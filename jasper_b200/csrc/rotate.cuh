// rotate.cuh -- random orthogonal prerotation (directional graphs).
#pragma once
#include <cuda_runtime.h>
#include <vector>
#include "jb_graph.h"

namespace jb {

// Column-major d x d rotation of the reference's set_rotation_matrix.
std::vector<float> rotation_matrix_f32(int d, uint64_t seed);

// Build the fp16 rotation for g (g.dir.rotation, prerotate = true).
void set_rotation(Graph& g, uint64_t seed);

// Y = rows of X rotated by P (fp16, padded stride dpad, pad lanes zero).
void rotate_rows(const uint16_t* P, uint32_t d, uint32_t dpad, const uint16_t* X, uint16_t* Y,
                 uint64_t n, cudaStream_t st);

// Tensor-core GEMM (rotate_tc.cu): Y = rows of X times Mp^T, where Mp is the
// dpad x dpad padded rotation (row i = column i of P).  16-byte aligned
// buffers; asynchronous on st.
void rotate_rows_tc(const uint16_t* Mp, uint32_t dpad, const uint16_t* X, uint16_t* Y, uint64_t n,
                    cudaStream_t st);
// Error code recorded by a rotate_rows_tc launch whose waits timed out (0 = none).
int rotate_tc_error(bool reset);

// dpad x dpad padded K-major copy of the column-major d x d matrix P (fp16).
std::vector<uint16_t> pad_rotation(const std::vector<uint16_t>& P, uint32_t d, uint32_t dpad);

// Rotate n padded rows in place with g's matrix (tensor cores).
void rotate_rows_inplace(const Graph& g, uint16_t* rows, uint64_t n, cudaStream_t st);

}  // namespace jb
