// rotate.cu -- random orthogonal prerotation of rows (directional graphs).
//
// Matrix: the reference's set_rotation_matrix
// (include/jasper/rotation/rotation.cuh:27-110): a d x d matrix of
// std::normal_distribution<float> draws from std::mt19937_64(seed), filled
// column by column, Householder QR in float, Q's columns sign-fixed so R's
// diagonal is positive, stored column-major and converted to fp16.  Same
// algorithm and the same float operation order here, so the matrix is
// bit-identical under the same standard library.
//
// Product (rotate_rows: a SIMT tiled GEMM kept as the reference for the
// tensor-core kernel in rotate_tc.cu, which rotate_rows_inplace uses): every
// row x (padded, fp16) becomes y = P^T x, i.e.
// y_i = sum_k P[k + i * d] x_k, accumulated in fp32 and rounded to fp16 --
// the reference's cublasGemmEx(OP_T, OP_N, ...) with fp16 I/O and fp32
// compute (construct.cuh:1077-1089, rotation.cuh:122-151).  Accumulation
// order differs from cuBLAS, so rotated values may differ in the last fp16
// bit; tests compare with a tolerance.
#include <cuda_fp16.h>
#include <cmath>
#include <cstring>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>
#include "jb_graph.h"
#include "rotate.cuh"

namespace jb {

void householder_qr_f32(int d, float* A, float* Q) {
  std::memset(Q, 0, sizeof(float) * size_t(d) * d);
  for (int i = 0; i < d; i++) Q[i + i * d] = 1.0f;
  std::vector<float> v(d);
  for (int k = 0; k < d; k++) {
    float norm_sq = 0;
    for (int i = k; i < d; i++) {
      v[i] = A[i + k * d];
      norm_sq += v[i] * v[i];
    }
    const float norm = std::sqrt(norm_sq);
    if (norm < 1e-12f) continue;
    const float sign = (A[k + k * d] >= 0) ? 1.0f : -1.0f;
    v[k] += sign * norm;
    float v_norm_sq = 0;
    for (int i = k; i < d; i++) v_norm_sq += v[i] * v[i];
    const float tau = 2.0f / v_norm_sq;
    for (int j = k; j < d; j++) {
      float dot = 0;
      for (int i = k; i < d; i++) dot += v[i] * A[i + j * d];
      for (int i = k; i < d; i++) A[i + j * d] -= tau * v[i] * dot;
    }
    for (int j = 0; j < d; j++) {
      float dot = 0;
      for (int i = k; i < d; i++) dot += v[i] * Q[i + j * d];
      for (int i = k; i < d; i++) Q[i + j * d] -= tau * v[i] * dot;
    }
  }
}

std::vector<float> rotation_matrix_f32(int d, uint64_t seed) {
  std::mt19937_64 rng(seed);
  std::normal_distribution<float> N(0, 1);
  std::vector<float> A(size_t(d) * d);
  for (int j = 0; j < d; j++)
    for (int i = 0; i < d; i++) A[i + size_t(j) * d] = N(rng);
  std::vector<float> Q(size_t(d) * d);
  householder_qr_f32(d, A.data(), Q.data());
  for (int i = 0; i < d; i++)
    if (A[i + size_t(i) * d] < 0.0f)
      for (int j = 0; j < d; j++) Q[j + size_t(i) * d] *= -1.0f;
  return Q;  // column-major P
}

namespace {

constexpr int kTileRows = 64;  // rows per block
constexpr int kTileCols = 64;  // output coordinates per block
constexpr int kTileK = 32;

// Y[r][i] = sum_k P[k + i d] X[r][k]; X, Y padded rows (stride dpad).
__global__ void __launch_bounds__(256) rotate_kernel(const uint16_t* __restrict__ X,
                                                     uint16_t* __restrict__ Y,
                                                     const uint16_t* __restrict__ P, uint32_t n,
                                                     uint32_t d, uint32_t dpad) {
  __shared__ float xs[kTileRows][kTileK + 1];
  __shared__ float ps[kTileK][kTileCols + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 16 threads, 4 x 4 outputs each
  const uint32_t r0 = blockIdx.x * kTileRows, c0 = blockIdx.y * kTileCols;
  float acc[4][4] = {};
  const __half* Xh = reinterpret_cast<const __half*>(X);
  const __half* Ph = reinterpret_cast<const __half*>(P);
  for (uint32_t k0 = 0; k0 < d; k0 += kTileK) {
    for (int t = threadIdx.x; t < kTileRows * kTileK; t += 256) {
      const int rr = t / kTileK, kk = t % kTileK;
      const uint32_t r = r0 + rr, kx = k0 + kk;
      xs[rr][kk] = (r < n && kx < d) ? __half2float(Xh[size_t(r) * dpad + kx]) : 0.f;
    }
    for (int t = threadIdx.x; t < kTileK * kTileCols; t += 256) {
      const int kk = t / kTileCols, cc = t % kTileCols;
      const uint32_t kx = k0 + kk, c = c0 + cc;
      ps[kk][cc] = (kx < d && c < d) ? __half2float(Ph[kx + size_t(c) * d]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kTileK; kk++) {
      float xv[4], pv[4];
#pragma unroll
      for (int a = 0; a < 4; a++) xv[a] = xs[ty * 4 + a][kk];
#pragma unroll
      for (int b = 0; b < 4; b++) pv[b] = ps[kk][tx * 4 + b];
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) acc[a][b] = fmaf(xv[a], pv[b], acc[a][b]);
    }
    __syncthreads();
  }
  __half* Yh = reinterpret_cast<__half*>(Y);
#pragma unroll
  for (int a = 0; a < 4; a++) {
    const uint32_t r = r0 + ty * 4 + a;
    if (r >= n) continue;
#pragma unroll
    for (int b = 0; b < 4; b++) {
      const uint32_t c = c0 + tx * 4 + b;
      if (c < d) Yh[size_t(r) * dpad + c] = __float2half_rn(acc[a][b]);
    }
  }
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
  }
}

}  // namespace

std::vector<uint16_t> pad_rotation(const std::vector<uint16_t>& P, uint32_t d, uint32_t dpad) {
  std::vector<uint16_t> M(size_t(dpad) * dpad, 0);
  for (uint32_t i = 0; i < d; i++)
    for (uint32_t k = 0; k < d; k++) M[size_t(i) * dpad + k] = P[k + size_t(i) * d];
  return M;
}

void set_rotation(Graph& g, uint64_t seed) {
  std::vector<float> P = rotation_matrix_f32(int(g.dim), seed);
  std::vector<uint16_t> Ph(P.size());
  for (size_t i = 0; i < P.size(); i++) {
    const __half h = __float2half_rn(P[i]);
    Ph[i] = *reinterpret_cast<const uint16_t*>(&h);
  }
  const std::vector<uint16_t> Mp = pad_rotation(Ph, g.dim, g.dpad);
  if (g.dir.rotation) cudaFree(g.dir.rotation);
  if (g.dir.rotation_pad) cudaFree(g.dir.rotation_pad);
  g.dir.rotation = nullptr;
  g.dir.rotation_pad = nullptr;
  check(cudaMalloc(&g.dir.rotation, Ph.size() * 2), "alloc rotation");
  check(cudaMemcpy(g.dir.rotation, Ph.data(), Ph.size() * 2, cudaMemcpyHostToDevice), "rotation");
  check(cudaMalloc(&g.dir.rotation_pad, Mp.size() * 2), "alloc padded rotation");
  check(cudaMemcpy(g.dir.rotation_pad, Mp.data(), Mp.size() * 2, cudaMemcpyHostToDevice),
        "padded rotation");
  g.dir.prerotate = true;
  g.dir.rotation_seed = seed;
}

void rotate_rows(const uint16_t* P, uint32_t d, uint32_t dpad, const uint16_t* X, uint16_t* Y,
                 uint64_t n, cudaStream_t st) {
  if (n == 0) return;
  if (dpad != d) check(cudaMemsetAsync(Y, 0, size_t(n) * dpad * 2, st), "clear rotated pad");
  const dim3 grid(uint32_t((n + kTileRows - 1) / kTileRows), (d + kTileCols - 1) / kTileCols);
  rotate_kernel<<<grid, 256, 0, st>>>(X, Y, P, uint32_t(n), d, dpad);
  check(cudaGetLastError(), "rotate launch");
}

void rotate_rows_inplace(const Graph& g, uint16_t* rows, uint64_t n, cudaStream_t st) {
  if (n == 0) return;
  if (!g.dir.rotation) throw std::runtime_error("graph has no rotation matrix");
  void* tmp = nullptr;
  check(cudaMallocAsync(&tmp, size_t(n) * g.dpad * 2, st), "alloc rotation scratch");
  try {
    rotate_rows_tc(g.dir.rotation_pad, g.dpad, rows, static_cast<uint16_t*>(tmp), n, st);
    check(cudaStreamSynchronize(st), "rotate");
    if (const int e = rotate_tc_error(true))
      throw std::runtime_error("rotation GEMM gave up waiting (code " + std::to_string(e) + ")");
  } catch (...) {
    cudaFreeAsync(tmp, st);
    throw;
  }
  check(cudaMemcpyAsync(rows, tmp, size_t(n) * g.dpad * 2, cudaMemcpyDeviceToDevice, st),
        "rotated rows");
  check(cudaFreeAsync(tmp, st), "free rotation scratch");
}

}  // namespace jb
