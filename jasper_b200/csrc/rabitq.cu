// rabitq.cu -- RaBitQ 1-bit codes: the reference's quantizer and the codes
// of a graph's rows.
//
// quantize_kernel restates rabitq_quantize_kernel<1, TILE_SIZE = 4>
// (include/jasper/rabitq/quantize.cuh:184-290) with the same lane layout: a
// 4-lane tile per row, lane t taking coordinates t, t+4, ...; residual
// r = x - c; partial sums with one fma per coordinate; the tile reduction of
// cg::reduce (xor 2, then xor 1); code bit = r >= 0 (at 1 bit per dimension
// the reference's t_const rounding always yields 0, so only the sign
// survives); factors
//   L2: f_add = |r|^2 + 2 |r|^2 <c, xu> / <r, xu>,  f_rescale = -2 |r| / ipn
//   IP: f_add = 1 - <r, c> + |r|^2 <c, xu> / <r, xu>, f_rescale = -|r| / ipn
// with xu = code - 1/2 and ipn = sum 0.5 |r_i| / |r|.  The node store is the
// reference's array of structs (layout.cuh:42-116): ceil(dim / 8) code bytes
// padded to 4, then f_add and f_rescale as f32.  For a graph's own rows the
// kernel also writes each row's estimate error scale (used by the search's
// RaBitQ candidate filter; the reference has no such output).
//
// jb_rabitq_quantize also restates the reference's rotations in fp32: rows
// by P^T (rotate_data_vec, OP_T) and the centroid by P (rotate_single_
// data_vec, OP_N), exactly as the reference applies them.
#include <cuda_fp16.h>
#include <stdexcept>
#include <string>
#include "jb_common.cuh"
#include "rabitq.cuh"

namespace jb {
namespace {

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
  }
}

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ float tile4_reduce(float v, unsigned mask) {
  v = __fadd_rn(v, __shfl_xor_sync(mask, v, 2));
  v = __fadd_rn(v, __shfl_xor_sync(mask, v, 1));
  return v;
}

// Column means in double, rows in order (one thread per coordinate).
__global__ void centroid_kernel(const uint16_t* __restrict__ vec, uint64_t n, uint32_t dim,
                                uint32_t dpad, float* __restrict__ out) {
  for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < dim; j += gridDim.x * blockDim.x) {
    double s = 0.0;
    for (uint64_t i = 0; i < n; i++) s += double(to_f(vec[i * dpad + j]));
    out[j] = float(s / double(n));
  }
}

template <typename T>
__global__ void quantize_kernel(const T* __restrict__ rows, uint64_t n, uint64_t stride,
                                uint32_t dim, const float* __restrict__ c, int ip,
                                uint8_t* __restrict__ out, uint32_t code_bytes,
                                float* __restrict__ err_out) {
  const int lane = threadIdx.x & 31, t = lane & 3;
  const unsigned mask = 0xFu << (lane & ~3);
  const uint64_t tile = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 2;
  const uint64_t ntiles = (uint64_t(gridDim.x) * blockDim.x) >> 2;
  const uint32_t node_bytes = code_bytes + 8;
  for (uint64_t i = tile; i < n; i += ntiles) {
    const T* x = rows + i * stride;
    float l2 = 0.0f;
    for (uint32_t j = t; j < dim; j += 4) {
      const float r = __fsub_rn(to_f(x[j]), c[j]);
      l2 = __fmaf_rn(r, r, l2);
    }
    const float l2_sqr = tile4_reduce(l2, mask);
    const float l2_norm = __fsqrt_rn(l2_sqr);
    float pn = 0.0f;
    for (uint32_t j = t; j < dim; j += 4) {
      const float r = __fsub_rn(to_f(x[j]), c[j]);
      pn = __fmaf_rn(0.5f, fabsf(__fdiv_rn(r, l2_norm)), pn);
    }
    const float ip_norm = tile4_reduce(pn, mask);
    float ipnorm_inv = __fdiv_rn(1.0f, ip_norm);
    if (isnan(ipnorm_inv)) ipnorm_inv = 1.0f;
    float pa = 0.0f, pb = 0.0f, pc = 0.0f;
    for (uint32_t j = t; j < dim; j += 4) {
      const float cj = c[j];
      const float r = __fsub_rn(to_f(x[j]), cj);
      const float xu = r >= 0.0f ? 0.5f : -0.5f;
      pa = __fmaf_rn(r, xu, pa);
      pb = __fmaf_rn(cj, xu, pb);
      pc = __fmaf_rn(r, cj, pc);
    }
    float ip_resi_xucb = tile4_reduce(pa, mask);
    const float ip_cent_xucb = tile4_reduce(pb, mask);
    const float ip_resi_cent = tile4_reduce(pc, mask);
    if (ip_resi_xucb == 0.0f) ip_resi_xucb = __int_as_float(0x7F800000);
    uint8_t* node = out + i * node_bytes;
    if (t == 0) {
      float f_add, f_rescale;
      if (!ip) {
        f_add = __fadd_rn(l2_sqr, __fdiv_rn(__fmul_rn(__fmul_rn(2.0f, l2_sqr), ip_cent_xucb), ip_resi_xucb));
        f_rescale = __fmul_rn(__fmul_rn(ipnorm_inv, -2.0f), l2_norm);
      } else {
        f_add = __fadd_rn(__fsub_rn(1.0f, ip_resi_cent),
                          __fdiv_rn(__fmul_rn(l2_sqr, ip_cent_xucb), ip_resi_xucb));
        f_rescale = __fmul_rn(ipnorm_inv, -l2_norm);
      }
      reinterpret_cast<float*>(node + code_bytes)[0] = f_add;
      reinterpret_cast<float*>(node + code_bytes)[1] = f_rescale;
      if (err_out != nullptr) {
        // error scale of the estimate (the search filter's bound): with
        // a = <o_bar, o> = 2 ipn / sqrt(dim), the 1-bit estimate of <r, q - c>
        // has standard error |r| |q - c| sqrt(1 - a^2) / (a sqrt(dim - 1));
        // stored without |q - c|, times 2 for L2.
        const float a = __fdiv_rn(__fmul_rn(2.0f, ip_norm), __fsqrt_rn(float(dim)));
        const float num = __fmul_rn(__fmul_rn(ip ? 1.0f : 2.0f, l2_norm),
                                    __fsqrt_rn(fmaxf(0.0f, __fsub_rn(1.0f, __fmul_rn(a, a)))));
        err_out[i] = __fdiv_rn(num, __fmul_rn(a, __fsqrt_rn(float(dim - 1))));
      }
    }
    for (uint32_t jb = t; jb < code_bytes; jb += 4) {
      uint32_t byte = 0;
#pragma unroll
      for (int b = 0; b < 8; b++) {
        const uint32_t d = jb * 8 + b;
        if (d < dim && __fsub_rn(to_f(x[d]), c[d]) >= 0.0f) byte |= 1u << b;
      }
      node[jb] = uint8_t(byte);
    }
  }
}

// y[r][i] = sum_k P[k + i d] x[r][k] (transpose = true: P^T x), or
// y[i] = sum_k P[i + k d] x[k] (transpose = false: P x), fp32.
__global__ void rotate_f32_kernel(const float* __restrict__ X, float* __restrict__ Y,
                                  const float* __restrict__ P, uint64_t n, uint32_t d,
                                  bool transpose) {
  const uint64_t total = n * d;
  for (uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t r = e / d;
    const uint32_t i = uint32_t(e % d);
    const float* x = X + r * d;
    float acc = 0.0f;
    if (transpose)
      for (uint32_t k = 0; k < d; k++) acc = __fmaf_rn(P[k + size_t(i) * d], x[k], acc);
    else
      for (uint32_t k = 0; k < d; k++) acc = __fmaf_rn(P[i + size_t(k) * d], x[k], acc);
    Y[e] = acc;
  }
}

uint32_t grid_for(uint64_t work, uint32_t block) {
  uint64_t g = (work + block - 1) / block;
  return uint32_t(g < 1 ? 1 : (g > 148 * 64 ? 148 * 64 : g));
}

}  // namespace

uint32_t rabitq_code_bytes(uint32_t dim) { return ((dim + 7) / 8 + 3) / 4 * 4; }

void rabitq_quantize_rows(const float* rows, uint64_t n, uint32_t dim, const float* rotation,
                          const float* centroid, int ip, uint8_t* out, cudaStream_t st) {
  if (n == 0) return;
  if (dim == 0) throw std::invalid_argument("dim must be > 0");
  const float* x = rows;
  const float* c = centroid;
  float* rot_rows = nullptr;
  float* rot_c = nullptr;
  if (rotation != nullptr) {
    check(cudaMallocAsync(&rot_rows, size_t(n) * dim * 4, st), "alloc rotated rows");
    check(cudaMallocAsync(&rot_c, size_t(dim) * 4, st), "alloc rotated centroid");
    rotate_f32_kernel<<<grid_for(n * dim, 256), 256, 0, st>>>(rows, rot_rows, rotation, n, dim, true);
    rotate_f32_kernel<<<grid_for(dim, 256), 256, 0, st>>>(centroid, rot_c, rotation, 1, dim, false);
    x = rot_rows;
    c = rot_c;
  }
  quantize_kernel<float><<<grid_for(n * 4, 256), 256, 0, st>>>(x, n, dim, dim, c, ip, out,
                                                               rabitq_code_bytes(dim), nullptr);
  const cudaError_t e = cudaGetLastError();
  if (rot_rows) cudaFreeAsync(rot_rows, st);
  if (rot_c) cudaFreeAsync(rot_c, st);
  check(e, "rabitq quantize launch");
}

void build_rabitq(Graph& g, cudaStream_t st) {
  if (g.n == 0) throw std::runtime_error("build_rabitq: graph is empty");
  DirArtifacts& d = g.dir;
  if (d.rq_store) cudaFree(d.rq_store);
  if (d.rq_centroid) cudaFree(d.rq_centroid);
  if (d.rq_err) cudaFree(d.rq_err);
  d.rq_store = nullptr;
  d.rq_centroid = nullptr;
  d.rq_err = nullptr;
  d.rq_code_bytes = rabitq_code_bytes(g.dim);
  d.rq_node_bytes = d.rq_code_bytes + 8;
  check(cudaMalloc(&d.rq_centroid, size_t(g.dim) * 4 + 16), "alloc rabitq centroid");
  check(cudaMalloc(&d.rq_store, size_t(g.n) * d.rq_node_bytes + 16), "alloc rabitq codes");
  check(cudaMalloc(&d.rq_err, size_t(g.n) * 4 + 16), "alloc rabitq error scales");
  centroid_kernel<<<(g.dim + 127) / 128, 128, 0, st>>>(g.vec, g.n, g.dim, g.dpad, d.rq_centroid);
  quantize_kernel<uint16_t><<<grid_for(uint64_t(g.n) * 4, 256), 256, 0, st>>>(
      g.vec, g.n, g.dpad, g.dim, d.rq_centroid, g.metric == kIP ? 1 : 0, d.rq_store,
      d.rq_code_bytes, d.rq_err);
  check(cudaGetLastError(), "rabitq build launch");
  check(cudaStreamSynchronize(st), "rabitq build");
  d.has_rabitq = true;
}

}  // namespace jb
