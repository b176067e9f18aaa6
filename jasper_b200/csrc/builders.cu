// builders.cu -- directional payload builders: cross-polytope LSH edge
// sketches and calibration, PQ codebooks and edge codes, exact row norms.
//
// Each kernel restates one reference builder with one warp per unit of work:
//  * lsh_edges_kernel      <- populate_lsh (include/jasper/lsh/lsh_kernels.cuh:9-131)
//  * lsh_sample_kernel     <- accumulate_rank_sums (lsh_globals.cuh:17-158)
//  * pq_sample_kernel      <- pq_sample_residuals (pq/pq_kernels.cuh:64-106)
//  * pq_init / pq_assign / pq_accumulate / pq_finalize <- pq_kmeans_* (:112-211)
//  * pq_codes_kernel       <- pq_populate (:252-295)
//  * norms_kernel          <- pq_compute_vector_norms (:218-247)
// Differences, all deliberate: only edge slots below the edge count are
// sketched (populate_lsh walks all R slots, reading unset slots); the LSH
// calibration and k-means sums are formed in a fixed order instead of with
// float atomics, so the artifacts are reproducible run to run.  Random
// sampling calls cuRAND's Philox generator exactly as the reference does.
// Where a builder reduces over a 128-thread block, the reduction is replayed
// in the same order (lane l plays threads l, l+32, l+64, l+96).
#include <curand_kernel.h>
#include <cfloat>
#include <stdexcept>
#include <string>
#include <vector>
#include "builders.cuh"
#include "jb_common.cuh"

namespace jb {
namespace {

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
  }
}

__device__ __forceinline__ float bfly(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(kFull, v, d);
  return v;
}

// Two-level xor butterfly of a 128-thread block (part[w] = thread lane + 32 w).
__device__ __forceinline__ float block128(const float part[4], int lane) {
  float s0 = bfly(part[0]), s1 = bfly(part[1]), s2 = bfly(part[2]), s3 = bfly(part[3]);
  float v = lane == 0 ? s0 : lane == 1 ? s1 : lane == 2 ? s2 : lane == 3 ? s3 : 0.0f;
  return bfly(v);
}

__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    const uint32_t o = __shfl_xor_sync(kFull, v, d);
    v = o > v ? o : v;
  }
  return v;
}

// Δ = v − u in fp16, its sort keys in `keys` (per warp, dpad words) and the
// block-reduced Σ float(Δ)^2.  coord_bits: 7 or 15 (sketch), 15 (calibration).
__device__ float delta_keys(const __half* u, const __half* v, uint32_t dpad, uint32_t coord_bits,
                            uint32_t mag_shift, uint32_t* keys, int lane) {
  float part[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t cmask = (1u << coord_bits) - 1u;
  for (uint32_t base = 0; base < dpad; base += 128) {
#pragma unroll
    for (int w = 0; w < 4; w++) {
      const uint32_t i = base + 32 * w + lane;
      if (i < dpad) {
        const __half d = __hsub(__ldg(v + i), __ldg(u + i));
        const uint16_t bits = __half_as_ushort(d);
        const uint32_t abs_key = bits & 0x7FFFu;
        const uint32_t sign_bit = (bits >> 15) & 1u;
        keys[i] = (abs_key << mag_shift) | (sign_bit << coord_bits) | (i & cmask);
        const float f = __half2float(d);
        part[w] = __fmaf_rn(f, f, part[w]);
      }
    }
  }
  __syncwarp();
  return block128(part, lane);
}

// Arg-max of the keys, then clear the winner (one round of the reference's
// top-k loop).
__device__ uint32_t take_max(uint32_t* keys, uint32_t dpad, uint32_t coord_mask, int lane) {
  uint32_t m = 0;
  for (uint32_t i = lane; i < dpad; i += 32) m = keys[i] > m ? keys[i] : m;
  m = warp_max_u32(m);
  __syncwarp();
  if (lane == 0) keys[m & coord_mask] = 0;
  __syncwarp();
  return m;
}

__global__ void lsh_edges_kernel(GraphView g, uint32_t k_ranks, uint32_t packed_bytes,
                                 void* packed, uint16_t* mag) {
  extern __shared__ __align__(16) uint32_t keys_all[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint32_t* keys = keys_all + size_t(wid) * g.dpad;
  const uint32_t coord_bits = packed_bytes == 1 ? 7u : 15u;
  const uint32_t cmask = (1u << coord_bits) - 1u;
  const uint32_t nw = gridDim.x * (blockDim.x >> 5);
  const __half* vec = reinterpret_cast<const __half*>(g.vec);
  for (uint32_t l = blockIdx.x * (blockDim.x >> 5) + wid; l < g.n; l += nw) {
    const __half* u = vec + size_t(l) * g.dpad;
    const uint32_t cnt = min(uint32_t(g.counts[l]), g.R);
    for (uint32_t e = 0; e < cnt; e++) {
      const uint32_t nb = g.edges[size_t(l) * g.R + e];
      if (nb - g.global_offset >= g.n) continue;  // not a row of this graph: no sketch
      const __half* v = vec + size_t(nb - g.global_offset) * g.dpad;
      const float m2 = delta_keys(u, v, g.dpad, coord_bits, coord_bits + 1, keys, lane);
      for (uint32_t r = 0; r < k_ranks; r++) {
        const uint32_t best = take_max(keys, g.dpad, cmask, lane);
        if (lane == 0) {
          const size_t w = (size_t(l) * g.R + e) * k_ranks + r;
          if (packed_bytes == 1) static_cast<uint8_t*>(packed)[w] = uint8_t(best);
          else static_cast<uint16_t*>(packed)[w] = uint16_t(best);
        }
      }
      if (lane == 0) mag[size_t(l) * g.R + e] = float_to_bf16_bits(m2);
      __syncwarp();
    }
  }
}

// One calibration sample per warp: contrib[s][r] = |Δ|_(r) / |Δ|, valid[s].
__global__ void lsh_sample_kernel(GraphView g, uint32_t k_ranks, uint32_t n_samples,
                                  uint64_t seed, float* contrib, uint32_t* valid) {
  extern __shared__ __align__(16) uint32_t keys_all[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint32_t* keys = keys_all + size_t(wid) * g.dpad;
  const uint32_t nw = gridDim.x * (blockDim.x >> 5);
  const __half* vec = reinterpret_cast<const __half*>(g.vec);
  for (uint32_t s = blockIdx.x * (blockDim.x >> 5) + wid; s < n_samples; s += nw) {
    uint32_t qg = kInvalid, ng = kInvalid;
    if (lane == 0) {
      curandStatePhilox4_32_10_t rng;
      curand_init(seed, /*subsequence=*/s, /*offset=*/0, &rng);
      for (int attempt = 0; attempt < 8; ++attempt) {
        const uint32_t ql = curand(&rng) % g.n;
        const uint32_t cnt = g.counts[ql];
        if (cnt == 0) continue;
        const uint32_t e = curand(&rng) % cnt;
        const uint32_t nb = g.edges[size_t(ql) * g.R + e];
        if (nb == kInvalid || nb - g.global_offset >= g.n) continue;
        qg = ql + g.global_offset;
        ng = nb;
        break;
      }
    }
    qg = __shfl_sync(kFull, qg, 0);
    ng = __shfl_sync(kFull, ng, 0);
    bool ok = qg != kInvalid;
    float inv = 0.f;
    if (ok) {
      const float m2 = delta_keys(vec + size_t(qg - g.global_offset) * g.dpad,
                                  vec + size_t(ng - g.global_offset) * g.dpad, g.dpad, 15u, 16u,
                                  keys, lane);
      inv = rsqrtf(m2 + 1e-20f);
      if (inv > 1e9f) ok = false;
    }
    for (uint32_t r = 0; r < k_ranks; r++) {
      float cval = 0.f;
      if (ok) {
        const uint32_t best = take_max(keys, g.dpad, 0x7FFFu, lane);
        const uint16_t abs_bits = uint16_t(best >> 16);
        cval = __half2float(__ushort_as_half(abs_bits)) * inv;
      }
      if (lane == 0) contrib[size_t(s) * k_ranks + r] = cval;
    }
    if (lane == 0) valid[s] = ok ? 1u : 0u;
    __syncwarp();
  }
}

__host__ __device__ inline uint64_t pq_mix(uint64_t x, uint64_t seed) {
  // splitmix64-style finaliser of the reference's PQ seeding (pq_kernels.cuh:18-23)
  x += seed + 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__global__ void pq_sample_kernel(GraphView g, __half* X, uint32_t n_train, uint64_t seed) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const uint32_t nw = gridDim.x * (blockDim.x >> 5);
  const __half* vec = reinterpret_cast<const __half*>(g.vec);
  for (uint32_t p = blockIdx.x * (blockDim.x >> 5) + wid; p < n_train; p += nw) {
    uint32_t ql = kInvalid, nl = kInvalid;
    if (lane == 0) {
      curandStatePhilox4_32_10_t rng;
      curand_init(seed, p, 0, &rng);
      for (int attempt = 0; attempt < 8; ++attempt) {
        const uint32_t q = curand(&rng) % g.n;
        const uint32_t cnt = g.counts[q];
        if (cnt == 0) continue;
        const uint32_t e = curand(&rng) % cnt;
        const uint32_t nb = g.edges[size_t(q) * g.R + e];
        if (nb == kInvalid || nb - g.global_offset >= g.n) continue;
        ql = q;
        nl = nb - g.global_offset;
        break;
      }
    }
    ql = __shfl_sync(kFull, ql, 0);
    nl = __shfl_sync(kFull, nl, 0);
    __half* row = X + size_t(p) * g.dpad;
    for (uint32_t i = lane; i < g.dpad; i += 32)
      row[i] = ql == kInvalid ? __float2half(0.0f)
                              : __hsub(vec[size_t(nl) * g.dpad + i], vec[size_t(ql) * g.dpad + i]);
  }
}

__global__ void pq_init_kernel(const __half* X, uint32_t n_train, uint32_t dpad, uint32_t M,
                               float* C, uint64_t seed) {
  const uint32_t dsub = dpad / M;
  for (uint32_t jc = blockIdx.x; jc < M * 256; jc += gridDim.x) {
    const uint32_t j = jc / 256;
    const uint32_t r = uint32_t(pq_mix(jc, seed) % n_train);
    for (uint32_t t = threadIdx.x; t < dsub; t += blockDim.x)
      C[size_t(jc) * dsub + t] = __half2float(X[size_t(r) * dpad + size_t(j) * dsub + t]);
  }
}

// Nearest centroid of one residual sub-vector: lane c covers centroids c,
// c+32, ...; ties go to the lower index (pq_block_argmin, pq_kernels.cuh:25-58).
__device__ int nearest_centroid(const float* rj, const float* Cj, uint32_t dsub, int lane) {
  float best = FLT_MAX;
  int bi = 0x7FFFFFFF;
  for (int c = lane; c < 256; c += 32) {
    const float* cc = Cj + size_t(c) * dsub;
    float d = 0.0f;
    for (uint32_t t = 0; t < dsub; ++t) {
      const float df = rj[t] - cc[t];
      d = __fmaf_rn(df, df, d);
    }
    if (d < best || (d == best && c < bi)) { best = d; bi = c; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float od = __shfl_xor_sync(kFull, best, o);
    const int oi = __shfl_xor_sync(kFull, bi, o);
    if (od < best || (od == best && oi < bi)) { best = od; bi = oi; }
  }
  return bi;
}

__global__ void pq_assign_kernel(const __half* X, uint32_t n_train, uint32_t dpad, uint32_t M,
                                 const float* C, uint8_t* labels) {
  extern __shared__ __align__(16) float res_all[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float* res = res_all + size_t(wid) * dpad;
  const uint32_t dsub = dpad / M;
  const uint32_t nw = gridDim.x * (blockDim.x >> 5);
  for (uint32_t p = blockIdx.x * (blockDim.x >> 5) + wid; p < n_train; p += nw) {
    for (uint32_t i = lane; i < dpad; i += 32) res[i] = __half2float(X[size_t(p) * dpad + i]);
    __syncwarp();
    for (uint32_t j = 0; j < M; ++j) {
      const int b = nearest_centroid(res + size_t(j) * dsub, C + size_t(j) * 256 * dsub, dsub, lane);
      if (lane == 0) labels[size_t(p) * M + j] = uint8_t(b);
    }
    __syncwarp();
  }
}

// Mean of the points assigned to centroid (j, c), summed in point order; an
// empty centroid is reseeded from a hashed training point
// (pq_kmeans_accumulate + pq_kmeans_finalize, pq_kernels.cuh:164-211).  One
// warp per centroid: ballots over 32 labels at a time find the members in
// order, lane t keeps coordinates t, t+32, ... (dsub <= 32 * kMaxSubPerLane).
constexpr uint32_t kMaxSubPerLane = 8;

__global__ void pq_update_kernel(const __half* X, uint32_t n_train, uint32_t dpad, uint32_t M,
                                 const uint8_t* labels, float* C, uint64_t seed, uint32_t iter) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const uint32_t dsub = dpad / M;
  const uint32_t nw = gridDim.x * (blockDim.x >> 5);
  for (uint32_t jc = blockIdx.x * (blockDim.x >> 5) + wid; jc < M * 256; jc += nw) {
    const uint32_t j = jc / 256, c = jc % 256;
    float s[kMaxSubPerLane];
#pragma unroll
    for (uint32_t q = 0; q < kMaxSubPerLane; q++) s[q] = 0.f;
    uint32_t cnt = 0;
    for (uint32_t base = 0; base < n_train; base += 32) {
      const uint32_t p = base + lane;
      const bool hit = p < n_train && labels[size_t(p) * M + j] == c;
      uint32_t m = __ballot_sync(kFull, hit);
      cnt += __popc(m);
      while (m) {
        const uint32_t pp = base + (__ffs(m) - 1);
        m &= m - 1;
        const __half* xr = X + size_t(pp) * dpad + size_t(j) * dsub;
#pragma unroll
        for (uint32_t q = 0; q < kMaxSubPerLane; q++) {
          const uint32_t t = lane + 32 * q;
          if (t < dsub) s[q] += __half2float(xr[t]);
        }
      }
    }
    float* Cjc = C + size_t(jc) * dsub;
    if (cnt > 0) {
      const float inv = 1.0f / static_cast<float>(cnt);
#pragma unroll
      for (uint32_t q = 0; q < kMaxSubPerLane; q++) {
        const uint32_t t = lane + 32 * q;
        if (t < dsub) Cjc[t] = s[q] * inv;
      }
    } else {
      const uint32_t r = uint32_t(pq_mix(jc ^ (uint64_t(iter) * 0x9E3779B9u), seed) % n_train);
      const __half* xr = X + size_t(r) * dpad + size_t(j) * dsub;
      for (uint32_t t = lane; t < dsub; t += 32) Cjc[t] = __half2float(xr[t]);
    }
  }
}

__global__ void pq_codes_kernel(GraphView g, uint32_t M, const float* C, uint8_t* codes) {
  extern __shared__ __align__(16) float res_all[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float* res = res_all + size_t(wid) * g.dpad;
  const uint32_t dsub = g.dpad / M;
  const uint32_t nw = gridDim.x * (blockDim.x >> 5);
  const __half* vec = reinterpret_cast<const __half*>(g.vec);
  for (uint32_t l = blockIdx.x * (blockDim.x >> 5) + wid; l < g.n; l += nw) {
    const __half* u = vec + size_t(l) * g.dpad;
    const uint32_t cnt = min(uint32_t(g.counts[l]), g.R);
    for (uint32_t e = 0; e < cnt; e++) {
      const uint32_t nb = g.edges[size_t(l) * g.R + e];
      if (nb - g.global_offset >= g.n) continue;  // not a row of this graph: no sketch
      const __half* v = vec + size_t(nb - g.global_offset) * g.dpad;
      for (uint32_t i = lane; i < g.dpad; i += 32) res[i] = __half2float(__hsub(v[i], u[i]));
      __syncwarp();
      for (uint32_t j = 0; j < M; ++j) {
        const int b = nearest_centroid(res + size_t(j) * dsub, C + size_t(j) * 256 * dsub, dsub, lane);
        if (lane == 0) codes[size_t(l) * M * g.R + size_t(j) * g.R + e] = uint8_t(b);
      }
      __syncwarp();
    }
  }
}

__global__ void norms_kernel(GraphView g, float* norms) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const uint32_t nw = gridDim.x * (blockDim.x >> 5);
  const __half* vec = reinterpret_cast<const __half*>(g.vec);
  for (uint32_t l = blockIdx.x * (blockDim.x >> 5) + wid; l < g.n; l += nw) {
    float part[4] = {0.f, 0.f, 0.f, 0.f};
    for (uint32_t base = 0; base < g.dpad; base += 128) {
#pragma unroll
      for (int w = 0; w < 4; w++) {
        const uint32_t i = base + 32 * w + lane;
        if (i < g.dpad) {
          const float v = __half2float(vec[size_t(l) * g.dpad + i]);
          part[w] = __fmaf_rn(v, v, part[w]);
        }
      }
    }
    const float s = block128(part, lane);
    if (lane == 0) norms[l] = s;
  }
}

int sm_count() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

uint32_t grid_for(uint64_t units, uint32_t per_block) {
  uint64_t b = (units + per_block - 1) / per_block;
  const uint64_t cap = uint64_t(sm_count()) * 32;
  return uint32_t(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

void build_lsh(Graph& graph, uint32_t k_ranks, uint32_t n_samples, uint64_t seed, cudaStream_t st) {
  if (graph.n == 0) throw std::runtime_error("build_lsh: graph is empty");
  if (k_ranks == 0 || k_ranks > 16) throw std::invalid_argument("k_ranks must be in [1, 16]");
  const GraphView g = graph.view();
  DirArtifacts& d = graph.dir;
  const uint32_t packed_bytes = g.dpad <= 128 ? 1u : 2u;
  if (g.dpad > 32768) throw std::invalid_argument("LSH coordinates are limited to 15 bits");
  if (d.lsh_packed) cudaFree(d.lsh_packed);
  if (d.lsh_mag) cudaFree(d.lsh_mag);
  d.lsh_packed = nullptr;
  d.lsh_mag = nullptr;
  const size_t nw = size_t(g.n) * g.R * k_ranks;
  check(cudaMalloc(&d.lsh_packed, nw * packed_bytes + 16), "alloc lsh words");
  check(cudaMalloc(&d.lsh_mag, size_t(g.n) * g.R * 2 + 16), "alloc lsh magnitudes");
  check(cudaMemsetAsync(d.lsh_packed, 0, nw * packed_bytes, st), "clear lsh words");
  check(cudaMemsetAsync(d.lsh_mag, 0, size_t(g.n) * g.R * 2, st), "clear lsh magnitudes");
  const size_t smem = size_t(4) * g.dpad * 4;
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(lsh_edges_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    cudaFuncSetAttribute(lsh_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  }
  lsh_edges_kernel<<<grid_for(g.n, 4), 128, smem, st>>>(g, k_ranks, packed_bytes, d.lsh_packed,
                                                         d.lsh_mag);
  check(cudaGetLastError(), "lsh edges");
  // calibration
  float* contrib = nullptr;
  uint32_t* valid = nullptr;
  check(cudaMallocAsync(&contrib, size_t(n_samples) * k_ranks * 4 + 16, st), "alloc samples");
  check(cudaMallocAsync(&valid, size_t(n_samples) * 4 + 16, st), "alloc sample flags");
  lsh_sample_kernel<<<grid_for(n_samples, 4), 128, smem, st>>>(g, k_ranks, n_samples, seed, contrib,
                                                                valid);
  check(cudaGetLastError(), "lsh samples");
  std::vector<float> hc(size_t(n_samples) * k_ranks);
  std::vector<uint32_t> hv(n_samples);
  check(cudaMemcpyAsync(hc.data(), contrib, hc.size() * 4, cudaMemcpyDeviceToHost, st), "samples");
  check(cudaMemcpyAsync(hv.data(), valid, hv.size() * 4, cudaMemcpyDeviceToHost, st), "flags");
  cudaFreeAsync(contrib, st);
  cudaFreeAsync(valid, st);
  check(cudaStreamSynchronize(st), "lsh build");
  // finalize_lsh_globals (lsh_globals.cuh:160-177), sums in sample order
  std::vector<float> sum(k_ranks, 0.f);
  uint32_t n_valid = 0;
  for (uint32_t s = 0; s < n_samples; s++) {
    if (!hv[s]) continue;
    n_valid++;
    for (uint32_t r = 0; r < k_ranks; r++) sum[r] += hc[size_t(s) * k_ranks + r];
  }
  const float inv_n = 1.0f / static_cast<float>(n_valid);
  float denom = 0.0f;
  for (uint32_t r = 0; r < 16; r++) d.lsh_c[r] = 0.f;
  for (uint32_t r = 0; r < k_ranks; r++) {
    const float c = sum[r] * inv_n;
    d.lsh_c[r] = c;
    denom = std::fma(c, c, denom);
  }
  d.norm_denom = denom;
  d.k_ranks = k_ranks;
  d.packed_bytes = packed_bytes;
  d.has_lsh = true;
}

void build_pq(Graph& graph, uint32_t M, uint32_t n_train, uint32_t kmeans_iter, uint64_t seed,
              cudaStream_t st) {
  if (graph.n == 0) throw std::runtime_error("build_pq: graph is empty");
  const GraphView g = graph.view();
  if (M == 0 || g.dpad % M != 0)
    throw std::invalid_argument("build_pq: padded dim (" + std::to_string(g.dpad) +
                                ") must be divisible by M=" + std::to_string(M));
  if (n_train < 256) n_train = 256;
  const uint32_t dsub = g.dpad / M;
  if (dsub > 32 * kMaxSubPerLane)
    throw std::invalid_argument("build_pq: sub-vector length above 256");
  DirArtifacts& d = graph.dir;
  if (d.pq_centroids) cudaFree(d.pq_centroids);
  if (d.pq_codes) cudaFree(d.pq_codes);
  if (d.norms) cudaFree(d.norms);
  d.pq_centroids = nullptr; d.pq_codes = nullptr; d.norms = nullptr;
  check(cudaMalloc(&d.pq_centroids, size_t(M) * 256 * dsub * 4), "alloc centroids");
  check(cudaMalloc(&d.pq_codes, size_t(g.n) * g.R * M + 16), "alloc codes");
  check(cudaMalloc(&d.norms, size_t(g.n) * 4 + 16), "alloc norms");
  check(cudaMemsetAsync(d.pq_codes, 0, size_t(g.n) * g.R * M, st), "clear codes");
  __half* X = nullptr;
  uint8_t* labels = nullptr;
  check(cudaMallocAsync(&X, size_t(n_train) * g.dpad * 2, st), "alloc training residuals");
  check(cudaMallocAsync(&labels, size_t(n_train) * M, st), "alloc labels");
  pq_sample_kernel<<<grid_for(n_train, 4), 128, 0, st>>>(g, X, n_train, seed);
  const uint64_t init_seed = seed ^ 0xA5A5A5A5ull;
  pq_init_kernel<<<M * 256, 128, 0, st>>>(X, n_train, g.dpad, M, d.pq_centroids, init_seed);
  const size_t smem = size_t(4) * g.dpad * 4;
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(pq_assign_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    cudaFuncSetAttribute(pq_codes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  }
  for (uint32_t it = 0; it < kmeans_iter; ++it) {
    pq_assign_kernel<<<grid_for(n_train, 4), 128, smem, st>>>(X, n_train, g.dpad, M,
                                                             d.pq_centroids, labels);
    pq_update_kernel<<<(M * 256 + 3) / 4, 128, 0, st>>>(X, n_train, g.dpad, M, labels,
                                                         d.pq_centroids, init_seed, it);
  }
  pq_codes_kernel<<<grid_for(g.n, 4), 128, smem, st>>>(g, M, d.pq_centroids, d.pq_codes);
  norms_kernel<<<grid_for(g.n, 4), 128, 0, st>>>(g, d.norms);
  check(cudaGetLastError(), "pq build");
  cudaFreeAsync(X, st);
  cudaFreeAsync(labels, st);
  check(cudaStreamSynchronize(st), "pq build");
  d.pq_m = M;
  d.pq_dsub = dsub;
  d.has_pq = true;
}

}  // namespace jb
