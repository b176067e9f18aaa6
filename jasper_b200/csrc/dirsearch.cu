// dirsearch.cu -- directional beam search (cross-polytope LSH or PQ-ADC
// estimated neighbour distances) for sm_100a, one warp per query.
//
// Reproduces graph_beam_search_kernel (include/jasper/beam_search/
// graph_beam_search.cuh:55-270) with the lsh_estimator
// (directional_beam_search.cuh:31-192) and pq_estimator
// (pq_beam_search.cuh:31-201):
//  * the candidate buffer is ordered by ESTIMATED distance and seeded with the
//    medoid at estimate 0; each round pops the first unvisited entry, reads
//    that node's row once to get its exact distance (the only row read per
//    expansion), inserts it into an exact top-k frontier, appends the node's
//    neighbours with estimates computed from per-edge payloads, then
//    sort + stable merge + adjacent-id dedup + clip to beam_width;
//  * estimates of one id reached from different nodes differ, so the buffer
//    may hold several copies of an id (the reference's adjacent dedup keeps
//    them too); no visited-set shortcut is taken here, the buffer semantics
//    are the reference's exactly;
//  * the exact visit emulates the reference's 128-thread block: lane l plays
//    threads l, l+32, l+64, l+96, per-thread partial sums use the same
//    expressions (__hsub2 / __hmul2 in fp16, then fp32), and the two-level
//    xor-butterfly reduction is replayed in the same order;
//  * the PQ lookup table is built one centroid per lane: each lane forms the
//    32 lane-strided partial dot products of the reference's warp-per-centroid
//    build and adds them in that warp's butterfly order.
#include <cfloat>
#include <stdexcept>
#include <string>
#include "dirsearch.cuh"
#include "jb_common.cuh"

namespace jb {
namespace {

constexpr uint32_t kEmpty31 = 0x7FFFFFFFu;

__host__ __device__ inline size_t a16(size_t x) { return (x + 15) & ~size_t(15); }

struct DirLayout {
  size_t beam, cand, qh, qu, lut, fid, fdist, total;
};

__host__ __device__ inline DirLayout dir_layout(uint32_t bwcap, uint32_t dpad, int kind,
                                                uint32_t pq_m, uint32_t k) {
  DirLayout L;
  size_t o = 0;
  const size_t cap = bwcap + 64;
  L.beam = o; o += a16(2 * cap * 8);
  L.cand = o; o += 64 * 8;
  L.qh = o; o += a16(size_t(dpad) * 2);
  L.qu = o; o += a16(size_t(dpad) * 2);
  L.lut = o; o += kind == kDirPq ? a16(size_t(pq_m) * 256 * 4) : 0;
  L.fid = o; o += a16(size_t(k) * 4);
  L.fdist = o; o += a16(size_t(k) * 4);
  L.total = o;
  return L;
}

__device__ __forceinline__ float butterfly32(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(kFull, v, d);
  return v;
}

// The reference's block reduction of 128 per-thread partials
// (beam_search_common.cuh:133-153): part[w] holds thread (lane + 32 w).
__device__ __forceinline__ float block128_sum(const float part[4], int lane) {
  float s[4];
#pragma unroll
  for (int w = 0; w < 4; w++) s[w] = butterfly32(part[w]);
  float v = lane == 0 ? s[0] : lane == 1 ? s[1] : lane == 2 ? s[2] : lane == 3 ? s[3] : 0.0f;
  return butterfly32(v);
}

// compute_qu_diff_and_exact (beam_search_common.cuh:87-154) for one warp.
template <bool IP>
__device__ float visit_exact(const uint16_t* qh, const uint16_t* urow, uint16_t* qu, uint32_t nv4,
                             int lane) {
  float part[4];
  const uint4* u_v4 = reinterpret_cast<const uint4*>(urow);
  const uint4* q_v4 = reinterpret_cast<const uint4*>(qh);
  uint4* d_v4 = reinterpret_cast<uint4*>(qu);
#pragma unroll
  for (int w = 0; w < 4; w++) {
    float local = 0.0f;
    for (uint32_t i = lane + 32 * w; i < nv4; i += 128) {
      const uint4 u = ldg16(u_v4 + i);
      const uint4 q = q_v4[i];
      uint4 d;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t qw = reinterpret_cast<const uint32_t*>(&q)[j];
        const uint32_t uw = reinterpret_cast<const uint32_t*>(&u)[j];
        const __half2 q2 = *reinterpret_cast<const __half2*>(&qw);
        const __half2 u2 = *reinterpret_cast<const __half2*>(&uw);
        if constexpr (!IP) {
          const __half2 dh = __hsub2(q2, u2);
          reinterpret_cast<uint32_t*>(&d)[j] = *reinterpret_cast<const uint32_t*>(&dh);
          const float f0 = __half2float(__low2half(dh));
          const float f1 = __half2float(__high2half(dh));
          local += f0 * f0 + f1 * f1;
        } else {
          const __half2 p2 = __hmul2(q2, u2);
          local += __half2float(__low2half(p2)) + __half2float(__high2half(p2));
        }
      }
      if constexpr (!IP) {
        if (qu != nullptr) d_v4[i] = d;
      }
    }
    part[w] = local;
  }
  return block128_sum(part, lane);
}

template <uint32_t BWCAP, int KIND, bool IP>
__global__ void __launch_bounds__(128) dir_search_kernel(DirSearchArgs a) {
  extern __shared__ __align__(16) char smem_raw[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const GraphView& g = a.g;
  const uint32_t dpad = g.dpad, nv4 = dpad / 8, R = g.R, bw = a.bw, k = a.k;
  const DirLayout L = dir_layout(BWCAP, dpad, KIND, a.pq_m, k);
  char* base = smem_raw + L.total * wid;
  uint64_t* beamA = reinterpret_cast<uint64_t*>(base + L.beam);
  uint64_t* beamB = beamA + (BWCAP + 64);
  uint64_t* cand = reinterpret_cast<uint64_t*>(base + L.cand);
  uint16_t* qh = reinterpret_cast<uint16_t*>(base + L.qh);
  uint16_t* qu = reinterpret_cast<uint16_t*>(base + L.qu);
  float* lut = reinterpret_cast<float*>(base + L.lut);
  uint32_t* fid = reinterpret_cast<uint32_t*>(base + L.fid);
  float* fdist = reinterpret_cast<float*>(base + L.fdist);
  const uint32_t lo = g.global_offset;

  for (;;) {
    uint32_t q = 0;
    if (lane == 0) q = atomicAdd(a.work_counter, 1u);
    q = __shfl_sync(kFull, q, 0);
    if (q >= a.nq) break;

    {  // query row into shared memory (raw into qu first when it is rotated here)
      const uint4* src = reinterpret_cast<const uint4*>(a.queries + size_t(q) * dpad);
      uint4* dst = reinterpret_cast<uint4*>(a.rot_pad != nullptr ? qu : qh);
      for (uint32_t c = lane; c < nv4; c += 32) dst[c] = ldg16(src + c);
    }
    __syncwarp();
    if (a.rot_pad != nullptr) {
      rotate_query_warp(qu, qh, a.rot_pad, g.dim, dpad, lane);
      __syncwarp();
    }

    float q_sq = 0.0f;
    if constexpr (KIND == kDirPq) {
      // pq_build_lut (pq_beam_search.cuh:31-60), one centroid per lane.
      const uint32_t dsub = a.pq_dsub;
      const __half* qv = reinterpret_cast<const __half*>(qh);
      for (uint32_t e = lane; e < a.pq_m * 256; e += 32) {
        const uint32_t j = e / 256;
        const float* Cj = a.centroids + size_t(e) * dsub;
        const __half* qj = qv + size_t(j) * dsub;
        float v[32];
#pragma unroll
        for (int l = 0; l < 32; l++) {
          float acc = 0.0f;
          for (uint32_t t = l; t < dsub; t += 32u) acc += static_cast<float>(qj[t]) * __ldg(Cj + t);
          v[l] = acc;
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
#pragma unroll
          for (int l = 0; l < 32; l++)
            if (l < d) v[l] = v[l] + v[l + d];
        }
        lut[e] = v[0];
      }
      if constexpr (!IP) {  // ||q||^2 over the 128-thread block
        float part[4];
#pragma unroll
        for (int w = 0; w < 4; w++) {
          float local = 0.0f;
          for (uint32_t i = lane + 32 * w; i < dpad; i += 128) {
            const float x = static_cast<float>(qv[i]);
            local += x * x;
          }
          part[w] = local;
        }
        q_sq = block128_sum(part, lane);
      }
      __syncwarp();
    }

    // Seed: medoid at estimate 0 (graph_beam_search.cuh:134-139).
    uint64_t* cur = beamA;
    uint64_t* nxt = beamB;
    if (lane == 0) cur[0] = make_key(0.0f, g.medoid);
    uint32_t cnt = 1, fc = 0;
    __syncwarp();

    uint32_t visited = 0, loop_count = 0;
    while (loop_count <= a.limit) {
      loop_count++;
      int pos = -1;
      for (uint32_t b0 = 0; b0 < cnt; b0 += 32) {
        const uint32_t i = b0 + lane;
        const bool unv = i < cnt && !key_visited(cur[i]);
        const uint32_t bal = __ballot_sync(kFull, unv);
        if (bal) { pos = int(b0) + __ffs(bal) - 1; break; }
      }
      if (pos < 0) break;
      const uint64_t fkey = cur[pos];
      __syncwarp();
      if (lane == 0) cur[pos] = fkey | 1ull;
      const uint32_t u = key_id(fkey);
      const uint16_t* urow = g.vec + size_t(u - lo) * dpad;

      float exact_u, dist_u;
      if constexpr (KIND == kDirLsh) {
        exact_u = visit_exact<IP>(qh, urow, IP ? nullptr : qu, nv4, lane);
        dist_u = IP ? -exact_u : exact_u;
      } else {
        exact_u = visit_exact<true>(qh, urow, nullptr, nv4, lane);  // <q, u>
        dist_u = IP ? -exact_u : q_sq - 2.0f * exact_u + a.norms[u - lo];
      }
      // frontier_insert_sorted (beam_search_common.cuh:158-185)
      if (lane == 0) {
        if (fc < k) {
          int j = int(fc);
          while (j > 0 && fdist[j - 1] > dist_u) { fdist[j] = fdist[j - 1]; fid[j] = fid[j - 1]; --j; }
          fdist[j] = dist_u; fid[j] = u;
          fc++;
        } else if (dist_u < fdist[k - 1]) {
          int j = int(k) - 1;
          while (j > 0 && fdist[j - 1] > dist_u) { fdist[j] = fdist[j - 1]; fid[j] = fid[j - 1]; --j; }
          fdist[j] = dist_u; fid[j] = u;
        }
      }
      fc = __shfl_sync(kFull, fc, 0);
      visited++;
      if (visited == a.max_result_size) break;
      __syncwarp();

      // Neighbours of u with estimated distances.
      const uint32_t lu = u - lo;
      const uint32_t ne = min(uint32_t(g.counts[lu]), R);
      int m = 0;
      for (uint32_t e0 = 0; e0 < ne; e0 += 32) {
        const uint32_t e = e0 + lane;
        uint32_t v = kInvalid;
        bool ok = false;
        float est = 0.0f;
        if (e < ne) {
          v = g.edges[size_t(lu) * R + e];
          ok = v - lo < g.n;
        }
        if (ok) {
          if constexpr (KIND == kDirLsh) {
            const __half* ev = reinterpret_cast<const __half*>(IP ? qh : qu);
            float dot_acc = 0.0f;
            const size_t wbase = (size_t(lu) * R + e) * a.k_ranks;
            for (uint32_t r = 0; r < a.k_ranks; ++r) {
              uint32_t coord;
              float sgn;
              if (a.packed_bytes == 1) {
                const uint8_t word = reinterpret_cast<const uint8_t*>(a.packed)[wbase + r];
                coord = word & 0x7Fu;
                sgn = (word & 0x80u) ? -1.0f : +1.0f;
              } else {
                const uint16_t word = reinterpret_cast<const uint16_t*>(a.packed)[wbase + r];
                coord = word & 0x7FFFu;
                sgn = (word & 0x8000u) ? -1.0f : +1.0f;
              }
              const float x = static_cast<float>(ev[coord]);
              dot_acc += a.c[r] * sgn * x;
            }
            const float dot_est = dot_acc * a.inv_norm_denom;
            const float mag_sq = bf16_bits_to_float(a.mag[size_t(lu) * R + e]);
            const float mag = sqrtf(mag_sq);
            if constexpr (!IP) {
              est = exact_u + mag_sq - 2.0f * mag * dot_est;
            } else {
              const float ipv = exact_u + mag * dot_est;
              est = -ipv;
            }
          } else {
            float acc = exact_u;
            for (uint32_t j = 0; j < a.pq_m; ++j)
              acc += lut[j * 256 + a.codes[size_t(lu) * a.pq_m * R + size_t(j) * R + e]];
            if constexpr (!IP) est = q_sq - 2.0f * acc + a.norms[v - lo];
            else est = -acc;
          }
        }
        const uint32_t bal = __ballot_sync(kFull, ok);
        if (ok) cand[m + __popc(bal & ((1u << lane) - 1u))] = make_key(est, v);
        m += __popc(bal);
      }
      __syncwarp();
      if (m == 0) continue;
      if (m <= 32) {
        uint64_t x = lane < m ? cand[lane] : kKeyMax;
        x = warp_sort32(x, lane);
        cand[lane] = x;
      } else {
        uint64_t x0 = lane < m ? cand[lane] : kKeyMax;
        uint64_t x1 = lane + 32 < m ? cand[lane + 32] : kKeyMax;
        warp_sort64(x0, x1, lane);
        cand[lane] = x0;
        cand[lane + 32] = x1;
      }
      __syncwarp();
      // Stable merge (buffer entries first on equal keys; the visited flag
      // never takes part), then keep the first of each run of one id.
      const uint32_t total = cnt + uint32_t(m);
      for (uint32_t i = lane; i < cnt; i += 32) {
        const uint64_t b = cur[i];
        const uint64_t bk = b & ~1ull;
        int lo2 = 0, hi2 = m;
        while (lo2 < hi2) { const int mid = (lo2 + hi2) >> 1; if (cand[mid] < bk) lo2 = mid + 1; else hi2 = mid; }
        nxt[i + lo2] = b;
      }
      for (int j = lane; j < m; j += 32) {
        const uint64_t c = cand[j];
        int lo2 = 0, hi2 = int(cnt);
        while (lo2 < hi2) { const int mid = (lo2 + hi2) >> 1; if ((cur[mid] & ~1ull) <= c) lo2 = mid + 1; else hi2 = mid; }
        nxt[j + lo2] = c;
      }
      __syncwarp();
      uint32_t w = 0;
      for (uint32_t b0 = 0; b0 < total && w < bw; b0 += 32) {
        const uint32_t i = b0 + lane;
        bool keep = false;
        uint64_t x = 0;
        if (i < total) {
          x = nxt[i];
          keep = i == 0 || key_id(nxt[i - 1]) != key_id(x);
        }
        const uint32_t bal = __ballot_sync(kFull, keep);
        const uint32_t p = w + __popc(bal & ((1u << lane) - 1u));
        if (keep && p < bw) cur[p] = x;
        w += __popc(bal);
      }
      cnt = w < bw ? w : bw;
      __syncwarp();
    }

    // Output: the exact frontier, skipping deleted rows (graph_beam_search.cuh:246-266).
    __syncwarp();
    if (lane == 0) {
      uint32_t out = 0;
      for (uint32_t i = 0; i < fc && out < k; i++) {
        const uint32_t id = fid[i];
        const uint32_t l = id - lo;
        if (l >= g.n) continue;
        if (g.deleted != nullptr && ((g.deleted[l >> 5] >> (l & 31)) & 1u)) continue;
        a.out_idx[size_t(q) * k + out] = int32_t(id);
        a.out_dist[size_t(q) * k + out] = fdist[i];
        out++;
      }
      for (; out < k; out++) {
        a.out_idx[size_t(q) * k + out] = int32_t(kEmpty31);
        a.out_dist[size_t(q) * k + out] = FLT_MAX;
      }
    }
    __syncwarp();
  }
}

template <uint32_t BWCAP, int KIND, bool IP>
void launch_t(const DirSearchArgs& a, cudaStream_t st) {
  auto kern = dir_search_kernel<BWCAP, KIND, IP>;
  const size_t per_warp = dir_layout(BWCAP, a.g.dpad, KIND, a.pq_m, a.k).total;
  int wpb = 4;
  while (wpb > 1 && per_warp * wpb > 200 * 1024) wpb--;
  if (per_warp * wpb > 220 * 1024) throw std::invalid_argument("directional search: k, beam_width or dim too large");
  const size_t smem = per_warp * wpb;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32 * wpb, smem);
  if (per_sm < 1) per_sm = 1;
  uint32_t grid = uint32_t(sms) * uint32_t(per_sm);
  const uint32_t need = (a.nq + wpb - 1) / wpb;
  if (grid > need) grid = need;
  kern<<<grid, 32 * wpb, smem, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("directional search launch: ") + cudaGetErrorString(e));
}

template <uint32_t BWCAP>
void dispatch_kind(const DirSearchArgs& a, cudaStream_t st) {
  const bool ip = a.g.metric == kIP;
  if (a.kind == kDirLsh) return ip ? launch_t<BWCAP, kDirLsh, true>(a, st) : launch_t<BWCAP, kDirLsh, false>(a, st);
  return ip ? launch_t<BWCAP, kDirPq, true>(a, st) : launch_t<BWCAP, kDirPq, false>(a, st);
}

}  // namespace

void launch_dir_search(const DirSearchArgs& a, cudaStream_t st) {
  if (a.nq == 0) return;
  if (a.g.R > 64) throw std::invalid_argument("directional search: R > 64");
  if (a.k == 0) throw std::invalid_argument("k must be > 0");
  if (a.bw == 0 || a.bw + 64 >= 2048)
    throw std::invalid_argument("beam_width " + std::to_string(a.bw) +
                                " is too large (beam_width + 64 must be < 2048)");
  if (a.kind == kDirLsh && (a.k_ranks == 0 || a.k_ranks > 16))
    throw std::invalid_argument("LSH k_ranks must be in [1, 16]");
  if (a.bw <= 64) return dispatch_kind<64>(a, st);
  if (a.bw <= 128) return dispatch_kind<128>(a, st);
  if (a.bw <= 256) return dispatch_kind<256>(a, st);
  if (a.bw <= 512) return dispatch_kind<512>(a, st);
  return dispatch_kind<2048>(a, st);
}

}  // namespace jb
