// search.cu -- warp-per-query Vamana beam search for sm_100a.
//
// Replaces beam_search_kernel (include/jasper/beam_search/beam_search.cuh:
// 25-259) and its device phases (device_kernels.cuh:23-288) with a design that
// returns the same top-k on the same graph:
//
//  * one warp owns one query (several warps per CTA, queries handed out by an
//    atomic counter), so every phase synchronises with __syncwarp only;
//  * the beam is a sorted array of 64-bit keys (jb_common.cuh) in shared
//    memory, double-buffered; a round merges the sorted new candidates into it
//    by rank (each element's output slot = own index + rank in the other
//    list) and clips to beam_width, which is the reference's
//    sort + dedup + clip_k on a buffer without duplicates;
//  * a per-query open-addressing hash set in shared memory remembers every id
//    whose distance was computed, so a neighbour is evaluated at most once.
//    The reference instead re-appends duplicates and removes them after a
//    full-buffer sort.  This does not change the traversal: a re-appended id
//    that is still in the beam is dropped by the reference's stable dedup
//    (the beam copy comes first and keeps its visited bit), and one that was
//    clipped before has at least beam_width strictly smaller entries ahead of
//    it and is clipped again.  When the table passes 5/8 full it is cleared
//    and refilled with the current beam, so beam members are always found;
//    forgotten clipped ids are merely recomputed, and clipped again;
//  * out-of-range neighbours (the global_offset range test of
//    device_kernels.cuh:110-121) are dropped instead of becoming visited
//    sentinels: a sentinel sorts after every real entry, is never expanded and
//    is never output, so dropping it changes nothing;
//  * the query sits in registers in the layout of the reference's 4-lane
//    distance tile: lane s of a tile holds 16-byte chunks s, s+4, ...; every
//    candidate row is gathered with 16-byte non-coherent loads, two rows per
//    tile in flight, and the per-lane sums and the tile reduction follow the
//    reference's order exactly, so distances are bit-identical.
//
// Loop bounds follow beam_search.cuh:129-203: at most limit + 1 rounds; a
// round expands the first unvisited beam entry; when the expansion count
// reaches max_result_size the loop stops before adding that node's neighbours.
#include <atomic>
#include <map>
#include <mutex>
#include <tuple>
#include <stdexcept>
#include <string>
#include <utility>
#include "jb_common.cuh"
#include "search.cuh"

namespace jb {
namespace {

constexpr uint32_t kHashEmpty = 0xFFFFFFFFu;
// The visited table is cleared (and refilled with the beam) before an
// expansion could take it past kHashFillNum / kHashFillDen of its slots.
#ifndef JB_HASH_FILL_NUM
#define JB_HASH_FILL_NUM 5
#define JB_HASH_FILL_DEN 8
#endif
constexpr uint32_t kHashFillNum = JB_HASH_FILL_NUM, kHashFillDen = JB_HASH_FILL_DEN;

// Optional per-phase cycle counters (build with -DJB_PHASE_CLOCKS; read with
// jb_debug_phase_clocks): 0 init, 1 choose, 2 neighbour list + filter,
// 3 distances, 4 candidate sort, 5 merge, 6 table reset, 7 output.
#ifdef JB_PHASE_CLOCKS
__device__ unsigned long long g_phase_clocks[8];
#define JB_CLK_DECL unsigned long long _clk_acc[8] = {0, 0, 0, 0, 0, 0, 0, 0}; long long _clk_t = clock64();
#define JB_CLK(p) { long long _n = clock64(); _clk_acc[p] += _n - _clk_t; _clk_t = _n; }
#define JB_CLK_FLUSH if (lane == 0) { for (int _i = 0; _i < 8; _i++) atomicAdd(&g_phase_clocks[_i], _clk_acc[_i]); }
#else
#define JB_CLK_DECL
#define JB_CLK(p)
#define JB_CLK_FLUSH
#endif

struct WarpSmem {
  uint64_t* beam0;
  uint64_t* beam1;
  uint64_t* cand_keys;  // [64]
  uint32_t* cand_ids;   // [64]
  uint32_t* hash;       // [1 << hbits]
  uint16_t* query;      // [dpad] (shared-memory query path only)
  float2* qpairs;       // [dpad / 2] query pairs (lane-per-row path)
};

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

// nq: chunk quads of the lane-per-row instance (template MAXC), 0 for the
// shared-memory-query instance.
__host__ __device__ inline size_t warp_smem_bytes(uint32_t bwcap, uint32_t hbits, uint32_t dpad,
                                                  uint32_t nq, uint32_t rq_words = 0) {
  const bool smem_query = nq == 0;
  size_t b = 0;
  b += 2 * sizeof(uint64_t) * bwcap;
  b += sizeof(uint64_t) * 64;
  b += sizeof(uint32_t) * 64;
  b += sizeof(uint32_t) * (size_t(1) << hbits);
  b = align16(b);
  // lane-per-row query pairs: 2 * nq chunk pairs x 8 float2
  if (smem_query) b += align16(sizeof(uint16_t) * dpad);
  else b += size_t(128) * nq + 64;  // query pairs, or the tile layout's padded chains
  b += align16(size_t(rq_words) * 4);  // RaBitQ query bit-planes (filter on)
  return b;
}

__device__ __forceinline__ WarpSmem carve(char* base, uint32_t bwcap, uint32_t hbits) {
  WarpSmem s;
  s.beam0 = reinterpret_cast<uint64_t*>(base);
  s.beam1 = s.beam0 + bwcap;
  s.cand_keys = s.beam1 + bwcap;
  s.cand_ids = reinterpret_cast<uint32_t*>(s.cand_keys + 64);
  s.hash = s.cand_ids + 64;
  size_t off = align16(reinterpret_cast<char*>(s.hash + (size_t(1) << hbits)) - base);
  s.query = reinterpret_cast<uint16_t*>(base + off);
  s.qpairs = reinterpret_cast<float2*>(base + off);
  return s;
}

// Insert id; true when it was absent.  The caller keeps the table below
// 5/8 full, so the probe sequence always ends at an empty slot.
__device__ __forceinline__ bool hash_insert(uint32_t* h, uint32_t hbits, uint32_t id) {
  const uint32_t mask = (1u << hbits) - 1u;
  uint32_t slot = (id * 0x9E3779B1u) >> (32 - hbits);
  for (uint32_t probe = 0; probe <= mask; probe++) {
    uint32_t prev = atomicCAS(&h[slot], kHashEmpty, id);
    if (prev == kHashEmpty) return true;
    if (prev == id) return false;
    slot = (slot + 1) & mask;
  }
  return true;
}

// Shared-memory query: any dpad, L2 or inner product.  Each lane loads whole
// 16-byte chunks s, s+4, ... in batches of eight before consuming them; the
// accumulation order is the reference's (chunks s, s+4, ... for L2; every
// chunk in order for IP, the words exchanged within the 4-lane tile).
template <int METRIC>
__device__ __forceinline__ float dist_smemq(const uint16_t* qs, const uint4* row, bool active,
                                            int nchunks, int s) {
  constexpr int B = 8;
  float acc = 0.f;
  if (METRIC == kL2) {
    const uint4* q4 = reinterpret_cast<const uint4*>(qs);
    for (int c0 = s; c0 < nchunks; c0 += 4 * B) {
      uint4 r[B];
#pragma unroll
      for (int u = 0; u < B; u++) {
        const int c = c0 + 4 * u;
        r[u] = (active && c < nchunks) ? ldg16(row + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < B; u++) {
        const int c = c0 + 4 * u;
        if (c < nchunks) acc = l2_chunk(q4[c], r[u], acc);
      }
    }
  } else {
    // element i belongs to lane i % 4: in chunk c lane s takes elements s and
    // s + 4, i.e. half (s & 1) of 32-bit words (s >> 1) and 2 + (s >> 1).
    // Lane s loads whole chunks c = s, s+4, ...; for every chunk, in order,
    // the tile's lanes take the words they need from the lane holding it.
    const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qs);
    const int w = s >> 1;
    const int tb = (threadIdx.x & 31) & ~3;
    for (int c0 = 0; c0 < nchunks; c0 += 4 * B) {
      uint4 r[B];
#pragma unroll
      for (int u = 0; u < B; u++) {
        const int c = c0 + 4 * u + s;
        r[u] = (active && c < nchunks) ? ldg16(row + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < B; u++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int c = c0 + 4 * u + j;  // warp-uniform
          if (c < nchunks) {
            const uint32_t x = __shfl_sync(kFull, r[u].x, tb + j);
            const uint32_t y = __shfl_sync(kFull, r[u].y, tb + j);
            const uint32_t z = __shfl_sync(kFull, r[u].z, tb + j);
            const uint32_t ww = __shfl_sync(kFull, r[u].w, tb + j);
            acc = ip_pair(q32[4 * c + w], q32[4 * c + 2 + w], w ? y : x, w ? ww : z, s, acc);
          }
        }
      }
    }
  }
  acc = tile4_sum(acc);
  return METRIC == kL2 ? acc : -acc;
}

#ifndef JB_SMEMQ2_BATCH
#define JB_SMEMQ2_BATCH 8
#endif
// Two rows per tile in one loop (independent chains interleaved), each row
// summed exactly as dist_smemq sums it.
template <int METRIC>
__device__ __forceinline__ float2 dist_smemq2(const uint16_t* qs, const uint4* row0, bool a0,
                                              const uint4* row1, bool a1, int nchunks, int s) {
  constexpr int B = JB_SMEMQ2_BATCH;  // 16-byte chunks per row in flight per lane
  float acc0 = 0.f, acc1 = 0.f;
  if (METRIC == kL2) {
    const uint4* q4 = reinterpret_cast<const uint4*>(qs);
    for (int c0 = s; c0 < nchunks; c0 += 4 * B) {
      uint4 x0[B], x1[B];
#pragma unroll
      for (int u = 0; u < B; u++) {
        const int c = c0 + 4 * u;
        x0[u] = (a0 && c < nchunks) ? ldg16(row0 + c) : make_uint4(0, 0, 0, 0);
        x1[u] = (a1 && c < nchunks) ? ldg16(row1 + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < B; u++) {
        const int c = c0 + 4 * u;
        if (c < nchunks) {
          const uint4 q = q4[c];
          acc0 = l2_chunk(q, x0[u], acc0);
          acc1 = l2_chunk(q, x1[u], acc1);
        }
      }
    }
  } else {
    const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qs);
    const int w = s >> 1;
    const int tb = (threadIdx.x & 31) & ~3;
    for (int c0 = 0; c0 < nchunks; c0 += 4 * B) {
      uint4 x0[B], x1[B];
#pragma unroll
      for (int u = 0; u < B; u++) {
        const int c = c0 + 4 * u + s;
        x0[u] = (a0 && c < nchunks) ? ldg16(row0 + c) : make_uint4(0, 0, 0, 0);
        x1[u] = (a1 && c < nchunks) ? ldg16(row1 + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < B; u++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int c = c0 + 4 * u + j;  // warp-uniform
          if (c < nchunks) {
            // the source lane sends all four words; each lane keeps its two
            const uint32_t ql = q32[4 * c + w], qh = q32[4 * c + 2 + w];
            const uint32_t a_x = __shfl_sync(kFull, x0[u].x, tb + j);
            const uint32_t a_y = __shfl_sync(kFull, x0[u].y, tb + j);
            const uint32_t a_z = __shfl_sync(kFull, x0[u].z, tb + j);
            const uint32_t a_w = __shfl_sync(kFull, x0[u].w, tb + j);
            const uint32_t b_x = __shfl_sync(kFull, x1[u].x, tb + j);
            const uint32_t b_y = __shfl_sync(kFull, x1[u].y, tb + j);
            const uint32_t b_z = __shfl_sync(kFull, x1[u].z, tb + j);
            const uint32_t b_w = __shfl_sync(kFull, x1[u].w, tb + j);
            acc0 = ip_pair(ql, qh, w ? a_y : a_x, w ? a_w : a_z, s, acc0);
            acc1 = ip_pair(ql, qh, w ? b_y : b_x, w ? b_w : b_z, s, acc1);
          }
        }
      }
    }
  }
  acc0 = tile4_sum(acc0);
  acc1 = tile4_sum(acc1);
  return METRIC == kL2 ? make_float2(acc0, acc1) : make_float2(-acc0, -acc1);
}

// ── lane-per-row distances (dpad <= 256) ───────────────────────────────────
// One lane computes a whole candidate row, reproducing the reference's four
// per-lane partial sums as two packed f32x2 chains: (s0, s1) and (s2, s3).
// L2: partial t walks 16-byte chunks t, t+4, ... with one fma per element, so
// chunks (4i, 4i+1) feed the pair (s0, s1) and (4i+2, 4i+3) feed (s2, s3),
// element by element; the query is kept negated, (x - q)^2 == (q - x)^2.
// Inner product: partial t walks elements t, t+4, ... of every chunk, so the
// half2 words (e0, e1), (e4, e5) feed (s0, s1) and (e2, e3), (e6, e7) feed
// (s2, s3) in that order.  Both end with (s0 + s2) + (s1 + s3), the
// reference's 4-lane butterfly.  L2 rows missing a chunk read zeros, which
// add nothing (fma(0, 0, acc) == acc for the non-negative partials).
//
// qpairs layout -- L2: qpairs[p * 8 + e] = (-q[2p][e], -q[2p + 1][e]) for
// chunk pairs p < 2 * NQ (zeros past the row); IP: qpairs[c * 4 + w] =
// (q[c][2w], q[c][2w + 1]) for c < nchunks <= 4 * NQ.  Both fit the 128 * NQ
// bytes warp_smem_bytes reserves for the instance.
template <int NQ, int METRIC>
__device__ __forceinline__ void build_qpairs(float2* qp, const uint16_t* qrow, int nchunks, int lane) {
  const __half* qh = reinterpret_cast<const __half*>(qrow);
  if (METRIC == kL2) {
    // every pair row_dist_lane<NQ> reads: 2 per chunk quad, zeros past the row
    const int npairs = 2 * NQ;
    for (int t = lane; t < npairs * 8; t += 32) {
      const int p = t >> 3, e = t & 7;
      const int c0 = 2 * p, c1 = 2 * p + 1;
      const float a = c0 < nchunks ? __half2float(qh[c0 * 8 + e]) : 0.f;
      const float b = c1 < nchunks ? __half2float(qh[c1 * 8 + e]) : 0.f;
      qp[t] = make_float2(-a, -b);
    }
  } else {
    for (int t = lane; t < nchunks * 4; t += 32)
      qp[t] = make_float2(__half2float(qh[2 * t]), __half2float(qh[2 * t + 1]));
  }
}

__device__ __forceinline__ float2 h2f(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

template <int NQ, int METRIC>
__device__ __forceinline__ float row_dist_lane(const float2* qp, const uint4* row, int nchunks) {
  float2 acc01 = make_float2(0.f, 0.f), acc23 = make_float2(0.f, 0.f);
#ifndef JB_LPR_GROUP
#define JB_LPR_GROUP 4
#endif
  // chunk quads per load group (4 * G 16-byte loads in flight per lane)
  constexpr int G = NQ < JB_LPR_GROUP ? NQ : JB_LPR_GROUP;
  if (METRIC == kL2) {
#pragma unroll
    for (int g0 = 0; g0 < NQ; g0 += G) {
      uint4 u[4 * G];
#pragma unroll
      for (int k = 0; k < 4 * G; k++) {
        const int c = 4 * g0 + k;
        u[k] = c < nchunks ? ldg16(row + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int qi = 0; qi < G; qi++) {
        const int i = g0 + qi;
#pragma unroll
        for (int half = 0; half < 2; half++) {
          const uint4 ua = u[4 * qi + 2 * half], ub = u[4 * qi + 2 * half + 1];
          const float2* qq = qp + (2 * i + half) * 8;
          float2& acc = half ? acc23 : acc01;
          const uint32_t aw[4] = {ua.x, ua.y, ua.z, ua.w};
          const uint32_t bw[4] = {ub.x, ub.y, ub.z, ub.w};
#pragma unroll
          for (int w = 0; w < 4; w++) {
            const float4 q2 = *reinterpret_cast<const float4*>(qq + 2 * w);
#if JB_MIXED_ADD
            float2 d0 = make_float2(add_f32_f16(aw[w], q2.x), add_f32_f16(bw[w], q2.y));
            acc = __ffma2_rn(d0, d0, acc);
            float2 d1 = make_float2(add_f32_f16(aw[w] >> 16, q2.z), add_f32_f16(bw[w] >> 16, q2.w));
            acc = __ffma2_rn(d1, d1, acc);
#else
            const float2 fa = h2f(aw[w]), fb = h2f(bw[w]);
            float2 d0 = __fadd2_rn(make_float2(fa.x, fb.x), make_float2(q2.x, q2.y));
            acc = __ffma2_rn(d0, d0, acc);
            float2 d1 = __fadd2_rn(make_float2(fa.y, fb.y), make_float2(q2.z, q2.w));
            acc = __ffma2_rn(d1, d1, acc);
#endif
          }
        }
      }
    }
  } else {
#pragma unroll
    for (int g0 = 0; g0 < 4 * NQ; g0 += 4 * G) {
      uint4 u[4 * G];
#pragma unroll
      for (int k = 0; k < 4 * G; k++) {
        const int c = g0 + k;
        u[k] = c < nchunks ? ldg16(row + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int k = 0; k < 4 * G; k++) {
        const int c = g0 + k;
        if (c < nchunks) {
          const float4 qa = *reinterpret_cast<const float4*>(qp + c * 4);
          const float4 qb = *reinterpret_cast<const float4*>(qp + c * 4 + 2);
          acc01 = __ffma2_rn(h2f(u[k].x), make_float2(qa.x, qa.y), acc01);
          acc23 = __ffma2_rn(h2f(u[k].y), make_float2(qa.z, qa.w), acc23);
          acc01 = __ffma2_rn(h2f(u[k].z), make_float2(qb.x, qb.y), acc01);
          acc23 = __ffma2_rn(h2f(u[k].w), make_float2(qb.z, qb.w), acc23);
        }
      }
    }
  }
  const float2 sum = __fadd2_rn(acc01, acc23);
  const float r = __fadd_rn(sum.x, sum.y);
  return METRIC == kL2 ? r : -r;
}

// ── tile-of-4 distances (L2, dpad <= 128) ──────────────────────────────────
// The reference's own lane layout: lane s of a 4-lane tile accumulates
// partial sum s of a row (16-byte chunks s, s+4, ..., one fma per element)
// and the tile ends with (s0 + s2) + (s1 + s3).  Here each tile carries four
// rows at once (rows t, t+8, t+16, t+24 of a 32-row round; 16 loads in
// flight per lane for dpad = 128) and packs two rows into one f32x2 chain,
// so a round of 32 rows costs the same math as lane-per-row but a short
// round (few candidates left) only costs the slots it uses.
// qtile layout: qt[s * QS + k * 8 + e] = -q[(s + 4k) * 8 + e], zeros past the
// row, QS = 8 * NQ + 4 (the pad staggers the four chains across banks).
#ifndef JB_T4_SLOTS
#define JB_T4_SLOTS 2  // rows per tile per round: 16 rows per warp, 8 loads per lane at dpad 128
#endif

template <int NQ>
__device__ __forceinline__ void build_qtile(float* qt, const uint16_t* qrow, int nchunks, int lane) {
  const __half* qh = reinterpret_cast<const __half*>(qrow);
  constexpr int QS = 8 * NQ + 4;
  for (int t = lane; t < 4 * QS; t += 32) {
    const int ch = t / QS, r = t % QS, k = r >> 3, e = r & 7;
    const int c = ch + 4 * k;
    qt[t] = (r < 8 * NQ && c < nchunks) ? -__half2float(qh[c * 8 + e]) : 0.f;
  }
}

template <int NQ>
__device__ __forceinline__ float2 tile4_pair_sum(float2 v) {
  float2 w = make_float2(__shfl_xor_sync(kFull, v.x, 2), __shfl_xor_sync(kFull, v.y, 2));
  v = __fadd2_rn(v, w);
  w = make_float2(__shfl_xor_sync(kFull, v.x, 1), __shfl_xor_sync(kFull, v.y, 1));
  return __fadd2_rn(v, w);
}

template <int NQ>
__device__ __forceinline__ float2 tile4_pair_chain(const float* qs, const uint4 (&ua)[NQ],
                                                   const uint4 (&ub)[NQ]) {
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < NQ; k++) {
    const float4 q0 = *reinterpret_cast<const float4*>(qs + k * 8);
    const float4 q1 = *reinterpret_cast<const float4*>(qs + k * 8 + 4);
    const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const uint32_t aw[4] = {ua[k].x, ua[k].y, ua[k].z, ua[k].w};
    const uint32_t bw[4] = {ub[k].x, ub[k].y, ub[k].z, ub[k].w};
#pragma unroll
    for (int w = 0; w < 4; w++) {
#if JB_MIXED_ADD
      // x + (-q) with the fp16 row element widened inside the add (exact, so
      // the same bits as converting first): one instruction per element.
      const float2 d0 = make_float2(add_f32_f16(aw[w], qv[2 * w]), add_f32_f16(bw[w], qv[2 * w]));
      acc = __ffma2_rn(d0, d0, acc);
      const float2 d1 = make_float2(add_f32_f16(aw[w] >> 16, qv[2 * w + 1]),
                                    add_f32_f16(bw[w] >> 16, qv[2 * w + 1]));
      acc = __ffma2_rn(d1, d1, acc);
#else
      const float2 fa = h2f(aw[w]), fb = h2f(bw[w]);
      const float2 d0 = __fadd2_rn(make_float2(fa.x, fb.x), make_float2(qv[2 * w], qv[2 * w]));
      acc = __ffma2_rn(d0, d0, acc);
      const float2 d1 = __fadd2_rn(make_float2(fa.y, fb.y), make_float2(qv[2 * w + 1], qv[2 * w + 1]));
      acc = __ffma2_rn(d1, d1, acc);
#endif
    }
  }
  return acc;
}

// RaBitQ estimate of the distance to node l (no reference counterpart):
// est = f_add + f_rescale * <code - 1/2, q~> + gadd (IP: minus 1), with
// <code - 1/2, q~> = 0.5 vl (2 popc(b) - dim) + 0.5 delta (2 A - S) and
// A = sum_p 2^p popc(b & plane_p) over the query's 4 bit-planes.
__device__ __forceinline__ float rabitq_est(const SearchArgs& a, uint32_t l, const uint32_t* planes,
                                            uint32_t nw, uint32_t dim, float vl, float delta, int S,
                                            float gadd, bool ip) {
  const uint8_t* node = a.rq_store + size_t(l) * a.rq_node_bytes;
  const uint32_t* cw = reinterpret_cast<const uint32_t*>(node);
  int A = 0, pb = 0;
  for (uint32_t w = 0; w < nw; w++) {
    const uint32_t b = __ldg(cw + w);
    pb += __popc(b);
    A += __popc(b & planes[w]) + (__popc(b & planes[nw + w]) << 1) +
         (__popc(b & planes[2 * nw + w]) << 2) + (__popc(b & planes[3 * nw + w]) << 3);
  }
  const float f_add = __ldg(reinterpret_cast<const float*>(node + a.rq_code_bytes));
  const float f_rescale = __ldg(reinterpret_cast<const float*>(node + a.rq_code_bytes) + 1);
  const float t1 = __fmul_rn(float(2 * pb - int(dim)), __fmul_rn(0.5f, vl));
  const float ipx = __fmaf_rn(float(2 * A - S), __fmul_rn(0.5f, delta), t1);
  const float est = __fadd_rn(__fmaf_rn(f_rescale, ipx, f_add), gadd);
  return ip ? __fsub_rn(est, 1.0f) : est;
}

__device__ __forceinline__ float warp_sum_xor(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = __fadd_rn(v, __shfl_xor_sync(kFull, v, d));
  return v;
}

// L2 prefetch hints (bit 0: rows of new candidates; bit 1: the neighbour
// list of every candidate that enters the beam, read when it is expanded).
#ifndef JB_PREFETCH
#define JB_PREFETCH 0
#endif
constexpr int kPrefetch = JB_PREFETCH;

__device__ __forceinline__ void prefetch_edges(const GraphView& g, uint32_t id) {
  const uint32_t l = id - g.global_offset;
  const char* e = reinterpret_cast<const char*>(g.edges + size_t(l) * g.R);
  for (uint32_t o = 0; o < 4 * g.R; o += 128) prefetch_l2(e + o);
  prefetch_l2(g.counts + l);
}

// Stages one query row from page-locked host memory into shared memory:
// 16-byte loads, lanes on consecutive chunks (each row crosses the host link
// once, in a few wide requests).  Plain loads: the non-coherent path is kept
// for device memory.
__device__ __forceinline__ void stage_query_row(uint16_t* dst, const uint16_t* src, int nchunks,
                                                int lane, int nthreads) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  for (int c = lane; c < nchunks; c += nthreads) d4[c] = s4[c];
}

#ifndef JB_SEARCH_MIN_BLOCKS
#define JB_SEARCH_MIN_BLOCKS 4
#endif
#ifndef JB_COUNT_MERGE
#define JB_COUNT_MERGE 32
#endif
// Up to this many kept candidates are merged by counting instead of sorting.
constexpr int kCountMerge = JB_COUNT_MERGE;
#ifndef JB_TILE_MIN_BLOCKS
#define JB_TILE_MIN_BLOCKS 6
#endif
#ifndef JB_TILE_MIN_BLOCKS_B32
#define JB_TILE_MIN_BLOCKS_B32 8
#endif
// The tile path fits in 80 registers; with a 2^11-slot visited table shared
// memory then allows 5 CTAs per SM.  Beams of at most 32 use a 2^10-slot
// table (6.4 KB per query), so 8 CTAs fit in shared memory and the kernel is
// compiled for 8 (64 registers): 32 queries in flight per SM instead of 20.
template <int MAXC, int METRIC, uint32_t BWCAP>
constexpr int search_min_blocks() {
  return (MAXC > 0 && MAXC <= 4 && METRIC == kL2)
             ? (BWCAP <= 32 ? JB_TILE_MIN_BLOCKS_B32 : JB_TILE_MIN_BLOCKS)
             : JB_SEARCH_MIN_BLOCKS;
}

template <uint32_t BWCAP, uint32_t HBITS, int MAXC, int METRIC>
__global__ void __launch_bounds__(128, search_min_blocks<MAXC, METRIC, BWCAP>())
    beam_search_warp_kernel(SearchArgs a) {
  constexpr bool kRegQ = (MAXC > 0);
#ifndef JB_NO_TILE4
  constexpr bool kTile = (MAXC > 0 && MAXC <= 4 && METRIC == kL2);
#else
  constexpr bool kTile = false;
#endif
  extern __shared__ __align__(16) char smem_raw[];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const uint32_t dpad = a.g.dpad;
  const uint32_t rq_nw = a.rq_on ? (a.g.dim + 31) / 32 : 0;
  const size_t per_warp = warp_smem_bytes(BWCAP, HBITS, dpad, MAXC, 4 * rq_nw);
  WarpSmem sm = carve(smem_raw + per_warp * wid, BWCAP, HBITS);
  uint32_t* rq_planes = reinterpret_cast<uint32_t*>(smem_raw + per_warp * wid + per_warp -
                                                    align16(size_t(4) * rq_nw * 4));
  const int tile = lane >> 2, s = lane & 3;
  const int nchunks = int(dpad / 8);
  const GraphView& g = a.g;
  const uint32_t hsize = 1u << HBITS;
  const uint32_t R = g.R;
  const uint32_t bw = a.bw;

  JB_CLK_DECL
  for (;;) {
    uint32_t q = 0;
    if (lane == 0) q = atomicAdd(a.work_counter, 1u);
    q = __shfl_sync(kFull, q, 0);
    if (q >= a.nq) break;

    const uint16_t* qrow = a.use_range
        ? g.vec + size_t(a.query_start + q - g.global_offset) * dpad
        : a.queries + size_t(q) * dpad;
    bool q_in_smem = false;
    if (a.rot_pad != nullptr) {
      // Prerotated graph: rotate the query here (rotate_query_warp).  The
      // visited table's slots are free until it is cleared below, so the raw
      // row (and, for the register layouts, the rotated one) sit there.
      uint16_t* raw = reinterpret_cast<uint16_t*>(sm.hash);
      uint16_t* rot = kRegQ ? raw + dpad : sm.query;
      const uint4* src = reinterpret_cast<const uint4*>(qrow);
      for (int c = lane; c < nchunks; c += 32) reinterpret_cast<uint4*>(raw)[c] = ldg16(src + c);
      __syncwarp();
      rotate_query_warp(raw, rot, a.rot_pad, g.dim, dpad, lane);
      __syncwarp();
      qrow = rot;
      q_in_smem = true;
    } else if (a.stage_query) {
      // Host-resident query: the register layouts build from a copy in the
      // visited table's slots (cleared below); the shared-memory layout
      // keeps it in sm.query.
      uint16_t* dst = kRegQ ? reinterpret_cast<uint16_t*>(sm.hash) : sm.query;
      stage_query_row(dst, qrow, nchunks, lane, 32);
      __syncwarp();
      qrow = dst;
      q_in_smem = true;
    }
    if constexpr (kTile) {
      build_qtile<MAXC>(reinterpret_cast<float*>(sm.qpairs), qrow, nchunks, lane);
      __syncwarp();
    } else if constexpr (kRegQ) {
      build_qpairs<MAXC, METRIC>(sm.qpairs, qrow, nchunks, lane);
      __syncwarp();
    } else if (!q_in_smem) {
      const uint4* src = reinterpret_cast<const uint4*>(qrow);
      uint4* dst = reinterpret_cast<uint4*>(sm.query);
      for (int c = lane; c < nchunks; c += 32) dst[c] = ldg16(src + c);
    }
    // RaBitQ filter: the query's 4-bit planes, offsets and centroid terms.
    float rq_vl = 0.0f, rq_delta = 0.0f, rq_gadd = 0.0f, rq_lq = 0.0f;
    int rq_S = 0;
    if (a.rq_on) {
      const __half* qv = reinterpret_cast<const __half*>(qrow);
      const uint32_t dim = g.dim;
      float vl = __int_as_float(0x7F800000), vr = -vl;
      for (uint32_t i = lane; i < dim; i += 32) {
        const float x = __half2float(qv[i]);
        vl = fminf(vl, x);
        vr = fmaxf(vr, x);
      }
#pragma unroll
      for (int d = 16; d > 0; d >>= 1) {
        vl = fminf(vl, __shfl_xor_sync(kFull, vl, d));
        vr = fmaxf(vr, __shfl_xor_sync(kFull, vr, d));
      }
      const float range = __fsub_rn(vr, vl);
      const float inv = range > 0.0f ? __fdiv_rn(15.0f, range) : 0.0f;
      int S = 0;
      for (uint32_t w = 0; w < rq_nw; w++) {
        const uint32_t i = 32 * w + lane;
        int qq = 0;
        if (i < dim) {
          qq = __float2int_rn(__fmul_rn(__fsub_rn(__half2float(qv[i]), vl), inv));
          qq = qq < 0 ? 0 : (qq > 15 ? 15 : qq);
        }
        S += qq;
#pragma unroll
        for (int p = 0; p < 4; p++) {
          const uint32_t bits = __ballot_sync(kFull, (qq >> p) & 1);
          if (lane == 0) rq_planes[p * rq_nw + w] = bits;
        }
      }
#pragma unroll
      for (int d = 16; d > 0; d >>= 1) S += __shfl_xor_sync(kFull, S, d);
      float acc_ip = 0.0f, acc_l2 = 0.0f;
      for (uint32_t i = lane; i < dim; i += 32) {
        const float x = __half2float(qv[i]);
        const float ci = __ldg(a.rq_centroid + i);
        acc_ip = __fmaf_rn(ci, x, acc_ip);
        const float dd = __fsub_rn(x, ci);
        acc_l2 = __fmaf_rn(dd, dd, acc_l2);
      }
      acc_ip = warp_sum_xor(acc_ip);
      acc_l2 = warp_sum_xor(acc_l2);
      rq_vl = vl;
      rq_delta = __fdiv_rn(range, 15.0f);
      rq_S = S;
      rq_gadd = METRIC == kIP ? -acc_ip : acc_l2;
      rq_lq = __fmul_rn(a.rq_margin, __fsqrt_rn(acc_l2));
    }
    __syncwarp();  // every read of a rotated query in the table's slots is done
    for (uint32_t i = lane; i < hsize; i += 32) sm.hash[i] = kHashEmpty;
    __syncwarp();

    uint32_t first_evals = 0;  // per lane; summed at the end (stats only)
    // Evaluate candidates sm.cand_ids[0, m) into sm.cand_keys (sorted on exit).
    uint64_t* cur = sm.beam0;
    uint64_t* nxt = sm.beam1;
    uint32_t cnt = 0;
    int pos = -1;  // beam position of the node being expanded
    // Evaluates sm.cand_ids[0, m), then keeps only candidates that can enter
    // the beam -- with the beam full, a key above its bw-th entry would land
    // past position bw in the merged order and be clipped -- and leaves them
    // sorted in sm.cand_keys.  Returns how many were kept.
    auto evaluate_and_sort = [&](int m) -> int {
      if constexpr (kTile) {
        const float* qs = reinterpret_cast<const float*>(sm.qpairs) + s * (8 * MAXC + 4);
        constexpr int SL = JB_T4_SLOTS;  // rows per tile per round
        for (int base = 0; base < m; base += 8 * SL) {
          const int nslot = min(SL, (m - base + 7) >> 3);  // warp-uniform
          uint4 u[SL][MAXC];
          uint32_t rid[SL];
#pragma unroll
          for (int i = 0; i < SL; i++) {
            const int j = base + tile + 8 * i;
            const bool act = i < nslot && j < m;
            rid[i] = act ? sm.cand_ids[j] : kInvalid;
            const uint4* row = reinterpret_cast<const uint4*>(
                g.vec + size_t(act ? rid[i] - g.global_offset : 0) * dpad);
#pragma unroll
            for (int k = 0; k < MAXC; k++) {
              const int c = s + 4 * k;
              u[i][k] = (act && c < nchunks) ? ldg16(row + c) : make_uint4(0, 0, 0, 0);
            }
          }
#pragma unroll
          for (int p = 0; p < SL / 2; p++) {
            if (2 * p >= nslot) break;
            const float2 v = tile4_pair_sum<MAXC>(tile4_pair_chain<MAXC>(qs, u[2 * p], u[2 * p + 1]));
            if (s == 0) {
#pragma unroll
              for (int h = 0; h < 2; h++) {
                const int i = 2 * p + h;
                const int j = base + tile + 8 * i;
                if (rid[i] != kInvalid) {
                  sm.cand_keys[j] = make_key(h ? v.y : v.x, rid[i]);
                  if (a.seen_bits != nullptr) {
                    uint32_t* bits = a.seen_bits + size_t(q) * ((g.n + 31) / 32);
                    const uint32_t l = rid[i] - g.global_offset;
                    if (!(atomicOr(&bits[l >> 5], 1u << (l & 31)) & (1u << (l & 31)))) first_evals++;
                  }
                }
              }
            }
          }
        }
      } else if constexpr (kRegQ) {
        // One lane per candidate row (32 rows per pass).
        for (int base = 0; base < m; base += 32) {
          const int j = base + lane;
          if (j < m) {
            const uint32_t id = sm.cand_ids[j];
            const uint4* row = reinterpret_cast<const uint4*>(g.vec + size_t(id - g.global_offset) * dpad);
            const float d = row_dist_lane<MAXC, METRIC>(sm.qpairs, row, nchunks);
            sm.cand_keys[j] = make_key(d, id);
            if (a.seen_bits != nullptr) {
              uint32_t* bits = a.seen_bits + size_t(q) * ((g.n + 31) / 32);
              const uint32_t l = id - g.global_offset;
              if (!(atomicOr(&bits[l >> 5], 1u << (l & 31)) & (1u << (l & 31)))) first_evals++;
            }
          }
        }
      } else
      for (int base = 0; base < m; base += 16) {
        const int i0 = base + tile, i1 = base + tile + 8;
        const bool a0 = i0 < m, a1 = i1 < m;
        const uint32_t id0 = a0 ? sm.cand_ids[i0] : g.global_offset;
        const uint32_t id1 = a1 ? sm.cand_ids[i1] : id0;
        const uint4* r0 = reinterpret_cast<const uint4*>(g.vec + size_t(id0 - g.global_offset) * dpad);
        const uint4* r1 = reinterpret_cast<const uint4*>(g.vec + size_t(id1 - g.global_offset) * dpad);
        const float2 dd = dist_smemq2<METRIC>(sm.query, r0, a0, r1, a1, nchunks, s);
        const float d0 = dd.x, d1 = dd.y;
        if (s == 0) {
          if (a0) sm.cand_keys[i0] = make_key(d0, id0);
          if (a1) sm.cand_keys[i1] = make_key(d1, id1);
          if (a.seen_bits != nullptr) {
            uint32_t* bits = a.seen_bits + size_t(q) * ((g.n + 31) / 32);
            const uint32_t l0 = id0 - g.global_offset, l1 = id1 - g.global_offset;
            if (a0 && !(atomicOr(&bits[l0 >> 5], 1u << (l0 & 31)) & (1u << (l0 & 31)))) first_evals++;
            if (a1 && !(atomicOr(&bits[l1 >> 5], 1u << (l1 & 31)) & (1u << (l1 & 31)))) first_evals++;
          }
        }
      }
      __syncwarp();
      JB_CLK(3)
      uint64_t v0 = lane < m ? sm.cand_keys[lane] : kKeyMax;
      uint64_t v1 = lane + 32 < m ? sm.cand_keys[lane + 32] : kKeyMax;
      if (cnt == bw) {
        const uint64_t worst = cur[bw - 1] | 1ull;  // ids differ: the flag bit never decides
        if (v0 > worst) v0 = kKeyMax;
        if (v1 > worst) v1 = kKeyMax;
      }
      const uint32_t k0 = __ballot_sync(kFull, v0 != kKeyMax);
      const uint32_t k1 = __ballot_sync(kFull, v1 != kKeyMax);
      const int kept = __popc(k0) + __popc(k1);
      __syncwarp();
      if (kept <= 32) {  // the common case: compact to one key per lane
        const uint32_t lt = (1u << lane) - 1u;
        if (v0 != kKeyMax) sm.cand_keys[__popc(k0 & lt)] = v0;
        if (v1 != kKeyMax) sm.cand_keys[__popc(k0) + __popc(k1 & lt)] = v1;
        __syncwarp();
        if (kept <= kCountMerge) return kept;  // left unsorted: merged by counting
        uint64_t v = lane < kept ? sm.cand_keys[lane] : kKeyMax;
        v = warp_sort32(v, lane);
        sm.cand_keys[lane] = v;
      } else {
        warp_sort64(v0, v1, lane);
        sm.cand_keys[lane] = v0;
        sm.cand_keys[lane + 32] = v1;
      }
      __syncwarp();
      JB_CLK(4)
      return kept;
    };

    // Seed the beam with the medoid (beam_search.cuh:114-123).
    if (lane == 0) {
      sm.cand_ids[0] = g.medoid;
      hash_insert(sm.hash, HBITS, g.medoid);
    }
    __syncwarp();
    evaluate_and_sort(1);
    if (lane == 0) cur[0] = sm.cand_keys[0];
    cnt = 1;
    uint32_t n_hash = 1;
    uint32_t expansions = 0, deg_sum = 0, evals = 1, resets = 0;
    __syncwarp();

    uint32_t loop_count = 0;
    JB_CLK(0)
    while (loop_count <= a.limit) {
      loop_count++;
      // choose_new_frontier: first unvisited entry of the sorted beam.
      pos = -1;
      for (uint32_t base = 0; base < cnt; base += 32) {
        const uint32_t i = base + lane;
        const bool unv = i < cnt && !key_visited(cur[i]);
        const uint32_t bal = __ballot_sync(kFull, unv);
        if (bal) { pos = int(base) + __ffs(bal) - 1; break; }
      }
      JB_CLK(1)
      if (pos < 0) break;
      const uint64_t fkey = cur[pos];
      __syncwarp();
      if (lane == 0) cur[pos] = fkey | 1ull;
      const uint32_t u = key_id(fkey);
      if (a.vis_idx != nullptr && lane == 0) {
        a.vis_idx[size_t(q) * a.max_result_size + expansions] = u;
        a.vis_dist[size_t(q) * a.max_result_size + expansions] = key_dist(fkey);
      }
      expansions++;
      if (expansions == a.max_result_size) break;

      // Keep the visited-distance table at most 5/8 full: clear it and refill
      // it with the beam, so beam members are always recognised.
      if (n_hash + R > kHashFillNum * (hsize / kHashFillDen)) {
        __syncwarp();
        for (uint32_t i = lane; i < hsize; i += 32) sm.hash[i] = kHashEmpty;
        __syncwarp();
        for (uint32_t i = lane; i < cnt; i += 32) hash_insert(sm.hash, HBITS, key_id(cur[i]));
        n_hash = cnt;
        resets++;
        __syncwarp();
      }
      JB_CLK(6)

      // add_frontier_out: the neighbour list of u, in-range ids not seen before.
      const uint32_t lu = u - g.global_offset;
      const uint32_t ne = g.counts[lu];
      const uint32_t* el = g.edges + size_t(lu) * R;
      // Issued together with the count load (slots past the count are masked
      // below), so the two dependent gathers overlap.
      uint32_t nb0 = lane < R ? __ldg(el + lane) : kInvalid;
      uint32_t nb1 = lane + 32 < R ? __ldg(el + lane + 32) : kInvalid;
      deg_sum += ne;
      bool f0 = (lane < ne) && (nb0 - g.global_offset < g.n) && hash_insert(sm.hash, HBITS, nb0);
      const uint32_t b0 = __ballot_sync(kFull, f0);
      bool f1 = (lane + 32 < ne) && (nb1 - g.global_offset < g.n) && hash_insert(sm.hash, HBITS, nb1);
      const uint32_t b1 = __ballot_sync(kFull, f1);
      const uint32_t lt = (1u << lane) - 1u;
      if (f0) sm.cand_ids[__popc(b0 & lt)] = nb0;
      if (f1) sm.cand_ids[__popc(b0) + __popc(b1 & lt)] = nb1;
      if constexpr ((kPrefetch & 1) != 0) {
        // the rows of every new candidate: the later distance rounds find
        // them in L2 while the first round's loads are still in flight
        if (f0 || f1) {
          const char* r0 = reinterpret_cast<const char*>(g.vec + size_t(nb0 - g.global_offset) * dpad);
          const char* r1 = reinterpret_cast<const char*>(g.vec + size_t(nb1 - g.global_offset) * dpad);
          for (uint32_t o = 0; o < 2 * dpad; o += 128) {
            if (f0) prefetch_l2(r0 + o);
            if (f1) prefetch_l2(r1 + o);
          }
        }
      }
      int m = __popc(b0) + __popc(b1);
      n_hash += m;
      __syncwarp();
      JB_CLK(2)
      if (m == 0) continue;
      if (a.rq_on && cnt == bw) {
        // RaBitQ filter: drop candidates that cannot enter the full beam.
        const float tau = key_dist(cur[bw - 1]);
        bool k0 = false, k1 = false;
        uint32_t c0 = 0, c1 = 0;
        if (lane < m) {
          c0 = sm.cand_ids[lane];
          const uint32_t l = c0 - g.global_offset;
          const float est = rabitq_est(a, l, rq_planes, rq_nw, g.dim, rq_vl, rq_delta, rq_S,
                                       rq_gadd, METRIC == kIP);
          k0 = !(__fsub_rn(est, __fmul_rn(rq_lq, __ldg(a.rq_err + l))) > tau);
        }
        if (lane + 32 < m) {
          c1 = sm.cand_ids[lane + 32];
          const uint32_t l = c1 - g.global_offset;
          const float est = rabitq_est(a, l, rq_planes, rq_nw, g.dim, rq_vl, rq_delta, rq_S,
                                       rq_gadd, METRIC == kIP);
          k1 = !(__fsub_rn(est, __fmul_rn(rq_lq, __ldg(a.rq_err + l))) > tau);
        }
        const uint32_t kb0 = __ballot_sync(kFull, k0), kb1 = __ballot_sync(kFull, k1);
        __syncwarp();
        if (k0) sm.cand_ids[__popc(kb0 & lt)] = c0;
        if (k1) sm.cand_ids[__popc(kb0) + __popc(kb1 & lt)] = c1;
        m = __popc(kb0) + __popc(kb1);
        __syncwarp();
        if (m == 0) continue;
      }
      evals += m;
      const int kept = evaluate_and_sort(m);
      if (kept == 0) continue;

      // Merge beam (cnt) and kept candidates by rank; keep the first bw.
      // A few kept candidates stay unsorted: each position is counted
      // directly (keys are distinct, so every rank is exact).
      if (BWCAP <= 32 && kept <= kCountMerge) {
        // beam of at most 32: one pass over the kept keys counts both the
        // beam entry's rank among them and the lane's own candidate's
        const uint64_t b = lane < int(cnt) ? cur[lane] : kKeyMax;
        const uint64_t c = lane < kept ? sm.cand_keys[lane] : kKeyMax;
        uint32_t rb = 0, rc = 0;
        for (int j = 0; j < kept; j++) {
          const uint64_t t = sm.cand_keys[j];
          rb += t < b;
          rc += t < c;
        }
        if (lane < int(cnt) && lane + rb < bw) nxt[lane + rb] = b;
        if (lane < kept) {
          const uint32_t p = rc + lower_rank(cur, int(cnt), c);
          if (p < bw) nxt[p] = c;
        }
      } else if (kept <= kCountMerge) {
        for (uint32_t i = lane; i < cnt; i += 32) {
          const uint64_t b = cur[i];
          uint32_t r = 0;
          for (int j = 0; j < kept; j++) r += sm.cand_keys[j] < b;
          if (i + r < bw) nxt[i + r] = b;
        }
        if (lane < kept) {
          const uint64_t c = sm.cand_keys[lane];
          uint32_t r = 0;
          for (int j = 0; j < kept; j++) r += sm.cand_keys[j] < c;
          const uint32_t p = r + lower_rank(cur, int(cnt), c);
          if (p < bw) {
            nxt[p] = c;
            if constexpr ((kPrefetch & 2) != 0) prefetch_edges(g, key_id(c));
          }
        }
      } else {
        for (uint32_t i = lane; i < cnt; i += 32) {
          const uint64_t b = cur[i];
          const uint32_t p = i + lower_rank(sm.cand_keys, kept, b);
          if (p < bw) nxt[p] = b;
        }
        for (int j = lane; j < kept; j += 32) {
          const uint64_t c = sm.cand_keys[j];
          const uint32_t p = j + lower_rank(cur, int(cnt), c);
          if (p < bw) {
            nxt[p] = c;
            if constexpr ((kPrefetch & 2) != 0) prefetch_edges(g, key_id(c));
          }
        }
      }
      cnt = min(bw, cnt + uint32_t(kept));
      uint64_t* t = cur; cur = nxt; nxt = t;
      __syncwarp();
      JB_CLK(5)
    }

    JB_CLK(1)
    // Output the first k non-deleted entries (beam_search.cuh:205-222).
    if (a.out_idx != nullptr) {
      uint32_t out = 0;
      for (uint32_t base = 0; base < cnt && out < a.k; base += 32) {
        const uint32_t i = base + lane;
        uint32_t id = 0;
        bool ok = false;
        if (i < cnt) {
          id = key_id(cur[i]);
          const uint32_t l = id - g.global_offset;
          ok = !(g.deleted != nullptr && ((g.deleted[l >> 5] >> (l & 31)) & 1u));
        }
        const uint32_t bal = __ballot_sync(kFull, ok);
        const uint32_t p = out + __popc(bal & ((1u << lane) - 1u));
        if (ok && p < a.k) {
          const uint32_t sid = g.ids_identity ? id : g.slot_to_id[id - g.global_offset];
          a.out_idx[size_t(q) * a.k + p] = int32_t(sid);
          a.out_dist[size_t(q) * a.k + p] = key_dist(cur[i]);
        }
        out += __popc(bal);
      }
      for (uint32_t p = out + lane; p < a.k; p += 32) {
        a.out_idx[size_t(q) * a.k + p] = -1;
        a.out_dist[size_t(q) * a.k + p] = 1e30f;
      }
    }
    if (a.stats != nullptr) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) first_evals += __shfl_xor_sync(kFull, first_evals, o);
    }
    if (lane == 0) {
      if (a.vis_cnt != nullptr) a.vis_cnt[q] = expansions;
      if (a.stats != nullptr) {
        a.stats[size_t(q) * 5 + 0] = expansions;
        a.stats[size_t(q) * 5 + 1] = deg_sum;
        a.stats[size_t(q) * 5 + 2] = evals;
        a.stats[size_t(q) * 5 + 3] = resets;
        a.stats[size_t(q) * 5 + 4] = a.seen_bits != nullptr ? first_evals : evals;
      }
    }
    __syncwarp();
    JB_CLK(7)
  }
  JB_CLK_FLUSH
}

// ── CTA per query (few queries per GPU) ─────────────────────────────────────
// The warp-per-query kernel needs thousands of queries to fill a B200; with
// a few hundred per GPU (a split query batch on many GPUs, or 1k wide rows)
// each query's latency decides the time.  Here one CTA of W warps owns a
// query and the warps share each expansion's candidate distances:
//   every warp     -- choose_new_frontier from the shared beam (identical
//                     result in every warp, so no barrier is needed for it);
//   warp 0         -- visited-table upkeep, neighbour list, filters;   B1
//   all W warps    -- the candidates' distances, 16-row (tile and shared-
//                     memory layouts) slices dealt round-robin;       B2
//   warp 0         -- keep / sort the candidates and merge the beam;  B3
// Every decision that steers the loop is read from shared memory after a
// barrier, so all warps take the same path and reach every barrier.  The
// traversal, the distances (same summation order) and the output are those
// of the warp-per-query kernel.
template <int MAXC>
__device__ __forceinline__ void cta_tile_rows(const WarpSmem& sm, const GraphView& g, const float* qs,
                                              int base, int m, int tile, int s, uint32_t dpad,
                                              int nchunks, uint32_t* seen, uint32_t& first) {
  constexpr int SL = JB_T4_SLOTS;
  const int nslot = min(SL, (m - base + 7) >> 3);
  uint4 u[SL][MAXC];
  uint32_t rid[SL];
#pragma unroll
  for (int i = 0; i < SL; i++) {
    const int j = base + tile + 8 * i;
    const bool act = i < nslot && j < m;
    rid[i] = act ? sm.cand_ids[j] : kInvalid;
    const uint4* row = reinterpret_cast<const uint4*>(
        g.vec + size_t(act ? rid[i] - g.global_offset : 0) * dpad);
#pragma unroll
    for (int k = 0; k < MAXC; k++) {
      const int c = s + 4 * k;
      u[i][k] = (act && c < nchunks) ? ldg16(row + c) : make_uint4(0, 0, 0, 0);
    }
  }
#pragma unroll
  for (int p = 0; p < SL / 2; p++) {
    if (2 * p >= nslot) break;
    const float2 v = tile4_pair_sum<MAXC>(tile4_pair_chain<MAXC>(qs, u[2 * p], u[2 * p + 1]));
    if (s == 0) {
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int i = 2 * p + h;
        const int j = base + tile + 8 * i;
        if (rid[i] != kInvalid) {
          sm.cand_keys[j] = make_key(h ? v.y : v.x, rid[i]);
          if (seen != nullptr) {
            const uint32_t l = rid[i] - g.global_offset;
            if (!(atomicOr(&seen[l >> 5], 1u << (l & 31)) & (1u << (l & 31)))) first++;
          }
        }
      }
    }
  }
}

template <int METRIC>
__device__ __forceinline__ void cta_smemq_rows(const WarpSmem& sm, const GraphView& g, int base,
                                               int m, int tile, int s, uint32_t dpad, int nchunks,
                                               uint32_t* seen, uint32_t& first) {
  const int i0 = base + tile, i1 = base + tile + 8;
  const bool a0 = i0 < m, a1 = i1 < m;
  const uint32_t id0 = a0 ? sm.cand_ids[i0] : g.global_offset;
  const uint32_t id1 = a1 ? sm.cand_ids[i1] : id0;
  const uint4* r0 = reinterpret_cast<const uint4*>(g.vec + size_t(id0 - g.global_offset) * dpad);
  const uint4* r1 = reinterpret_cast<const uint4*>(g.vec + size_t(id1 - g.global_offset) * dpad);
  const float2 dd = dist_smemq2<METRIC>(sm.query, r0, a0, r1, a1, nchunks, s);
  if (s == 0) {
    if (a0) sm.cand_keys[i0] = make_key(dd.x, id0);
    if (a1) sm.cand_keys[i1] = make_key(dd.y, id1);
    if (seen != nullptr) {
      const uint32_t l0 = id0 - g.global_offset, l1 = id1 - g.global_offset;
      if (a0 && !(atomicOr(&seen[l0 >> 5], 1u << (l0 & 31)) & (1u << (l0 & 31)))) first++;
      if (a1 && !(atomicOr(&seen[l1 >> 5], 1u << (l1 & 31)) & (1u << (l1 & 31)))) first++;
    }
  }
}

// MAXC: 1..4 = tile-of-4 layout (L2, dpad <= 128); 0 = shared-memory query
// (any dpad, L2 or inner product).
template <uint32_t BWCAP, uint32_t HBITS, int MAXC, int METRIC, int W>
__global__ void __launch_bounds__(32 * W, 16 / W) beam_search_cta_kernel(SearchArgs a) {
  constexpr bool kTile = MAXC > 0;
  extern __shared__ __align__(16) char smem_raw[];
  __shared__ uint32_t s_q, s_m, s_cnt, s_flip, s_first;
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const uint32_t dpad = a.g.dpad;
  const uint32_t rq_nw = a.rq_on ? (a.g.dim + 31) / 32 : 0;
  const size_t per_q = warp_smem_bytes(BWCAP, HBITS, dpad, MAXC, 4 * rq_nw);
  WarpSmem sm = carve(smem_raw, BWCAP, HBITS);
  uint32_t* rq_planes = reinterpret_cast<uint32_t*>(smem_raw + per_q - align16(size_t(4) * rq_nw * 4));
  const int tile = lane >> 2, s = lane & 3;
  const int nchunks = int(dpad / 8);
  const GraphView& g = a.g;
  const uint32_t hsize = 1u << HBITS;
  const uint32_t R = g.R;
  const uint32_t bw = a.bw;
  const float* qs = reinterpret_cast<const float*>(sm.qpairs) + s * (8 * MAXC + 4);

  for (;;) {
    if (threadIdx.x == 0) s_q = atomicAdd(a.work_counter, 1u);
    __syncthreads();
    const uint32_t q = s_q;
    if (q >= a.nq) break;
    uint32_t* seen = a.seen_bits != nullptr ? a.seen_bits + size_t(q) * ((g.n + 31) / 32) : nullptr;

    // ── prologue: query layout and RaBitQ terms (warp 0), table clear (all)
    float rq_vl = 0.0f, rq_delta = 0.0f, rq_gadd = 0.0f, rq_lq = 0.0f;
    int rq_S = 0;
    if (wid == 0) {
      const uint16_t* qrow = a.queries + size_t(q) * dpad;
      if (a.rot_pad != nullptr) {
        uint16_t* raw = reinterpret_cast<uint16_t*>(sm.hash);
        uint16_t* rot = kTile ? raw + dpad : sm.query;
        const uint4* src = reinterpret_cast<const uint4*>(qrow);
        for (int c = lane; c < nchunks; c += 32) reinterpret_cast<uint4*>(raw)[c] = ldg16(src + c);
        __syncwarp();
        rotate_query_warp(raw, rot, a.rot_pad, g.dim, dpad, lane);
        __syncwarp();
        qrow = rot;
      } else if (a.stage_query) {
        // Host-resident query (see the warp kernel)
        uint16_t* dst = kTile ? reinterpret_cast<uint16_t*>(sm.hash) : sm.query;
        stage_query_row(dst, qrow, nchunks, lane, 32);
        __syncwarp();
        qrow = dst;
      } else if constexpr (!kTile) {
        const uint4* src = reinterpret_cast<const uint4*>(qrow);
        for (int c = lane; c < nchunks; c += 32) reinterpret_cast<uint4*>(sm.query)[c] = ldg16(src + c);
        __syncwarp();
        qrow = sm.query;
      }
      if constexpr (kTile) build_qtile<(kTile ? MAXC : 1)>(reinterpret_cast<float*>(sm.qpairs), qrow, nchunks, lane);
      if (a.rq_on) {
        const __half* qv = reinterpret_cast<const __half*>(qrow);
        const uint32_t dim = g.dim;
        float vl = __int_as_float(0x7F800000), vr = -vl;
        for (uint32_t i = lane; i < dim; i += 32) {
          const float x = __half2float(qv[i]);
          vl = fminf(vl, x);
          vr = fmaxf(vr, x);
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
          vl = fminf(vl, __shfl_xor_sync(kFull, vl, d));
          vr = fmaxf(vr, __shfl_xor_sync(kFull, vr, d));
        }
        const float range = __fsub_rn(vr, vl);
        const float inv = range > 0.0f ? __fdiv_rn(15.0f, range) : 0.0f;
        int S = 0;
        for (uint32_t w = 0; w < rq_nw; w++) {
          const uint32_t i = 32 * w + lane;
          int qq = 0;
          if (i < dim) {
            qq = __float2int_rn(__fmul_rn(__fsub_rn(__half2float(qv[i]), vl), inv));
            qq = qq < 0 ? 0 : (qq > 15 ? 15 : qq);
          }
          S += qq;
#pragma unroll
          for (int p = 0; p < 4; p++) {
            const uint32_t bits = __ballot_sync(kFull, (qq >> p) & 1);
            if (lane == 0) rq_planes[p * rq_nw + w] = bits;
          }
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) S += __shfl_xor_sync(kFull, S, d);
        float acc_ip = 0.0f, acc_l2 = 0.0f;
        for (uint32_t i = lane; i < dim; i += 32) {
          const float x = __half2float(qv[i]);
          const float ci = __ldg(a.rq_centroid + i);
          acc_ip = __fmaf_rn(ci, x, acc_ip);
          const float dd = __fsub_rn(x, ci);
          acc_l2 = __fmaf_rn(dd, dd, acc_l2);
        }
        acc_ip = warp_sum_xor(acc_ip);
        acc_l2 = warp_sum_xor(acc_l2);
        rq_vl = vl;
        rq_delta = __fdiv_rn(range, 15.0f);
        rq_S = S;
        rq_gadd = METRIC == kIP ? -acc_ip : acc_l2;
        rq_lq = __fmul_rn(a.rq_margin, __fsqrt_rn(acc_l2));
      }
    }
    if (threadIdx.x == 0) s_first = 0;
    __syncthreads();  // every read of a query staged in the table's slots is done
    for (uint32_t i = threadIdx.x; i < hsize; i += 32 * W) sm.hash[i] = kHashEmpty;
    __syncthreads();

    // ── seed with the medoid (warp 0)
    uint64_t* cur = sm.beam0;
    uint64_t* nxt = sm.beam1;
    uint32_t first = 0, n_hash = 1, expansions = 0, deg_sum = 0, evals = 1, resets = 0;
    if (wid == 0) {
      if (lane == 0) {
        sm.cand_ids[0] = g.medoid;
        hash_insert(sm.hash, HBITS, g.medoid);
      }
      __syncwarp();
      if constexpr (kTile) cta_tile_rows<(kTile ? MAXC : 1)>(sm, g, qs, 0, 1, tile, s, dpad, nchunks, seen, first);
      else cta_smemq_rows<METRIC>(sm, g, 0, 1, tile, s, dpad, nchunks, seen, first);
      __syncwarp();
      if (lane == 0) cur[0] = sm.cand_keys[0];
    }
    uint32_t cnt = 1;
    __syncthreads();

    uint32_t loop_count = 0;
    while (loop_count <= a.limit) {
      loop_count++;
      int pos = -1;  // choose_new_frontier, identical in every warp
      for (uint32_t b0 = 0; b0 < cnt; b0 += 32) {
        const uint32_t i = b0 + lane;
        const bool unv = i < cnt && !key_visited(cur[i]);
        const uint32_t bal = __ballot_sync(kFull, unv);
        if (bal) { pos = int(b0) + __ffs(bal) - 1; break; }
      }
      if (pos < 0) break;
      const uint64_t fkey = cur[pos];
      expansions++;
      if (expansions == a.max_result_size) break;
      const uint32_t u = key_id(fkey);

      if (wid == 0) {
        if (n_hash + R > kHashFillNum * (hsize / kHashFillDen)) {
          for (uint32_t i = lane; i < hsize; i += 32) sm.hash[i] = kHashEmpty;
          __syncwarp();
          for (uint32_t i = lane; i < cnt; i += 32) hash_insert(sm.hash, HBITS, key_id(cur[i]));
          n_hash = cnt;
          resets++;
          __syncwarp();
        }
        const uint32_t lu = u - g.global_offset;
        const uint32_t ne = g.counts[lu];
        const uint32_t* el = g.edges + size_t(lu) * R;
        const uint32_t nb0 = lane < R ? __ldg(el + lane) : kInvalid;
        const uint32_t nb1 = lane + 32 < R ? __ldg(el + lane + 32) : kInvalid;
        deg_sum += ne;
        const bool f0 = (lane < ne) && (nb0 - g.global_offset < g.n) && hash_insert(sm.hash, HBITS, nb0);
        const uint32_t b0 = __ballot_sync(kFull, f0);
        const bool f1 = (lane + 32 < ne) && (nb1 - g.global_offset < g.n) && hash_insert(sm.hash, HBITS, nb1);
        const uint32_t b1 = __ballot_sync(kFull, f1);
        const uint32_t lt = (1u << lane) - 1u;
        if (f0) sm.cand_ids[__popc(b0 & lt)] = nb0;
        if (f1) sm.cand_ids[__popc(b0) + __popc(b1 & lt)] = nb1;
        int m = __popc(b0) + __popc(b1);
        n_hash += m;
        __syncwarp();
        if (a.rq_on && cnt == bw && m > 0) {
          const float tau = key_dist(cur[bw - 1]);
          bool k0 = false, k1 = false;
          uint32_t c0 = 0, c1 = 0;
          if (lane < m) {
            c0 = sm.cand_ids[lane];
            const uint32_t l = c0 - g.global_offset;
            const float est = rabitq_est(a, l, rq_planes, rq_nw, g.dim, rq_vl, rq_delta, rq_S,
                                         rq_gadd, METRIC == kIP);
            k0 = !(__fsub_rn(est, __fmul_rn(rq_lq, __ldg(a.rq_err + l))) > tau);
          }
          if (lane + 32 < m) {
            c1 = sm.cand_ids[lane + 32];
            const uint32_t l = c1 - g.global_offset;
            const float est = rabitq_est(a, l, rq_planes, rq_nw, g.dim, rq_vl, rq_delta, rq_S,
                                         rq_gadd, METRIC == kIP);
            k1 = !(__fsub_rn(est, __fmul_rn(rq_lq, __ldg(a.rq_err + l))) > tau);
          }
          const uint32_t kb0 = __ballot_sync(kFull, k0), kb1 = __ballot_sync(kFull, k1);
          __syncwarp();
          if (k0) sm.cand_ids[__popc(kb0 & lt)] = c0;
          if (k1) sm.cand_ids[__popc(kb0) + __popc(kb1 & lt)] = c1;
          m = __popc(kb0) + __popc(kb1);
        }
        evals += m;
        if (lane == 0) s_m = uint32_t(m);
      }
      __syncthreads();  // B1: candidates listed
      const int m = int(s_m);
      if (threadIdx.x == 0) cur[pos] = fkey | 1ull;
      // distances: 16-row slices dealt round-robin over the warps
      for (int base = 16 * wid; base < m; base += 16 * W) {
        if constexpr (kTile) cta_tile_rows<(kTile ? MAXC : 1)>(sm, g, qs, base, m, tile, s, dpad, nchunks, seen, first);
        else cta_smemq_rows<METRIC>(sm, g, base, m, tile, s, dpad, nchunks, seen, first);
      }
      __syncthreads();  // B2: candidate keys written

      if (wid == 0) {
        uint64_t v0 = lane < m ? sm.cand_keys[lane] : kKeyMax;
        uint64_t v1 = lane + 32 < m ? sm.cand_keys[lane + 32] : kKeyMax;
        if (cnt == bw) {
          const uint64_t worst = cur[bw - 1] | 1ull;
          if (v0 > worst) v0 = kKeyMax;
          if (v1 > worst) v1 = kKeyMax;
        }
        const uint32_t k0 = __ballot_sync(kFull, v0 != kKeyMax);
        const uint32_t k1 = __ballot_sync(kFull, v1 != kKeyMax);
        const int kept = __popc(k0) + __popc(k1);
        __syncwarp();
        bool sorted = true;
        if (kept > 0 && kept <= 32) {
          const uint32_t lt = (1u << lane) - 1u;
          if (v0 != kKeyMax) sm.cand_keys[__popc(k0 & lt)] = v0;
          if (v1 != kKeyMax) sm.cand_keys[__popc(k0) + __popc(k1 & lt)] = v1;
          __syncwarp();
          if (kept <= kCountMerge) {
            sorted = false;
          } else {
            uint64_t v = lane < kept ? sm.cand_keys[lane] : kKeyMax;
            v = warp_sort32(v, lane);
            sm.cand_keys[lane] = v;
          }
        } else if (kept > 32) {
          warp_sort64(v0, v1, lane);
          sm.cand_keys[lane] = v0;
          sm.cand_keys[lane + 32] = v1;
        }
        __syncwarp();
        if (kept > 0) {
          if (!sorted) {
            for (uint32_t i = lane; i < cnt; i += 32) {
              const uint64_t b = cur[i];
              uint32_t r = 0;
              for (int j = 0; j < kept; j++) r += sm.cand_keys[j] < b;
              if (i + r < bw) nxt[i + r] = b;
            }
            if (lane < kept) {
              const uint64_t c = sm.cand_keys[lane];
              uint32_t r = 0;
              for (int j = 0; j < kept; j++) r += sm.cand_keys[j] < c;
              const uint32_t p = r + lower_rank(cur, int(cnt), c);
              if (p < bw) nxt[p] = c;
            }
          } else {
            for (uint32_t i = lane; i < cnt; i += 32) {
              const uint64_t b = cur[i];
              const uint32_t p = i + lower_rank(sm.cand_keys, kept, b);
              if (p < bw) nxt[p] = b;
            }
            for (int j = lane; j < kept; j += 32) {
              const uint64_t c = sm.cand_keys[j];
              const uint32_t p = j + lower_rank(cur, int(cnt), c);
              if (p < bw) nxt[p] = c;
            }
          }
        }
        if (lane == 0) {
          s_flip = kept > 0 ? 1u : 0u;
          s_cnt = kept > 0 ? min(bw, cnt + uint32_t(kept)) : cnt;
        }
      }
      __syncthreads();  // B3: beam merged
      cnt = s_cnt;
      if (s_flip) { uint64_t* t = cur; cur = nxt; nxt = t; }
    }

    if (a.stats != nullptr && s == 0) atomicAdd(&s_first, first);
    __syncthreads();
    // output: the first k non-deleted entries (beam_search.cuh:205-222)
    if (wid == 0) {
      uint32_t out = 0;
      for (uint32_t b0 = 0; b0 < cnt && out < a.k; b0 += 32) {
        const uint32_t i = b0 + lane;
        uint32_t id = 0;
        bool ok = false;
        if (i < cnt) {
          id = key_id(cur[i]);
          const uint32_t l = id - g.global_offset;
          ok = !(g.deleted != nullptr && ((g.deleted[l >> 5] >> (l & 31)) & 1u));
        }
        const uint32_t bal = __ballot_sync(kFull, ok);
        const uint32_t p = out + __popc(bal & ((1u << lane) - 1u));
        if (ok && p < a.k) {
          const uint32_t sid = g.ids_identity ? id : g.slot_to_id[id - g.global_offset];
          a.out_idx[size_t(q) * a.k + p] = int32_t(sid);
          a.out_dist[size_t(q) * a.k + p] = key_dist(cur[i]);
        }
        out += __popc(bal);
      }
      for (uint32_t p = out + lane; p < a.k; p += 32) {
        a.out_idx[size_t(q) * a.k + p] = -1;
        a.out_dist[size_t(q) * a.k + p] = 1e30f;
      }
      if (lane == 0 && a.stats != nullptr) {
        a.stats[size_t(q) * 5 + 0] = expansions;
        a.stats[size_t(q) * 5 + 1] = deg_sum;
        a.stats[size_t(q) * 5 + 2] = evals;
        a.stats[size_t(q) * 5 + 3] = resets;
        a.stats[size_t(q) * 5 + 4] = seen != nullptr ? s_first : evals;
      }
    }
    __syncthreads();  // shared state is reused by the next query
  }
}

// The shared-memory opt-in and the occupancy query cost a few microseconds
// each, so they are cached per (kernel, device, shared memory).  The opt-in
// is a maximum: it is only ever raised, never lowered by a smaller launch, so
// a cached larger launch stays valid.
struct LaunchShape { int sms, per_sm; };
using SearchKernel = void (*)(SearchArgs);

LaunchShape launch_shape(SearchKernel kern, int threads, size_t smem) {
  static std::mutex m;
  static std::map<std::tuple<const void*, int, size_t>, LaunchShape> cache;
  static std::map<std::pair<const void*, int>, size_t> opted;
  int dev = 0;
  cudaGetDevice(&dev);
  const void* key = reinterpret_cast<const void*>(kern);
  std::lock_guard<std::mutex> lock(m);
  size_t& cur = opted[{key, dev}];
  if (smem > cur) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    cur = smem;
  }
  auto it = cache.find({key, dev, smem});
  if (it != cache.end()) return it->second;
  LaunchShape L{};
  cudaDeviceGetAttribute(&L.sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&L.per_sm, kern, threads, smem);
  if (L.per_sm < 1) L.per_sm = 1;
  cache[{key, dev, smem}] = L;
  return L;
}

void check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("search launch: ") + cudaGetErrorString(e));
}

template <uint32_t BWCAP, uint32_t HBITS, int MAXC, int METRIC>
void launch_t(const SearchArgs& a, cudaStream_t stream) {
  auto kern = beam_search_warp_kernel<BWCAP, HBITS, MAXC, METRIC>;
  const size_t per_warp =
      warp_smem_bytes(BWCAP, HBITS, a.g.dpad, MAXC, a.rq_on ? 4 * ((a.g.dim + 31) / 32) : 0);
  int wpb = 4;
  while (wpb > 1 && per_warp * wpb > 200 * 1024) wpb--;
  if (per_warp * wpb > 220 * 1024) throw std::runtime_error("search: shared memory per query too large");
  const size_t smem = per_warp * wpb;
  const LaunchShape L = launch_shape(kern, 32 * wpb, smem);
  const uint32_t need = (a.nq + wpb - 1) / wpb;
  uint32_t grid = uint32_t(L.sms) * uint32_t(L.per_sm);
  if (grid > need) grid = need;
  if (grid == 0) return;
  kern<<<grid, 32 * wpb, smem, stream>>>(a);
  check_launch();
}

#ifndef JB_CTA_WARPS
#define JB_CTA_WARPS 2
#endif
constexpr int kCtaWarps = JB_CTA_WARPS;

template <uint32_t BWCAP, uint32_t HBITS, int MAXC, int METRIC>
void launch_cta(const SearchArgs& a, cudaStream_t stream) {
  auto kern = beam_search_cta_kernel<BWCAP, HBITS, MAXC, METRIC, kCtaWarps>;
  const size_t smem =
      warp_smem_bytes(BWCAP, HBITS, a.g.dpad, MAXC, a.rq_on ? 4 * ((a.g.dim + 31) / 32) : 0);
  if (smem > 220 * 1024) throw std::runtime_error("search: shared memory per query too large");
  const LaunchShape L = launch_shape(kern, 32 * kCtaWarps, smem);
  uint32_t grid = uint32_t(L.sms) * uint32_t(L.per_sm);
  if (grid > a.nq) grid = a.nq;
  if (grid == 0) return;
  kern<<<grid, 32 * kCtaWarps, smem, stream>>>(a);
  check_launch();
}

// 0: choose per launch; 1: always a warp per query; 2 or more: always a CTA
// (of kCtaWarps warps) per query.
std::atomic<int> g_search_mode{0};

#ifndef JB_CTA_QUERIES_PER_SM
#define JB_CTA_QUERIES_PER_SM 8
#endif
// A CTA per query when the launch has fewer than this many queries per SM
// (the warp-per-query kernel would leave most warp slots idle) and is a
// query search (not the build's range search, which records expansions).
bool use_cta(const SearchArgs& a) {
  if (a.use_range || a.vis_idx != nullptr) return false;
  const int mode = g_search_mode.load(std::memory_order_relaxed);
  if (mode == 1) return false;
  if (mode >= 2) return true;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return a.nq < uint32_t(JB_CTA_QUERIES_PER_SM) * uint32_t(sms > 0 ? sms : 1);
}

template <uint32_t BWCAP, uint32_t HBITS>
void dispatch_dim(const SearchArgs& a, cudaStream_t stream) {
  const uint32_t nchunks = a.g.dpad / 8;
  if (use_cta(a)) {
    // tile-of-4 layout for L2 rows up to 128 dims, the shared-memory query
    // layout for everything else (same summation orders as the warp kernel)
    if (a.g.metric == kIP) return launch_cta<BWCAP, HBITS, 0, kIP>(a, stream);
    if (nchunks <= 4) return launch_cta<BWCAP, HBITS, 1, kL2>(a, stream);
    if (nchunks <= 8) return launch_cta<BWCAP, HBITS, 2, kL2>(a, stream);
    if (nchunks <= 12) return launch_cta<BWCAP, HBITS, 3, kL2>(a, stream);
    if (nchunks <= 16) return launch_cta<BWCAP, HBITS, 4, kL2>(a, stream);
    return launch_cta<BWCAP, HBITS, 0, kL2>(a, stream);
  }
  if (a.g.metric == kIP) {
    if (nchunks <= 4) return launch_t<BWCAP, HBITS, 1, kIP>(a, stream);
    if (nchunks <= 8) return launch_t<BWCAP, HBITS, 2, kIP>(a, stream);
    if (nchunks <= 12) return launch_t<BWCAP, HBITS, 3, kIP>(a, stream);
    if (nchunks <= 16) return launch_t<BWCAP, HBITS, 4, kIP>(a, stream);
    if (nchunks <= 32) return launch_t<BWCAP, HBITS, 8, kIP>(a, stream);
    return launch_t<BWCAP, HBITS, 0, kIP>(a, stream);
  }
  if (nchunks <= 4) return launch_t<BWCAP, HBITS, 1, kL2>(a, stream);
  if (nchunks <= 8) return launch_t<BWCAP, HBITS, 2, kL2>(a, stream);
  if (nchunks <= 12) return launch_t<BWCAP, HBITS, 3, kL2>(a, stream);
  if (nchunks <= 16) return launch_t<BWCAP, HBITS, 4, kL2>(a, stream);
  if (nchunks <= 32) return launch_t<BWCAP, HBITS, 8, kL2>(a, stream);
  return launch_t<BWCAP, HBITS, 0, kL2>(a, stream);
}

}  // namespace

#ifdef JB_PHASE_CLOCKS
extern "C" int jb_debug_phase_clocks(unsigned long long* out, int reset) {
  if (cudaMemcpyFromSymbol(out, g_phase_clocks, sizeof(unsigned long long) * 8) != cudaSuccess) return 1;
  if (reset) {
    unsigned long long z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    cudaMemcpyToSymbol(g_phase_clocks, z, sizeof(z));
  }
  return 0;
}
#endif

void set_search_mode(int warps_per_query) {
  if (warps_per_query < 0) throw std::invalid_argument("warps per query must be >= 0");
  g_search_mode.store(warps_per_query >= 2 ? kCtaWarps : warps_per_query, std::memory_order_relaxed);
}

void launch_search(const SearchArgs& a, cudaStream_t stream) {
  if (a.nq == 0) return;
  if (a.g.R > 64) throw std::runtime_error("search: R > 64 is not supported");
  if (a.bw == 0) throw std::runtime_error("search: beam_width must be > 0");
  // Same bound as the reference's width dispatch (beam_search/api.cuh:64-72).
  if (a.bw + 64 >= 2048)
    throw std::invalid_argument("beam_width " + std::to_string(a.bw) +
                                " is too large (beam_width + 64 must be < 2048)");
#ifndef JB_HBITS64
#define JB_HBITS64 11
#endif
#ifndef JB_HBITS32
#define JB_HBITS32 10
#endif
  if (a.bw <= 32) return dispatch_dim<32, JB_HBITS32>(a, stream);
  if (a.bw <= 64) return dispatch_dim<64, JB_HBITS64>(a, stream);
  if (a.bw <= 128) return dispatch_dim<128, 11>(a, stream);
  if (a.bw <= 256) return dispatch_dim<256, 11>(a, stream);
  if (a.bw <= 512) return dispatch_dim<512, 12>(a, stream);
  return dispatch_dim<2048, 14>(a, stream);
}

}  // namespace jb
