// construct.cu -- batched Vamana construction (greedy search + RobustPrune).
//
// Follows construct_graph / construction_round / process_batch of the
// reference (include/jasper/index/construct.cuh:743-1160): rows are inserted
// in id order in batches of 1, 2, 4, ... up to max_batch_size; for each batch
//   (a) beam search from the medoid for every batch row (L = beam = 64,
//       limit 256, expansion list capped at 256), recording the expansion
//       order with exact distances -- the same warp-per-query kernel as the
//       query search (search.cu) in range mode;
//   (b) candidates = the row's existing edges (stored bf16 distances) plus the
//       expansion list minus the row itself, sorted by (distance, id)
//       (merge_candidates_kernel, construct.cuh:280-377);
//   (c) RobustPrune(alpha): walk the sorted candidates, keep c unless a kept
//       s has d(c, s) * alpha < d(row, c), stop at R (construct.cuh:379-473);
//   (d) reverse edges (target = new neighbour, sink = batch row) are sorted
//       by (target, sink) and split into one group per target
//       (fill_reverse_edges + thrust semisort, construct.cuh:475-558; here a
//       stable radix sort of our own on the target id);
//   (e) for every target: existing edges plus the sinks with fresh distances,
//       sorted, pruned again and written back (construct.cuh:560-741).
//
// Device design: one warp per batch row / per target, candidates sorted by a
// bitonic network in shared memory, the pruned candidate's row held in
// registers in the 4-lane distance layout while each 4-lane tile tests it
// against two kept rows at a time; the scan over kept rows stops at the first
// pass that prunes (the reference evaluates all of them; the OR is the same).
// Every phase is stream-ordered with no host round trip, so a whole build is
// a sequence of asynchronous launches.
//
// Candidate cap in (e): at most 256 + R candidates per target
// (construct.cuh:574).  When a target has more, the reference keeps whichever
// ones its shared-memory atomics place first -- in practice the existing edges
// (one cheap pass) and then the sinks in group order.  This code keeps exactly
// that, deterministically: existing edges, then sinks in (target, sink) order
// until the cap; the sinks past the cap are never evaluated.
#include <algorithm>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include "construct.cuh"
#include "jb_common.cuh"
#include "search.cuh"

namespace jb {
namespace {

constexpr uint32_t kMaxCandSort = 512;  // sort capacity per warp

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
  }
}

// Candidate-row distances for the prune: the candidate row is the tile's
// "query".  nchunks is dim / 8 (the reference passes the unpadded dim to
// compute_distance in the prune kernels, construct.cuh:437-439).
template <int MAXC, int METRIC>
struct RowReg {
  uint4 q[MAXC > 0 ? MAXC : 1];
  const uint16_t* qs;  // shared-memory copy when MAXC == 0
  __device__ __forceinline__ void load(const GraphView& g, uint32_t id, int nchunks, int lane,
                                       uint16_t* smem_row) {
    const uint4* row = reinterpret_cast<const uint4*>(g.vec + size_t(id - g.global_offset) * g.dpad);
    const int s = lane & 3;
    if constexpr (MAXC > 0) {
#pragma unroll
      for (int i = 0; i < MAXC; i++) {
        int c = s + 4 * i;
        q[i] = c < nchunks ? ldg16(row + c) : make_uint4(0, 0, 0, 0);
      }
    } else {
      __syncwarp();
      uint4* dst = reinterpret_cast<uint4*>(smem_row);
      for (int c = lane; c < int(g.dpad / 8); c += 32) dst[c] = ldg16(row + c);
      __syncwarp();
      qs = smem_row;
    }
  }
  // Kept-row cache (L2, register path): kept row j lives at sel + j * stride
  // (stride = dpad / 8 chunks); with swz its chunk c sits at c ^ 4 on odd
  // rows, so tiles 2p and 2p+1 (rows j, j+1) read disjoint bank groups.
  __device__ __forceinline__ static int sel_slot(int j, int c, int stride, bool swz) {
    return j * stride + (swz ? (c ^ ((j & 1) << 2)) : c);
  }
  __device__ __forceinline__ void store_sel(uint4* sel, int j, int nchunks, int stride, bool swz,
                                            int s) const {
    if constexpr (MAXC > 0) {
#pragma unroll
      for (int i = 0; i < MAXC; i++) {
        const int c = s + 4 * i;
        if (c < nchunks) sel[sel_slot(j, c, stride, swz)] = q[i];
      }
    }
  }
  __device__ __forceinline__ float dist_sel(const uint4* sel, int j, bool active, int nchunks,
                                            int stride, bool swz, int s) const {
    float acc = 0.f;
    if constexpr (MAXC > 0) {
#pragma unroll
      for (int i = 0; i < MAXC; i++) {
        const int c = s + 4 * i;
        if (c < nchunks) {
          const uint4 x = active ? sel[sel_slot(j, c, stride, swz)] : make_uint4(0, 0, 0, 0);
          acc = l2_chunk(q[i], x, acc);
        }
      }
    }
    return tile4_sum(acc);
  }
  // dist() from global memory for one tile on its own path.
  __device__ __forceinline__ float dist_local(const GraphView& g, uint32_t id, int nchunks,
                                              int lane) const {
    const uint4* row = reinterpret_cast<const uint4*>(g.vec + size_t(id - g.global_offset) * g.dpad);
    const int s = lane & 3;
    float acc = 0.f;
    if constexpr (MAXC > 0) {
      uint4 x[MAXC];
#pragma unroll
      for (int i = 0; i < MAXC; i++) {
        const int c = s + 4 * i;
        x[i] = c < nchunks ? ldg16(row + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < MAXC; i++)
        if (s + 4 * i < nchunks) acc = l2_chunk(q[i], x[i], acc);
    }
    return tile4_sum_local(acc, lane);
  }
  // dist_sel for one tile on its own path (tile-local reduction).
  __device__ __forceinline__ float dist_sel_local(const uint4* sel, int j, int nchunks,
                                                  int stride, bool swz, int lane) const {
    float acc = 0.f;
    const int s = lane & 3;
    if constexpr (MAXC > 0) {
#pragma unroll
      for (int i = 0; i < MAXC; i++) {
        const int c = s + 4 * i;
        if (c < nchunks) acc = l2_chunk(q[i], sel[sel_slot(j, c, stride, swz)], acc);
      }
    }
    return tile4_sum_local(acc, lane);
  }
  __device__ __forceinline__ float dist(const GraphView& g, uint32_t id, bool active,
                                        int nchunks, int s) const {
    const uint4* row = reinterpret_cast<const uint4*>(g.vec + size_t(id - g.global_offset) * g.dpad);
    float acc = 0.f;
    if constexpr (MAXC > 0 && METRIC == kL2) {
      uint4 x[MAXC];
#pragma unroll
      for (int i = 0; i < MAXC; i++) {
        int c = s + 4 * i;
        x[i] = (active && c < nchunks) ? ldg16(row + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < MAXC; i++)
        if (s + 4 * i < nchunks) acc = l2_chunk(q[i], x[i], acc);
      return tile4_sum(acc);
    } else if constexpr (METRIC == kL2) {
      const uint4* q4 = reinterpret_cast<const uint4*>(qs);
      for (int c = s; c < nchunks; c += 4) {
        uint4 r = active ? ldg16(row + c) : make_uint4(0, 0, 0, 0);
        acc = l2_chunk(q4[c], r, acc);
      }
      return tile4_sum(acc);
    } else {
      const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qs);
      const uint32_t* r32 = reinterpret_cast<const uint32_t*>(row);
      const int w = s >> 1;
      const int nck = int(g.dpad / 8);
      for (int c = 0; c < nck; c++) {
        uint32_t rlo = active ? __ldg(r32 + 4 * c + w) : 0u;
        uint32_t rhi = active ? __ldg(r32 + 4 * c + 2 + w) : 0u;
        acc = ip_pair(q32[4 * c + w], q32[4 * c + 2 + w], rlo, rhi, s, acc);
      }
      return -tile4_sum(acc);
    }
  }
};

struct PruneSmem {
  uint64_t* cand;   // [kMaxCandSort]
  uint32_t* sel;    // [64]
  float* sel_d;     // [64]
  uint16_t* row;    // [dpad] (shared-memory row path)
  uint4* selrows;   // [64][dpad / 8] kept rows (L2 register path only)
};
constexpr int kPruneGroup = 8;

// RobustPrune strategy: 0 one candidate at a time, kept rows re-read from
// global memory; 1 groups of 8 candidates, kept rows from global memory;
// 2 groups of 8, kept rows cached in shared memory.
#ifndef JB_PRUNE_MODE
#define JB_PRUNE_MODE 1
#endif

#ifdef JB_BUILD_CLOCKS
__device__ unsigned long long g_build_clk[8];
#endif  // candidates tested at once, one per 4-lane tile

// The kept-row cache is used where the candidate row sits in registers (L2,
// dpad <= 256): every prune test then reads the kept row from shared memory.
template <int MAXC, int METRIC>
struct SelCache {
  static constexpr bool on = JB_PRUNE_MODE == 2 && MAXC > 0 && METRIC == kL2;
  static constexpr bool batch = JB_PRUNE_MODE >= 1 && MAXC > 0 && METRIC == kL2;
};

__host__ __device__ inline size_t prune_warp_bytes(uint32_t dpad, bool sel_cache) {
  size_t b = kMaxCandSort * 8 + 64 * 4 + 64 * 4 + ((size_t(dpad) * 2 + 15) & ~size_t(15));
  if (sel_cache) b += size_t(64) * dpad * 2;
  return b;
}

__device__ __forceinline__ PruneSmem prune_carve(char* base, uint32_t dpad) {
  PruneSmem p;
  p.cand = reinterpret_cast<uint64_t*>(base);
  p.sel = reinterpret_cast<uint32_t*>(p.cand + kMaxCandSort);
  p.sel_d = reinterpret_cast<float*>(p.sel + 64);
  p.row = reinterpret_cast<uint16_t*>(p.sel_d + 64);
  p.selrows = reinterpret_cast<uint4*>(reinterpret_cast<char*>(p.row) +
                                       ((size_t(dpad) * 2 + 15) & ~size_t(15)));
  return p;
}

// Write the kept list sm.sel / sm.sel_d (ns entries) as the row of `self`:
// ids, bf16 distances, count and, when the build keeps them, the prune flags
// (bit i: the distance kept slot i was tested with is exactly its stored
// bf16 value).
__device__ __forceinline__ void write_pruned_row(const GraphView& g, uint32_t self,
                                                 const PruneSmem& sm, uint32_t ns, int lane) {
  const uint32_t l = self - g.global_offset;
  const uint32_t R = g.R;
  uint64_t mask = 0;
  for (uint32_t i0 = 0; i0 < ns; i0 += 32) {
    const uint32_t i = i0 + lane;
    bool exact = false;
    if (i < ns) {
      const float d = sm.sel_d[i];
      const uint16_t b = float_to_bf16_bits(d);
      g.edges[size_t(l) * R + i] = sm.sel[i];
      g.edist[size_t(l) * R + i] = b;
      exact = bf16_bits_to_float(b) == d;
    }
    mask |= uint64_t(__ballot_sync(kFull, exact)) << i0;
  }
  if (lane == 0) {
    g.counts[l] = uint8_t(ns);
    if (g.eflag != nullptr) g.eflag[l] = mask;
  }
  __syncwarp();
}

// Sort cand[0, nc) ascending (pads the power-of-two tail with the max key).
__device__ __forceinline__ void sort_cands(uint64_t* cand, int nc, int lane) {
  int n = 32;
  while (n < nc) n <<= 1;
  for (int i = nc + lane; i < n; i += 32) cand[i] = kKeyMax;
  __syncwarp();
  warp_sort_smem(cand, n, lane);
}

// Sort cand[0, nc) where cand[0, na) are a target's existing edges and
// cand[na, nc) its new sinks.  The existing edges were written in candidate
// order with bf16-rounded distances, so they are usually sorted already
// (rounding is monotone; only ids inside a bf16 tie can be out of order).
// When they are and the sinks fit in one warp, the sinks are ranked in
// registers and both lists are merged in place by rank; otherwise the full
// bitonic sort runs.  Equal keys are identical values, so both give the same
// array.
__device__ __forceinline__ void sort_cands_merge(uint64_t* cand, int na, int nc, int lane) {
  const int nb = nc - na;
  bool fast = na <= 64 && nb <= 32;
  if (fast) {
    bool bad = false;
    for (int i = lane; i + 1 < na; i += 32) bad |= cand[i] > cand[i + 1];
    fast = !__any_sync(kFull, bad);
  }
  if (!fast) {
    sort_cands(cand, nc, lane);
    return;
  }
  const uint64_t b = lane < nb ? cand[na + lane] : kKeyMax;
  const uint64_t a0 = lane < na ? cand[lane] : kKeyMax;
  const uint64_t a1 = lane + 32 < na ? cand[lane + 32] : kKeyMax;
  int rb = 0, c0 = 0, c1 = 0;
  for (int t = 0; t < nb; t++) {
    const uint64_t o = __shfl_sync(kFull, b, t);
    rb += (o < b || (o == b && t < lane)) ? 1 : 0;
    c0 += o < a0 ? 1 : 0;
    c1 += o < a1 ? 1 : 0;
  }
  int ca = 0;  // existing edges <= b
  if (lane < nb) {
    int lo = 0, hi = na;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (cand[mid] <= b) lo = mid + 1; else hi = mid;
    }
    ca = lo;
  }
  __syncwarp();
  if (lane < na) cand[lane + c0] = a0;
  if (lane + 32 < na) cand[lane + 32 + c1] = a1;
  if (lane < nb) cand[rb + ca] = b;
  __syncwarp();
}

// RobustPrune over sorted candidate pair keys; writes the row of `self`.
template <int MAXC, int METRIC>
__device__ void prune_and_write(const GraphView& gv, uint32_t self, PruneSmem& sm, int nc,
                                float alpha, int lane) {
  const GraphView& g = gv;
  const int tile = lane >> 2, s = lane & 3;
  const int nchunks = int(g.dim / 8);
  const uint32_t R = g.R;
  uint32_t ns = 0;
  RowReg<MAXC, METRIC> cr;
  constexpr bool kSel = SelCache<MAXC, METRIC>::on;
  constexpr bool kBatch = SelCache<MAXC, METRIC>::batch;
  const int stride = int(g.dpad / 8);
  const bool swz = (stride & 7) == 0;
  if constexpr (kBatch) {
    // Groups of up to 8 candidates in list order, one per 4-lane tile.
    // Phase 1: each tile tests its candidate against the kept set as it was
    // when the group started (its own early exit).  Phase 2, in list order:
    // a survivor is accepted unless a row accepted earlier in this group
    // prunes it.  Pruning only grows with the kept set, so this accepts
    // exactly what the one-at-a-time loop accepts.
    const int tile = lane >> 2;
    int i = 0;
    while (i < nc && ns < R) {
      const int w = i + lane;
      const uint64_t wk = w < nc ? sm.cand[w] : kKeyMax;
      const bool valid = w < nc && pair_id(wk) != self && pair_id(wk) != kInvalid;
      const uint32_t bal = __ballot_sync(kFull, valid);
      const int nvalid = __popc(bal);
      if (nvalid == 0) { i += 32; continue; }
      const int gsz = nvalid < kPruneGroup ? nvalid : kPruneGroup;
      // position of the tile-th valid candidate in the window
      uint32_t rem = bal;
      for (int t = 0; t < tile && rem; t++) rem &= rem - 1;
      const bool mine = tile < gsz;
      const int pos = mine ? i + __ffs(rem) - 1 : i;
      int last = i;  // window position of the g-th valid candidate
      {
        uint32_t r2 = bal;
        for (int t = 0; t < gsz - 1; t++) r2 &= r2 - 1;
        last = i + __ffs(r2) - 1;
      }
      const uint64_t key = sm.cand[pos];
      const uint32_t cid = pair_id(key);
      const float cd = key_dist(key);
      if (mine) cr.load(gv, cid, nchunks, lane, sm.row);
      bool pruned = !mine;
      if (mine) {
        for (uint32_t j = 0; j < ns; j++) {
          const float d = kSel ? cr.dist_sel_local(sm.selrows, int(j), nchunks, stride, swz, lane)
                               : cr.dist_local(g, sm.sel[j], nchunks, lane);
          if (d * alpha < cd) { pruned = true; break; }
        }
      }
      __syncwarp();
      for (int t = 0; t < gsz; t++) {
        if (ns >= R) break;
        const bool tp = __shfl_sync(kFull, pruned ? 1 : 0, t * 4) != 0;
        if (tp) continue;
        const float tcd = __shfl_sync(kFull, cd, t * 4);
        const uint32_t tid = __shfl_sync(kFull, cid, t * 4);
        if (lane == 0) { sm.sel[ns] = tid; sm.sel_d[ns] = tcd; }
        if (kSel && tile == t) cr.store_sel(sm.selrows, int(ns), nchunks, stride, swz, lane & 3);
        __syncwarp();
        // later survivors of the group against the row just accepted
        const bool act = tile > t && !pruned;
        const float d = kSel ? cr.dist_sel(sm.selrows, int(ns), act, nchunks, stride, swz, lane & 3)
                             : cr.dist(g, act ? tid : cid, act, nchunks, lane & 3);
        if (tile > t && !pruned && d * alpha < cd) pruned = true;
        ns++;
        __syncwarp();
      }
      i = last + 1;
    }
  } else
  for (int i = 0; i < nc; i++) {
    if (ns >= R) break;
    const uint64_t key = sm.cand[i];
    const uint32_t cid = pair_id(key);
    if (cid == self || cid == kInvalid) continue;
    const float cd = key_dist(key);
    cr.load(g, cid, nchunks, lane, sm.row);
    bool pruned = false;
    for (uint32_t base = 0; base < ns; base += 16) {
      const uint32_t j0 = base + tile, j1 = base + tile + 8;
      const bool a0 = j0 < ns, a1 = j1 < ns;
      float d0, d1;
      if constexpr (kSel) {
        d0 = cr.dist_sel(sm.selrows, int(j0), a0, nchunks, stride, swz, s);
        d1 = cr.dist_sel(sm.selrows, int(j1), a1, nchunks, stride, swz, s);
      } else {
        d0 = cr.dist(g, a0 ? sm.sel[j0] : cid, a0, nchunks, s);
        d1 = cr.dist(g, a1 ? sm.sel[j1] : cid, a1, nchunks, s);
      }
      const bool p = (a0 && d0 * alpha < cd) || (a1 && d1 * alpha < cd);
      if (__any_sync(kFull, p)) { pruned = true; break; }
    }
    if (!pruned) {
      if (lane == 0) { sm.sel[ns] = cid; sm.sel_d[ns] = cd; }
      if constexpr (kSel) {
        if (lane < 4) cr.store_sel(sm.selrows, int(ns), nchunks, stride, swz, s);
      }
      ns++;
      __syncwarp();
    }
  }
  __syncwarp();
  write_pruned_row(g, self, sm, ns, lane);
}

// ---------------------------------------------------------------------------
// Incremental RobustPrune for one reverse-edge target.
//
// A kept edge is "trusted" (GraphView::eflag) when the prune that kept it
// tested it with exactly the distance now stored for it (the bf16 value):
// every existing edge a re-prune kept, and every new candidate whose fp32
// distance is exact in bf16.  For two trusted edges a before b nothing about
// their test has changed since b was kept: same keys, so the same relative
// order; same distances; and b passed against every kept row before it,
// a among them.  So in a re-prune a trusted b can only be pruned by an
// untrusted kept candidate before it (a new sink, or an edge whose test used
// its unrounded distance), and untrusted candidates need the full test.
// This path computes only the distances between the untrusted candidates and
// all others (the pair distance is symmetric bit for bit: (x - y)^2 and
// x * y are), then walks the sorted list exactly like prune_and_write, so
// the kept list is the one the full walk keeps.
// Used when at most kIncrMaxNew candidates are untrusted and nc <= 96; the
// distances live in the unused tail of sm.cand ([kIncrMaxNew][96] floats).
// ---------------------------------------------------------------------------
#ifndef JB_INCR_MAX_NEW
#define JB_INCR_MAX_NEW 8
#endif
constexpr int kIncrMaxNew = JB_INCR_MAX_NEW;
constexpr int kIncrMaxCand = 96;

// Scratch (inside the Gram scratch of the warp): the existing edges' keys
// before the sort, the untrusted candidates' rows, their distances.
struct IncrScratch {
  uint64_t* oldkeys;  // [64]
  uint4* nrows;       // [kIncrMaxNew][dpad / 8]
  float* dn;          // [kIncrMaxNew][kIncrMaxCand]
};
__host__ __device__ inline size_t incr_scratch_bytes(uint32_t dpad) {
  return 64 * 8 + size_t(kIncrMaxNew) * dpad * 2 + size_t(kIncrMaxNew) * kIncrMaxCand * 4;
}
__device__ __forceinline__ IncrScratch incr_carve(char* base, uint32_t dpad) {
  IncrScratch x;
  x.oldkeys = reinterpret_cast<uint64_t*>(base);
  x.nrows = reinterpret_cast<uint4*>(x.oldkeys + 64);
  x.dn = reinterpret_cast<float*>(reinterpret_cast<char*>(x.nrows) + size_t(kIncrMaxNew) * dpad * 2);
  return x;
}

// L2 with the candidate rows in registers (MAXC chunks per lane) only.
// oldtrust: bit a = existing edge a (x.oldkeys[a], a < na) is trusted.
template <int MAXC>
__device__ bool incremental_prune_and_write(const GraphView& g, uint32_t self, PruneSmem& sm,
                                            const IncrScratch& x, int na, int nc, float alpha,
                                            int lane, uint64_t oldtrust) {
  if (nc > kIncrMaxCand) return false;
  const int tile = lane >> 2, s = lane & 3;
  const int nchunks = int(g.dim / 8);
  const int stride = int(g.dpad / 8);
  // trusted positions: candidates whose key is a trusted existing edge's
  uint64_t t0 = 0, t1 = 0;
  for (int p0 = 0; p0 < nc; p0 += 32) {
    const int p = p0 + lane;
    bool tr = false;
    if (p < nc) {
      const uint64_t key = sm.cand[p];
      // a key present twice (an existing edge again as a sink) is trusted
      // at its first position only: the second is tested like a new one
      if (p == 0 || sm.cand[p - 1] != key)
        for (int j = 0; j < na; j++)
          if (x.oldkeys[j] == key) { tr = (oldtrust >> j) & 1ull; break; }
    }
    const uint64_t b = __ballot_sync(kFull, tr);
    if (p0 < 64) t0 |= b << p0; else t1 |= b << (p0 - 64);
  }
  const uint64_t u0 = ~t0 & (nc >= 64 ? ~0ull : ((1ull << nc) - 1ull));
  const uint64_t u1 = nc > 64 ? (~t1 & ((1ull << (nc - 64)) - 1ull)) : 0ull;
  const int nn = __popcll(u0) + __popcll(u1);
  if (nn > kIncrMaxNew) return false;
  // positions of the untrusted candidates, in order (the keys are no longer
  // needed: their slots hold the positions)
  int* upos = reinterpret_cast<int*>(x.oldkeys);
  __syncwarp();
  if (lane == 0) {
    uint64_t a = u0, b = u1;
    for (int k = 0; k < nn; k++) {
      if (a) { upos[k] = __ffsll(static_cast<long long>(a)) - 1; a &= a - 1; }
      else { upos[k] = 64 + __ffsll(static_cast<long long>(b)) - 1; b &= b - 1; }
    }
  }
  __syncwarp();
  // stage the untrusted rows
  for (int k = 0; k < nn; k++) {
    const int pk = upos[k];
    const uint4* row = reinterpret_cast<const uint4*>(
        g.vec + size_t(pair_id(sm.cand[pk]) - g.global_offset) * g.dpad);
    for (int c = lane; c < stride; c += 32) x.nrows[k * stride + c] = ldg16(row + c);
  }
  __syncwarp();
  // d(untrusted k, candidate j): each tile holds two candidate rows and runs
  // them against every staged row -- RowReg::dist's chunks and order
  for (int base = 0; base < nc; base += 16) {
    int jj[2];
    uint4 u[2][MAXC];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      jj[h] = base + tile + 8 * h;
      const bool act = jj[h] < nc;
      const uint4* row = reinterpret_cast<const uint4*>(
          g.vec + size_t(act ? pair_id(sm.cand[jj[h]]) - g.global_offset : 0) * g.dpad);
#pragma unroll
      for (int i = 0; i < MAXC; i++) {
        const int c = s + 4 * i;
        u[h][i] = (act && c < nchunks) ? ldg16(row + c) : make_uint4(0, 0, 0, 0);
      }
    }
    for (int k = 0; k < nn; k++) {
#pragma unroll
      for (int h = 0; h < 2; h++) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < MAXC; i++) {
          const int c = s + 4 * i;
          if (c < nchunks) acc = l2_chunk(u[h][i], x.nrows[k * stride + c], acc);
        }
        acc = tile4_sum(acc);
        if (s == 0 && jj[h] < nc) x.dn[k * kIncrMaxCand + jj[h]] = acc;
      }
    }
  }
  __syncwarp();
  // The walk of prune_and_write.  Between two untrusted candidates every
  // trusted one depends only on the untrusted candidates kept before it, so
  // a run of trusted candidates is decided at once; each untrusted candidate
  // is tested against everything kept before it.  The cap R keeps the first
  // R kept candidates.
  const uint32_t R = g.R;
  uint32_t ns = 0;
  uint64_t k0 = 0, k1 = 0;  // kept positions
  int lo = 0;               // first undecided position
  for (int k = 0; k <= nn && ns < R; k++) {
    const int hi = k < nn ? upos[k] : nc;  // next untrusted position
    // trusted run [lo, hi)
    for (int p0 = lo; p0 < hi && ns < R; p0 += 32) {
      const int p = p0 + lane;
      bool keep = false;
      if (p < hi) {
        const float cd = key_dist(sm.cand[p]);
        keep = true;
        for (int m = 0; m < k; m++) {
          const int pm = upos[m];
          const bool km = pm < 64 ? ((k0 >> pm) & 1ull) : ((k1 >> (pm - 64)) & 1ull);
          if (km && x.dn[m * kIncrMaxCand + p] * alpha < cd) keep = false;
        }
      }
      uint32_t bal = __ballot_sync(kFull, keep);
      const uint32_t room = R - ns;
      if (uint32_t(__popc(bal)) > room) {  // the walk stops at the R-th kept
        for (uint32_t r = uint32_t(__popc(bal)); r > room; r--) bal &= ~(1u << (31 - __clz(bal)));
      }
      if ((bal >> lane) & 1u) {
        const int slot = int(ns) + __popc(bal & ((1u << lane) - 1u));
        sm.sel[slot] = pair_id(sm.cand[p]);
        sm.sel_d[slot] = key_dist(sm.cand[p]);
      }
      const uint64_t wb = uint64_t(bal);
      if (p0 < 64) { k0 |= wb << p0; if (p0 > 32) k1 |= wb >> (64 - p0); }
      else k1 |= wb << (p0 - 64);
      ns += __popc(bal);
    }
    if (k == nn || ns >= R) break;
    // untrusted candidate at hi: every kept candidate before it
    const float cd = key_dist(sm.cand[hi]);
    bool p = false;
    for (int j = lane; j < hi; j += 32) {
      const bool kj = j < 64 ? ((k0 >> j) & 1ull) : ((k1 >> (j - 64)) & 1ull);
      if (kj && x.dn[k * kIncrMaxCand + j] * alpha < cd) p = true;
    }
    if (!__any_sync(kFull, p)) {
      if (lane == 0) {
        sm.sel[ns] = pair_id(sm.cand[hi]);
        sm.sel_d[ns] = cd;
      }
      if (hi < 64) k0 |= 1ull << hi; else k1 |= 1ull << (hi - 64);
      ns++;
    }
    lo = hi + 1;
  }
  __syncwarp();
  write_pruned_row(g, self, sm, ns, lane);
  return true;
}

// ---------------------------------------------------------------------------
// Gram-filtered RobustPrune for one reverse-edge target (dpad <= 128).
//
// The warp stages the nc <= kGramMax candidate rows in shared memory and
// computes their pairwise dot products G = X X^T with mma.sync m16n8k16
// (fp16 in, fp32 accumulate), one 16-row block row at a time, lower blocks
// only.  From G it forms an approximate pair distance
//     L2: d~ = G_ii + G_jj - 2 G_ij        IP: d~ = -G_ij
// and tests every kept row j against candidate i at once, one or two kept
// rows per lane.  The prune decision the reference takes is
// fl(d(i, j) * alpha) < cd with d(i, j) its tile-order fp32 sum.  With
// |d(i, j) - d~| <= eps (below), rounding is monotone, so
//     fl((d~ + eps) * alpha) <  cd  =>  pruned,
//     fl((d~ - eps) * alpha) >= cd  =>  not pruned by j,
// and only pairs inside the band are evaluated exactly, in the reference's
// order from the staged rows (exact_pair_smem).  The decisions, and so the kept list, are the
// ones prune_and_write takes.
//
// eps = 2^-12 (G_ii + G_jj).  Error budget: the fp16 products are exact in
// fp32; one m16n8k16 step adds 16 of them to the accumulator with an error
// of at most ~17 * 2^-23 of (sum of |terms| + |accumulator|), so over
// dpad/16 <= 8 steps G_ij is off by at most ~2^-15.7 sum |a_k b_k| <=
// 2^-16.7 (|a|^2 + |b|^2), and d~ by at most ~2^-14.7 (G_ii + G_jj).  The
// reference's fp32 tile-order sum is within ~(dpad/4 + 2) 2^-24 of the sum
// of its terms (<= 2 (|a|^2 + |b|^2)), i.e. below 2^-17 (G_ii + G_jj).  The
// total stays under 2^-14.4 (G_ii + G_jj), a 5x margin below eps.
// ---------------------------------------------------------------------------
#ifndef JB_GRAM_MAX
#define JB_GRAM_MAX 96
#endif
#ifndef JB_GRAM_WARPS
#define JB_GRAM_WARPS 2
#endif
constexpr int kGramMax = JB_GRAM_MAX;    // candidates per target on this path
#ifndef JB_GRAM_EPS_LOG2
#define JB_GRAM_EPS_LOG2 12
#endif
constexpr float kGramEps = 1.0f / float(1 << JB_GRAM_EPS_LOG2);
constexpr int kGramBrow = kGramMax + 8;  // floats per row of the block-row buffer

__host__ __device__ inline uint32_t gram_k(uint32_t dpad) { return (dpad + 15u) & ~15u; }
__host__ __device__ inline uint32_t gram_stride(uint32_t dpad) { return gram_k(dpad) * 2u + 16u; }
__host__ __device__ inline size_t gram_warp_bytes(uint32_t dpad) {
  const size_t b = size_t(kGramMax) * gram_stride(dpad) + size_t(16) * kGramBrow * 4 +
                   kGramMax * 4 + 64 * 4;
  return (b + 15) & ~size_t(15);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t sa = uint32_t(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* smem) {
  const uint32_t sa = uint32_t(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(sa));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// d(i, j) of two staged rows in the prune's own order, computed by the
// calling 4-lane tile: L2 over chunks 0 .. dim/8 - 1 (lane s: chunks s,
// s+4, ...), IP over all dpad/8 chunks (lane s: elements 8c + s, 8c + 4 + s),
// both reduced xor 2 then xor 1 -- RowReg::dist / dist_local with row i as
// the candidate.  nck is the number of staged chunks (dim/8 for L2, dpad/8
// for IP); the staged chunks are the rows' own bytes.
template <int METRIC>
__device__ __forceinline__ float exact_pair_smem(const char* rows, int stride, int i, int j,
                                                 int nck, int lane) {
  const int s = lane & 3;
  const uint4* ra = reinterpret_cast<const uint4*>(rows + size_t(i) * stride);
  const uint4* rb = reinterpret_cast<const uint4*>(rows + size_t(j) * stride);
  float acc = 0.f;
  if constexpr (METRIC == kL2) {
    for (int c = s; c < nck; c += 4) acc = l2_chunk(ra[c], rb[c], acc);
    return tile4_sum_local(acc, lane);
  } else {
    const uint32_t* a32 = reinterpret_cast<const uint32_t*>(ra);
    const uint32_t* b32 = reinterpret_cast<const uint32_t*>(rb);
    const int w = s >> 1;
    for (int c = 0; c < nck; c++)
      acc = ip_pair(a32[4 * c + w], a32[4 * c + 2 + w], b32[4 * c + w], b32[4 * c + 2 + w], s, acc);
    return -tile4_sum_local(acc, lane);
  }
}

// RobustPrune of sorted cand[0, nc) (nc <= kGramMax) through the Gram
// filter; writes the row of `self` like prune_and_write.
template <int METRIC>
__device__ void gram_prune_and_write(const GraphView& g, uint32_t self, PruneSmem& sm,
                                     char* gbase, int nc, float alpha, int lane) {
  const uint32_t R = g.R;
  const int K = int(gram_k(g.dpad));
  const int stride = int(gram_stride(g.dpad));
  const int nuse = METRIC == kL2 ? int(g.dim / 8) : int(g.dpad / 8);
  char* rows = gbase;
  float* brow = reinterpret_cast<float*>(gbase + size_t(kGramMax) * stride);
  float* norm = brow + 16 * kGramBrow;
  uint32_t* kpos = reinterpret_cast<uint32_t*>(norm + kGramMax);
  // Stage the rows: lane -> chunk (lane & 15) of row r0 + (lane >> 4).
  {
    const int kc = K / 8;
    const int c = lane & 15;
    for (int r = lane >> 4; r < nc; r += 2) {
      if (c >= kc) continue;
      char* dst = rows + size_t(r) * stride + c * 16;
      if (c < nuse) {
        const uint32_t id = pair_id(sm.cand[r]);
        cp_async16(dst, g.vec + size_t(id - g.global_offset) * g.dpad + c * 8);
      } else {
        *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_wait_all();
    __syncwarp();
  }
  const int gq = lane >> 2, tq = lane & 3;
  const int nb = (nc + 15) >> 4;
  const int nks = K / 16;
  uint32_t ns = 0;
  // ldmatrix row addresses: A rows (lane & 15), k half (lane >> 4);
  // B rows (lane & 7) + 8 (lane >> 4), k half ((lane >> 3) & 1).
  const int a_row = lane & 15, a_k = (lane >> 4) * 8;
  const int b_row = (lane & 7) + ((lane >> 4) << 3), b_k = ((lane >> 3) & 1) * 8;
  // This lane's kept slots lane and lane + 32: candidate position and norm.
  int kj[2] = {0, 0};
  float knorm[2] = {0.f, 0.f};
  for (int I = 0; I < nb && ns < R; I++) {
    uint32_t af[8][4];
#pragma unroll
    for (int kk = 0; kk < 8; kk++)
      if (kk < nks) ldsm_x4(af[kk], rows + size_t(16 * I + a_row) * stride + (16 * kk + a_k) * 2);
    for (int J = 0; J <= I; J++) {
      float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < 8; kk++) {
        if (kk < nks) {
          uint32_t bf[4];
          ldsm_x4(bf, rows + size_t(16 * J + b_row) * stride + (16 * kk + b_k) * 2);
          mma16816(c0, af[kk], bf[0], bf[1]);
          mma16816(c1, af[kk], bf[2], bf[3]);
        }
      }
      float* r0 = brow + gq * kGramBrow + 16 * J + 2 * tq;
      float* r1 = r0 + 8 * kGramBrow;
      *reinterpret_cast<float2*>(r0) = make_float2(c0[0], c0[1]);
      *reinterpret_cast<float2*>(r1) = make_float2(c0[2], c0[3]);
      *reinterpret_cast<float2*>(r0 + 8) = make_float2(c1[0], c1[1]);
      *reinterpret_cast<float2*>(r1 + 8) = make_float2(c1[2], c1[3]);
    }
    __syncwarp();
    if (lane < 16) norm[16 * I + lane] = brow[lane * kGramBrow + 16 * I + lane];
    __syncwarp();
    const int iend = min(nc, 16 * I + 16);
    for (int i = 16 * I; i < iend && ns < R; i++) {
      const uint64_t key = sm.cand[i];
      const uint32_t cid = pair_id(key);
      if (cid == self || cid == kInvalid) continue;
      const float cd = key_dist(key);
      const float* gr = brow + (i - 16 * I) * kGramBrow;
      const float ni = norm[i];
      bool pr = false;
      uint32_t amb = 0;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const uint32_t m = uint32_t(lane + 32 * h);
        if (m < ns) {
          const int j = kj[h];
          const float nj = knorm[h];
          const float gij = gr[j];
          const float approx = METRIC == kL2 ? __fsub_rn(__fadd_rn(ni, nj), __fmul_rn(2.f, gij)) : -gij;
          const float eps = __fmul_rn(__fadd_rn(ni, nj), kGramEps);
          if (__fmul_rn(__fadd_rn(approx, eps), alpha) < cd) pr = true;
          else if (!(__fmul_rn(__fsub_rn(approx, eps), alpha) >= cd)) amb |= 1u << h;
        }
      }
      bool pruned = __any_sync(kFull, pr);
      if (!pruned) {
        uint64_t am = uint64_t(__ballot_sync(kFull, amb & 1u)) |
                      (uint64_t(__ballot_sync(kFull, (amb >> 1) & 1u)) << 32);
        while (am != 0 && !pruned) {
          // tile t takes the t-th ambiguous kept row of this pass
          uint64_t rem = am;
          const int tile = lane >> 2;
          for (int t = 0; t < tile && rem; t++) rem &= rem - 1;
          bool p = false;
          if (rem != 0) {
            const int m = __ffsll(static_cast<long long>(rem)) - 1;
            const float d = exact_pair_smem<METRIC>(rows, stride, i, int(kpos[m]), nuse, lane);
            p = __fmul_rn(d, alpha) < cd;
          }
          pruned = __any_sync(kFull, p);
          for (int t = 0; t < 8 && am; t++) am &= am - 1;
        }
      }
      if (!pruned) {
        if (lane == 0) {
          sm.sel[ns] = cid;
          sm.sel_d[ns] = cd;
          kpos[ns] = uint32_t(i);
        }
        // kept slot ns lives in lane ns % 32, register ns / 32
        if (lane == int(ns & 31u)) {
          if (ns < 32) { kj[0] = i; knorm[0] = ni; }
          else { kj[1] = i; knorm[1] = ni; }
        }
        ns++;
        __syncwarp();
      }
    }
    __syncwarp();
  }
  __syncwarp();
  write_pruned_row(g, self, sm, ns, lane);
}

// (b) + (c) for batch rows [off, off + bs).
template <int MAXC, int METRIC>
__global__ void __launch_bounds__(128) batch_prune_kernel(GraphView g, uint32_t off, uint32_t bs,
                                                          const uint32_t* vis_idx,
                                                          const float* vis_dist,
                                                          const uint32_t* vis_cnt, uint32_t mrs,
                                                          float alpha) {
  extern __shared__ __align__(16) char smem_raw[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  PruneSmem sm = prune_carve(smem_raw + prune_warp_bytes(g.dpad, SelCache<MAXC, METRIC>::on) * wid, g.dpad);
  const uint32_t R = g.R;
  const uint32_t nwarps = gridDim.x * (blockDim.x >> 5);
  for (uint32_t b = blockIdx.x * (blockDim.x >> 5) + wid; b < bs; b += nwarps) {
    const uint32_t gid = off + b;
    const uint32_t l = gid - g.global_offset;
    int nc = 0;
    const uint32_t ne = g.counts[l];
    for (uint32_t base = 0; base < ne; base += 32) {
      const uint32_t e = base + lane;
      uint32_t id = e < ne ? g.edges[size_t(l) * R + e] : kInvalid;
      const bool ok = e < ne && id != kInvalid;
      const uint32_t bal = __ballot_sync(kFull, ok);
      if (ok) {
        const float d = bf16_bits_to_float(g.edist[size_t(l) * R + e]);
        sm.cand[nc + __popc(bal & ((1u << lane) - 1u))] = make_pair_key(d, id);
      }
      nc += __popc(bal);
    }
    const uint32_t vc = vis_cnt[b];
    for (uint32_t base = 0; base < vc; base += 32) {
      const uint32_t i = base + lane;
      uint32_t id = i < vc ? vis_idx[size_t(b) * mrs + i] : kInvalid;
      const bool ok = i < vc && id != gid && id != kInvalid;
      const uint32_t bal = __ballot_sync(kFull, ok);
      if (ok) sm.cand[nc + __popc(bal & ((1u << lane) - 1u))] =
          make_pair_key(vis_dist[size_t(b) * mrs + i], id);
      nc += __popc(bal);
    }
    __syncwarp();
    sort_cands(sm.cand, nc, lane);
    prune_and_write<MAXC, METRIC>(g, gid, sm, nc, alpha, lane);
  }
}

// (d) reverse pairs: key = target << 32 | sink, empty slots = max key.
__global__ void fill_reverse_kernel(GraphView g, uint32_t off, uint32_t bs, uint64_t* keys) {
  const size_t total = size_t(bs) * g.R;
  for (size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += size_t(gridDim.x) * blockDim.x) {
    const uint32_t b = uint32_t(t / g.R), e = uint32_t(t % g.R);
    const uint32_t gid = off + b;
    const uint32_t l = gid - g.global_offset;
    uint64_t k = kKeyMax;
    if (e < g.counts[l]) k = (uint64_t(g.edges[size_t(l) * g.R + e]) << 32) | gid;
    keys[t] = k;
  }
}

__global__ void group_starts_kernel(const uint64_t* keys, size_t total, uint32_t* starts,
                                    uint32_t* n_groups) {
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += size_t(gridDim.x) * blockDim.x) {
    const uint64_t k = keys[i];
    if (k == kKeyMax) continue;
    if (i == 0 || (keys[i - 1] >> 32) != (k >> 32)) starts[atomicAdd(n_groups, 1u)] = uint32_t(i);
  }
}

// (d') The semisort: a stable LSD radix sort of the reverse pairs on their
// target id alone.  The pairs are produced sink-major (pair b * R + e belongs
// to batch row b), so among equal targets input order is already ascending
// sink order, and a stable sort by target yields the (target, sink) order of
// the reference's thrust sort (construct.cuh:832-879) exactly.  Targets are
// taken relative to the graph's first id; empty slots (target 0xFFFFFFFF)
// map to n and so sort after every real target.  8-bit digits: per pass a
// per-block digit histogram, an exclusive scan of every digit's row of block
// counts (one block per digit), and a stable scatter that adds the digits'
// bases and ranks each warp's keys round by round with __match_any_sync.
constexpr int kSortThreads = 256, kSortItems = 16, kSortTile = kSortThreads * kSortItems;
constexpr int kSortWarps = kSortThreads / 32;

__device__ __forceinline__ uint32_t sort_digit(uint64_t k, uint32_t first, uint32_t n, int shift) {
  uint32_t t = uint32_t(k >> 32) - first;
  if (t > n) t = n;
  return (t >> shift) & 0xFFu;
}

__global__ void __launch_bounds__(kSortThreads) radix_hist_kernel(const uint64_t* keys, size_t total,
                                                                  uint32_t first, uint32_t n,
                                                                  int shift, uint32_t* counts,
                                                                  uint32_t nblocks) {
  __shared__ uint32_t h[256];
  for (int i = threadIdx.x; i < 256; i += kSortThreads) h[i] = 0;
  __syncthreads();
  const size_t base = size_t(blockIdx.x) * kSortTile;
  for (int j = threadIdx.x; j < kSortTile; j += kSortThreads) {
    const size_t i = base + j;
    if (i < total) atomicAdd(&h[sort_digit(keys[i], first, n, shift)], 1u);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < 256; d += kSortThreads) counts[size_t(d) * nblocks + blockIdx.x] = h[d];
}

// Exclusive prefix sum of digit d's row counts[d][0, nblocks) in place, one
// block per digit; the row total goes to totals[d].
__global__ void __launch_bounds__(1024) digit_rows_scan_kernel(uint32_t* counts, uint32_t nblocks,
                                                               uint32_t* totals) {
  __shared__ uint32_t wsum[32];
  __shared__ uint32_t carry;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t* a = counts + size_t(blockIdx.x) * nblocks;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (uint32_t base = 0; base < nblocks; base += 1024) {
    const uint32_t i = base + threadIdx.x;
    const uint32_t v = i < nblocks ? a[i] : 0u;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(kFull, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
      uint32_t t = wsum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(kFull, t, o);
        if (lane >= o) t += y;
      }
      wsum[lane] = t;
    }
    __syncthreads();
    const uint32_t before = carry + (w ? wsum[w - 1] : 0u);
    if (i < nblocks) a[i] = before + x - v;
    __syncthreads();
    if (threadIdx.x == 0) carry += wsum[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) totals[blockIdx.x] = carry;
}

__global__ void __launch_bounds__(kSortThreads) radix_scatter_kernel(const uint64_t* in, uint64_t* out,
                                                                     size_t total, uint32_t first,
                                                                     uint32_t n, int shift,
                                                                     const uint32_t* offsets,
                                                                     uint32_t nblocks,
                                                                     const uint32_t* totals) {
  __shared__ uint32_t wh[kSortWarps][256];
  __shared__ uint32_t digit_base[256];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kSortWarps * 256; i += kSortThreads) (&wh[0][0])[i] = 0;
  if (w == 0) {  // exclusive prefix of the 256 digit totals, 8 per lane
    uint32_t v[8], run = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) { v[j] = totals[8 * lane + j]; run += v[j]; }
    uint32_t x = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(kFull, x, o);
      if (lane >= o) x += y;
    }
    uint32_t b = x - run;
#pragma unroll
    for (int j = 0; j < 8; j++) { digit_base[8 * lane + j] = b; b += v[j]; }
  }
  __syncthreads();
  // warp w holds keys [wbase, wbase + 32 * kSortItems) of the block's tile,
  // round u covering 32 consecutive keys, so (warp, round, lane) is input order
  const size_t wbase = size_t(blockIdx.x) * kSortTile + size_t(w) * 32 * kSortItems;
  const uint32_t lt = (1u << lane) - 1u;
  uint64_t key[kSortItems];
  uint32_t rank[kSortItems];
#pragma unroll
  for (int u = 0; u < kSortItems; u++) {
    const size_t i = wbase + size_t(u) * 32 + lane;
    const bool valid = i < total;
    key[u] = valid ? in[i] : 0ull;
    const uint32_t d = valid ? sort_digit(key[u], first, n, shift) : 256u;
    const uint32_t peers = __match_any_sync(kFull, d);
    const uint32_t before = valid ? wh[w][d] : 0u;
    __syncwarp();
    if (valid && lane == __ffs(peers) - 1) wh[w][d] = before + __popc(peers);
    __syncwarp();
    rank[u] = before + __popc(peers & lt);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < 256; d += kSortThreads) {  // warps in input order
    uint32_t run = 0;
#pragma unroll
    for (int ww = 0; ww < kSortWarps; ww++) {
      const uint32_t c = wh[ww][d];
      wh[ww][d] = run;
      run += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int u = 0; u < kSortItems; u++) {
    const size_t i = wbase + size_t(u) * 32 + lane;
    if (i < total) {
      const uint32_t d = sort_digit(key[u], first, n, shift);
      out[digit_base[d] + offsets[size_t(d) * nblocks + blockIdx.x] + wh[w][d] + rank[u]] = key[u];
    }
  }
}

// Sorts keys[0, total) (contents clobbered) using tmp; returns the buffer
// holding the sorted keys.
const uint64_t* sort_reverse_pairs(uint64_t* keys, uint64_t* tmp, size_t total, uint32_t first,
                                   uint32_t n, uint32_t* counts, cudaStream_t st) {
  if (total == 0) return keys;
  const int bits = 32 - __builtin_clz(n | 1u);  // digits of 0 .. n
  const int passes = (bits + 7) / 8;
  const uint32_t nblocks = uint32_t((total + kSortTile - 1) / kSortTile);
  uint64_t* src = keys;
  uint64_t* dst = tmp;
  for (int p = 0; p < passes; p++) {
    radix_hist_kernel<<<nblocks, kSortThreads, 0, st>>>(src, total, first, n, 8 * p, counts, nblocks);
    digit_rows_scan_kernel<<<256, 1024, 0, st>>>(counts, nblocks, counts + size_t(256) * nblocks);
    radix_scatter_kernel<<<nblocks, kSortThreads, 0, st>>>(src, dst, total, first, n, 8 * p, counts,
                                                          nblocks, counts + size_t(256) * nblocks);
    uint64_t* t = src; src = dst; dst = t;
  }
  return src;
}

// (e) one warp per reverse-edge target.
// PASS 0: every target group, one kernel (incremental prune when GRAM
//         applies to L2 register rows, else the Gram / plain prune);
// PASS 1: every group, incremental prune only: a group it cannot take is
//         appended to `deferred`.  No Gram scratch, so several times the
//         warps fit per SM;
// PASS 2: the deferred groups, Gram / plain prune.
template <int MAXC, int METRIC, bool GRAM, int PASS>
__global__ void __launch_bounds__(128) reverse_prune_kernel(GraphView g, const uint64_t* keys,
                                                            size_t total, const uint32_t* starts,
                                                            const uint32_t* n_groups, float alpha,
                                                            uint32_t* deferred,
                                                            uint32_t* n_deferred) {
  extern __shared__ __align__(16) char smem_raw[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int tile = lane >> 2, s = lane & 3;
  const size_t wbytes = prune_warp_bytes(g.dpad, SelCache<MAXC, METRIC>::on);
  const size_t gbytes = PASS == 1 ? incr_scratch_bytes(g.dpad) : (GRAM ? gram_warp_bytes(g.dpad) : 0);
  char* wbase = smem_raw + (wbytes + gbytes) * wid;
  PruneSmem sm = prune_carve(wbase, g.dpad);
  const uint32_t R = g.R;
  const uint32_t cap = 256 + R;  // MAX_CANDS of construct.cuh:574
  const uint32_t ng = PASS == 2 ? *n_deferred : *n_groups;
  const uint32_t nwarps = gridDim.x * (blockDim.x >> 5);
  const int nchunks = int(g.dim / 8);
  for (uint32_t gw = blockIdx.x * (blockDim.x >> 5) + wid; gw < ng; gw += nwarps) {
    const uint32_t gi = PASS == 2 ? deferred[gw] : gw;
    const size_t start = starts[gi];
    const uint32_t t = uint32_t(keys[start] >> 32);
    const uint32_t l = t - g.global_offset;
    int nc = 0;
    const uint32_t ne = g.counts[l];
    constexpr bool kIncr = (PASS == 1) || (PASS == 0 && GRAM && MAXC > 0 && METRIC == kL2);
    const uint64_t rowflags = (kIncr && g.eflag != nullptr) ? g.eflag[l] : 0ull;
    uint64_t oldtrust = 0;  // trusted existing edges by index in cand
    for (uint32_t base = 0; base < ne; base += 32) {
      const uint32_t e = base + lane;
      uint32_t id = e < ne ? g.edges[size_t(l) * R + e] : kInvalid;
      const bool ok = e < ne && id != kInvalid;
      const uint32_t bal = __ballot_sync(kFull, ok);
      const int p = nc + __popc(bal & ((1u << lane) - 1u));
      if (ok) sm.cand[p] = make_pair_key(bf16_bits_to_float(g.edist[size_t(l) * R + e]), id);
      if (ok && ((rowflags >> e) & 1ull) && p < 64) oldtrust |= 1ull << p;
      nc += __popc(bal);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) oldtrust |= __shfl_xor_sync(kFull, oldtrust, o);
    const IncrScratch incr = incr_carve(wbase + wbytes, g.dpad);
    if (kIncr && oldtrust != 0)
      for (int i = lane; i < nc; i += 32) incr.oldkeys[i] = sm.cand[i];
#ifdef JB_BUILD_CLOCKS
    long long _c0 = clock64();
#endif
    const int na = nc;
    RowReg<MAXC, METRIC> tr;
    tr.load(g, t, nchunks, lane, sm.row);
    // The group is the contiguous run of keys with this target.
    size_t end = start;
    for (;;) {
      const size_t i = end + lane;
      const bool in = i < total && keys[i] != kKeyMax && uint32_t(keys[i] >> 32) == t;
      const uint32_t bal = __ballot_sync(kFull, in);
      if (bal == kFull) { end += 32; continue; }
      end += __ffs(~bal) - 1;
      break;
    }
    // Sinks with fresh distances, 16 per pass (two rows per 4-lane tile), in
    // group order, until the candidate cap.
    for (size_t i = start; i < end && nc < int(cap); i += 16) {
      const size_t i0 = i + tile, i1 = i + tile + 8;
      const uint32_t s0 = i0 < end ? uint32_t(keys[i0]) : kInvalid;
      const uint32_t s1 = i1 < end ? uint32_t(keys[i1]) : kInvalid;
      const bool a0 = i0 < end && s0 != t && s0 != kInvalid;
      const bool a1 = i1 < end && s1 != t && s1 != kInvalid;
      const float d0 = tr.dist(g, a0 ? s0 : t, a0, nchunks, s);
      const float d1 = tr.dist(g, a1 ? s1 : t, a1, nchunks, s);
      const uint32_t b0 = __ballot_sync(kFull, a0 && s == 0);
      const uint32_t b1 = __ballot_sync(kFull, a1 && s == 0);
      if (s == 0) {
        const uint32_t lt = (1u << lane) - 1u;
        const int p0 = nc + __popc(b0 & lt);
        const int p1 = nc + __popc(b0) + __popc(b1 & lt);
        if (a0 && p0 < int(cap)) sm.cand[p0] = make_pair_key(d0, s0);
        if (a1 && p1 < int(cap)) sm.cand[p1] = make_pair_key(d1, s1);
      }
      nc = min(int(cap), nc + __popc(b0) + __popc(b1));
      __syncwarp();
    }
    __syncwarp();
#ifdef JB_BUILD_CLOCKS
    long long _c1 = clock64();
#endif
    sort_cands_merge(sm.cand, na, nc, lane);
#ifdef JB_BUILD_CLOCKS
    long long _c2 = clock64();
#endif
    if (kIncr && oldtrust != 0 &&
        incremental_prune_and_write<(MAXC > 0 ? MAXC : 1)>(g, t, sm, incr, na, nc, alpha, lane,
                                                           oldtrust)) {
#ifdef JB_BUILD_CLOCKS
      if (lane == 0) {
        atomicAdd(&g_build_clk[4], 1ull);
        atomicAdd(&g_build_clk[5], (unsigned long long)(clock64() - _c2));
      }
#endif
    } else if (PASS == 1) {
      if (lane == 0) deferred[atomicAdd(n_deferred, 1u)] = gi;
    } else if (GRAM && nc <= kGramMax) {
      gram_prune_and_write<METRIC>(g, t, sm, wbase + wbytes, nc, alpha, lane);
    } else {
      prune_and_write<MAXC, METRIC>(g, t, sm, nc, alpha, lane);
    }
#ifdef JB_BUILD_CLOCKS
    long long _c3 = clock64();
    if (lane == 0) {
      atomicAdd(&g_build_clk[0], (unsigned long long)(_c1 - _c0));
      atomicAdd(&g_build_clk[1], (unsigned long long)(_c2 - _c1));
      atomicAdd(&g_build_clk[2], (unsigned long long)(_c3 - _c2));
      atomicAdd(&g_build_clk[3], 1ull);
      atomicAdd(&g_build_clk[6], (unsigned long long)nc);
    }
#endif
  }
}

// The Gram filter takes the same prune decisions as the plain loop; the
// environment variable JB_GRAM_PRUNE=0 selects the plain loop (for timing
// comparisons).
bool gram_prune_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("JB_GRAM_PRUNE");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

template <int MAXC, int METRIC>
struct Kernels {
  static void prune(const GraphView& g, uint32_t off, uint32_t bs, const BuildWorkspace& ws,
                    float alpha, cudaStream_t st) {
    const size_t smem = prune_warp_bytes(g.dpad, SelCache<MAXC, METRIC>::on) * 4;
    auto k = batch_prune_kernel<MAXC, METRIC>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    const uint32_t blocks = (bs + 3) / 4;
    k<<<blocks, 128, smem, st>>>(g, off, bs, ws.vis_idx, ws.vis_dist, ws.vis_cnt, kBuildMaxResult,
                                 alpha);
  }
  template <bool GRAM, int PASS>
  static void reverse_launch(const GraphView& g, size_t total, const BuildWorkspace& ws,
                             const uint64_t* sorted, float alpha, cudaStream_t st) {
    const int warps = PASS == 1 ? 4 : (GRAM ? JB_GRAM_WARPS : 4);
    const size_t extra = PASS == 1 ? incr_scratch_bytes(g.dpad) : (GRAM ? gram_warp_bytes(g.dpad) : 0);
    const size_t smem = (prune_warp_bytes(g.dpad, SelCache<MAXC, METRIC>::on) + extra) * warps;
    auto k = reverse_prune_kernel<MAXC, METRIC, GRAM, PASS>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    int dev = 0, sms = 0, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, 32 * warps, smem);
    if (per_sm < 1) per_sm = 1;
    size_t blocks = size_t(sms) * per_sm;
    const size_t need = (total + warps - 1) / warps;
    if (blocks > need) blocks = need;
    if (blocks == 0) blocks = 1;
    k<<<uint32_t(blocks), 32 * warps, smem, st>>>(g, sorted, total, ws.group_starts,
                                                  ws.counters + 1, alpha, ws.deferred,
                                                  ws.counters + 2);
  }
  static void reverse(const GraphView& g, size_t total, const BuildWorkspace& ws,
                      const uint64_t* sorted, float alpha, cudaStream_t st) {
    const bool gram = gram_prune_enabled() && g.dpad <= 128 && alpha > 0.f;
    if (gram && g.eflag != nullptr && MAXC > 0 && METRIC == kL2) {
      // incremental targets at high occupancy, then the rest with the Gram filter
      reverse_launch<false, 1>(g, total, ws, sorted, alpha, st);
      reverse_launch<true, 2>(g, total, ws, sorted, alpha, st);
    } else if (gram) {
      reverse_launch<true, 0>(g, total, ws, sorted, alpha, st);
    } else {
      reverse_launch<false, 0>(g, total, ws, sorted, alpha, st);
    }
  }
};

template <int METRIC>
void dispatch_prune(const GraphView& g, uint32_t off, uint32_t bs, const BuildWorkspace& ws,
                    float alpha, cudaStream_t st, bool reverse, size_t total,
                    const uint64_t* sorted = nullptr) {
  const uint32_t nchunks = g.dim / 8;
  auto run = [&](auto kernels) {
    if (reverse) decltype(kernels)::reverse(g, total, ws, sorted, alpha, st);
    else decltype(kernels)::prune(g, off, bs, ws, alpha, st);
  };
  if (METRIC == kIP) return run(Kernels<0, METRIC>{});
  if (nchunks <= 4) return run(Kernels<1, METRIC>{});
  if (nchunks <= 8) return run(Kernels<2, METRIC>{});
  if (nchunks <= 12) return run(Kernels<3, METRIC>{});
  if (nchunks <= 16) return run(Kernels<4, METRIC>{});
  if (nchunks <= 32) return run(Kernels<8, METRIC>{});
  return run(Kernels<0, METRIC>{});
}

}  // namespace

#ifdef JB_BUILD_CLOCKS
extern "C" int jb_debug_build_clocks(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, g_build_clk, sizeof(unsigned long long) * 8) == cudaSuccess ? 0 : 1;
}
#endif

uint32_t reference_max_batch_size(uint64_t budget_bytes, uint32_t n, uint32_t R) {
  // graph_construct_workspace::max_batch_size_for_budget (construct.cuh:233-258)
  // with L = 64, max_result_size = 256, entry = 8 B, edge_pair = 8 B, index = 4 B,
  // then min(., n / 50) as ConstructGraph does (ffi/jasper_ffi_common.cuh:245-248).
  const uint64_t L = 64, mrs = 256;
  const uint64_t per_item = 8 * L + 8 * mrs + 4 + 8 * (mrs + R) + 4 + 8ull * R + 4ull * R + 4ull * R;
  const uint64_t fixed = 4;
  uint64_t b = budget_bytes <= fixed ? 0 : (budget_bytes - fixed) / per_item;
  if (b > 0xFFFFFFFFull) b = 0xFFFFFFFFull;
  uint32_t batch = uint32_t(b);
  uint32_t cap = n / 50;
  return batch < cap ? batch : cap;
}

void workspace_allocate(BuildWorkspace& ws, uint32_t max_batch, uint32_t R) {
  ws = BuildWorkspace{};
  ws.max_batch = max_batch;
  const size_t pairs = size_t(max_batch) * R;
  check(cudaMalloc(&ws.vis_idx, size_t(max_batch) * kBuildMaxResult * 4), "alloc visited ids");
  check(cudaMalloc(&ws.vis_dist, size_t(max_batch) * kBuildMaxResult * 4), "alloc visited dists");
  check(cudaMalloc(&ws.vis_cnt, size_t(max_batch) * 4), "alloc visited counts");
  check(cudaMalloc(&ws.rev_keys, pairs * 8), "alloc reverse pairs");
  check(cudaMalloc(&ws.rev_sorted, pairs * 8), "alloc sorted reverse pairs");
  check(cudaMalloc(&ws.group_starts, pairs * 4), "alloc group starts");
  check(cudaMalloc(&ws.deferred, pairs * 4 + 4), "alloc deferred groups");
  check(cudaMalloc(&ws.counters, 256), "alloc counters");
  ws.sort_tmp_bytes = size_t(256) * ((pairs + kSortTile - 1) / kSortTile + 1) * 4;
  check(cudaMalloc(&ws.sort_tmp, ws.sort_tmp_bytes ? ws.sort_tmp_bytes : 16), "alloc sort counts");
}

void workspace_free(BuildWorkspace& ws) {
  cudaFree(ws.vis_idx); cudaFree(ws.vis_dist); cudaFree(ws.vis_cnt);
  cudaFree(ws.rev_keys); cudaFree(ws.rev_sorted); cudaFree(ws.group_starts); cudaFree(ws.deferred);
  cudaFree(ws.counters); cudaFree(ws.sort_tmp);
  ws = BuildWorkspace{};
}

// JB_INCR_PRUNE=0 in the environment turns the incremental reverse prune
// (and the flags it keeps) off, for timing comparisons; the graphs are the
// same either way.
bool incr_prune_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("JB_INCR_PRUNE");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

void process_batch(Graph& graph, BuildWorkspace& ws, uint32_t off, uint32_t bs, float alpha,
                   cudaStream_t st) {
  GraphView g = graph.view();
  if (!incr_prune_enabled()) g.eflag = nullptr;
  check(cudaMemsetAsync(ws.counters, 0, 256, st), "clear counters");
  SearchArgs a{};
  a.g = g;
  a.use_range = 1;
  a.query_start = off;
  a.nq = bs;
  a.k = kBuildL;
  a.bw = kBuildL;
  a.limit = kBuildLimit;
  a.max_result_size = kBuildMaxResult;
  a.vis_idx = ws.vis_idx;
  a.vis_dist = ws.vis_dist;
  a.vis_cnt = ws.vis_cnt;
  a.work_counter = ws.counters;
  launch_search(a, st);
  if (g.metric == kIP) dispatch_prune<kIP>(g, off, bs, ws, alpha, st, false, 0);
  else dispatch_prune<kL2>(g, off, bs, ws, alpha, st, false, 0);
  const size_t total = size_t(bs) * g.R;
  const uint32_t fb = uint32_t(std::min<size_t>((total + 255) / 256, 4096));
  fill_reverse_kernel<<<fb, 256, 0, st>>>(g, off, bs, ws.rev_keys);
  const uint64_t* sorted = sort_reverse_pairs(ws.rev_keys, ws.rev_sorted, total, g.global_offset,
                                              g.n, static_cast<uint32_t*>(ws.sort_tmp), st);
  group_starts_kernel<<<fb, 256, 0, st>>>(sorted, total, ws.group_starts, ws.counters + 1);
  if (g.metric == kIP) dispatch_prune<kIP>(g, off, bs, ws, alpha, st, true, total, sorted);
  else dispatch_prune<kL2>(g, off, bs, ws, alpha, st, true, total, sorted);
  check(cudaGetLastError(), "construct batch launch");
}

// The build's prune flags (GraphView::eflag), zero (nothing trusted) for
// rows whose edges no prune of this process wrote.
void ensure_prune_flags(Graph& g) {
  if (g.eflag != nullptr || g.on_host) return;
  const size_t rows = std::max<size_t>(g.capacity, 1);
  check(cudaMalloc(&g.eflag, rows * 8), "alloc prune flags");
  check(cudaMemset(g.eflag, 0, rows * 8), "clear prune flags");
}

// append_batch (include/jasper/index/construct.cuh:1169-1265): the new rows
// take slots [n, n + count), their edges are wired by process_batch in
// batches of min(count, 100000) rows -- no ramp -- and they get the stable
// ids next_id, next_id + 1, ...  Arrays grow geometrically (1.5x), so a
// sequence of appends costs amortised O(rows appended) in copies.
std::vector<uint32_t> graph_append(Graph& graph, const uint16_t* rows, uint64_t count,
                                   uint32_t stride, float alpha, cudaStream_t st) {
  std::vector<uint32_t> ids;
  if (count == 0) return ids;
  if (graph.on_host) throw std::runtime_error("append requires a device-resident graph");
  if (graph.global_offset != 0) throw std::runtime_error("append requires global_offset == 0");
  if (graph.dir.has_lsh || graph.dir.has_pq || graph.dir.has_rabitq || graph.dir.prerotate)
    throw std::runtime_error("append is for plain graphs (the graph has directional, RaBitQ or "
                             "prerotation artifacts)");
  if (stride < graph.dim) throw std::invalid_argument("row stride is smaller than dim");
  const uint64_t old_n = graph.n, new_n = old_n + count;
  if (new_n >= 0x7FFFFFFFull) throw std::invalid_argument("graphs are limited to 2^31 - 1 rows");
  if (graph.next_id + count > 0xFFFFFFFFull) throw std::runtime_error("stable ids exhausted");
  if (new_n > graph.capacity) {
    const uint64_t grown = uint64_t(graph.capacity) + graph.capacity / 2;
    graph_reserve(graph, uint32_t(std::min<uint64_t>(std::max(new_n, grown), 0x7FFFFFFEull)));
  }
  const size_t dp = graph.dpad;
  uint16_t* dst = graph.vec + old_n * dp;
  if (dp != graph.dim) check(cudaMemsetAsync(dst, 0, count * dp * 2, st), "clear appended rows");
  check(cudaMemcpy2DAsync(dst, dp * 2, rows, size_t(stride) * 2, size_t(graph.dim) * 2, count,
                          cudaMemcpyDefault, st),
        "copy appended rows");
  check(cudaMemsetAsync(graph.counts + old_n, 0, count, st), "clear appended counts");
  ids.resize(count);
  for (uint64_t i = 0; i < count; i++) ids[i] = uint32_t(graph.next_id + i);
  check(cudaMemcpyAsync(graph.slot_to_id + old_n, ids.data(), count * 4, cudaMemcpyHostToDevice,
                        st),
        "write appended ids");
  check(cudaStreamSynchronize(st), "append upload");
  if (graph.next_id != old_n) graph.ids_identity = false;
  graph.n = uint32_t(new_n);
  graph.next_id += count;
  const uint32_t max_batch = uint32_t(std::min<uint64_t>(count, 100000));
  ensure_prune_flags(graph);
  BuildWorkspace ws;
  workspace_allocate(ws, max_batch, graph.R);
  try {
    for (uint64_t off = old_n; off < new_n;) {
      const uint32_t bs = uint32_t(std::min<uint64_t>(max_batch, new_n - off));
      process_batch(graph, ws, uint32_t(off), bs, alpha, st);
      off += bs;
    }
    check(cudaStreamSynchronize(st), "append");
  } catch (...) {
    cudaStreamSynchronize(st);
    workspace_free(ws);
    throw;
  }
  workspace_free(ws);
  return ids;
}

void construct_graph(Graph& graph, float alpha, uint32_t max_batch, cudaStream_t st) {
  if (max_batch == 0) max_batch = 1;
  if (graph.n == 0) return;
  ensure_prune_flags(graph);
  BuildWorkspace ws;
  workspace_allocate(ws, max_batch, graph.R);
  try {
    uint32_t count = 0, bs = 1;
    while (count < graph.n) {
      bs = std::min(bs, graph.n - count);
      bs = std::min(bs, max_batch);
      process_batch(graph, ws, graph.global_offset + count, bs, alpha, st);
      count += bs;
      if (bs < max_batch) bs = std::min(max_batch, bs * 2);
    }
    check(cudaStreamSynchronize(st), "construct");
  } catch (...) {
    cudaStreamSynchronize(st);
    workspace_free(ws);
    throw;
  }
  workspace_free(ws);
}

}  // namespace jb
