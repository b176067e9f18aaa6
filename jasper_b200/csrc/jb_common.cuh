// jb_common.cuh -- device helpers shared by the search and build kernels.
//
// Beam entries are 64-bit keys that sort in the reference's CustomPairLess
// order (include/jasper/beam_search/device_kernels.cuh:132-151: distance
// ascending, then 31-bit id ascending):
//     key = ordered_bits(dist) << 32 | id << 1 | visited
// ordered_bits() maps an IEEE float to an unsigned integer with the same
// order, so one 64-bit integer compare is the reference comparator.  The
// visited flag lives in bit 0 below the id: it never decides the order of two
// distinct ids, and the beam never holds two copies of one id.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace jb {

constexpr uint32_t kFull = 0xFFFFFFFFu;
constexpr uint32_t kInvalid = 0xFFFFFFFFu;
constexpr uint64_t kKeyMax = ~0ull;

__device__ __forceinline__ uint32_t ordered_bits(float d) {
  d = d + 0.0f;  // -0.0 -> +0.0: the reference compares floats, where they tie
  uint32_t u = __float_as_uint(d);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float from_ordered_bits(uint32_t u) {
  u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
  return __uint_as_float(u);
}

__device__ __forceinline__ uint64_t make_key(float d, uint32_t id) {
  return (uint64_t(ordered_bits(d)) << 32) | (uint64_t(id & 0x7FFFFFFFu) << 1);
}
__device__ __forceinline__ uint32_t key_id(uint64_t k) { return uint32_t(k) >> 1; }
__device__ __forceinline__ float key_dist(uint64_t k) { return from_ordered_bits(uint32_t(k >> 32)); }
__device__ __forceinline__ bool key_visited(uint64_t k) { return k & 1ull; }

// Candidate pairs of the build (id is a full 32-bit id there, no flag).
__device__ __forceinline__ uint64_t make_pair_key(float d, uint32_t id) {
  return (uint64_t(ordered_bits(d)) << 32) | uint64_t(id);
}
__device__ __forceinline__ uint32_t pair_id(uint64_t k) { return uint32_t(k); }

// Read-only 16-byte gather through the non-coherent path.
// Hint: bring the 128-byte line holding p into L2 (no register, no wait).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ uint4 ldg16(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// sm_100 mixed-precision arithmetic: the fp16 operands are widened exactly
// inside the instruction, so each gives the same bits as converting first
// and then using the fp32 instruction -- with fewer instructions.
#ifndef JB_MIXED_ADD
#define JB_MIXED_ADD 1
#endif
// fl(f32(h) + c), h the low fp16 half of w
__device__ __forceinline__ float add_f32_f16(uint32_t w, float c) {
  float d;
  const unsigned short h = static_cast<unsigned short>(w & 0xFFFFu);
  asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(d) : "h"(h), "f"(c));
  return d;
}
// fl(f32(h) - c), h the low fp16 half of w
__device__ __forceinline__ float sub_f32_f16(uint32_t w, float c) {
  float d;
  const unsigned short h = static_cast<unsigned short>(w & 0xFFFFu);
  asm("sub.rn.f32.f16 %0, %1, %2;" : "=f"(d) : "h"(h), "f"(c));
  return d;
}
// fl(f32(a) * f32(b) + c) (one rounding; the product of two fp16 values is
// exact in fp32), a and b the low fp16 halves of wa and wb
__device__ __forceinline__ float fma_f32_f16(uint32_t wa, uint32_t wb, float c) {
  float d;
  const unsigned short a = static_cast<unsigned short>(wa & 0xFFFFu);
  const unsigned short b = static_cast<unsigned short>(wb & 0xFFFFu);
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}

// The query's prerotation, fused into a search prologue (one warp per query):
// y_i = fp16(sum_k x_k P[k][i]) for i < d, 0 for d <= i < dpad, with the sum
// taken in k order by fp32 fma -- the order of the SIMT rotation GEMM
// (rotate.cu, rotate_kernel), which walks k in tiles of 32 and adds the zero
// products of a partial last tile (one fma(0, 0, acc) is the same as several).
// x, y: padded fp16 rows in shared memory (x's pad lanes zero); Mp: dpad x
// dpad, row i = column i of P, zero padded (16-byte aligned rows).
static __device__ __noinline__ void rotate_query_warp(const uint16_t* x, uint16_t* y,
                                                  const uint16_t* Mp, uint32_t d, uint32_t dpad,
                                                  int lane) {
  const uint4* x4 = reinterpret_cast<const uint4*>(x);
  for (uint32_t i = lane; i < dpad; i += 32) {
    float acc = 0.0f;
    if (i < d) {
      const uint4* row = reinterpret_cast<const uint4*>(Mp + size_t(i) * dpad);
      for (uint32_t c = 0; c < dpad / 8; c++) {
        const uint4 pw = ldg16(row + c), xw = x4[c];
        const uint32_t pv[4] = {pw.x, pw.y, pw.z, pw.w}, xv[4] = {xw.x, xw.y, xw.z, xw.w};
#pragma unroll
        for (int w = 0; w < 4; w++) {
          const uint32_t k = 8 * c + 2 * w;
#if JB_MIXED_ADD
          if (k < d) acc = fma_f32_f16(xv[w], pv[w], acc);
          if (k + 1 < d) acc = fma_f32_f16(xv[w] >> 16, pv[w] >> 16, acc);
#else
          const float2 pf = __half22float2(*reinterpret_cast<const __half2*>(&pv[w]));
          const float2 xf = __half22float2(*reinterpret_cast<const __half2*>(&xv[w]));
          if (k < d) acc = __fmaf_rn(xf.x, pf.x, acc);
          if (k + 1 < d) acc = __fmaf_rn(xf.y, pf.y, acc);
#endif
        }
      }
      if (d % 32 != 0) acc = __fmaf_rn(0.0f, 0.0f, acc);
    }
    const __half h = __float2half_rn(acc);
    y[i] = i < d ? *reinterpret_cast<const uint16_t*>(&h) : uint16_t(0);
  }
}

// One 16-byte chunk (8 halves) of the L2 sum, element order 0..7, each term
// fused as fma(d, d, acc): the reference's per-lane accumulation
// (include/jasper/distance/distance.cuh:131-141).
__device__ __forceinline__ float l2_chunk(uint4 a, uint4 b, float acc) {
  const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
  const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
  for (int w = 0; w < 4; w++) {
    __half2 hb = *reinterpret_cast<const __half2*>(&bw[w]);
    float2 fb = __half22float2(hb);
#if JB_MIXED_ADD
    float d0 = sub_f32_f16(aw[w], fb.x);
    acc = __fmaf_rn(d0, d0, acc);
    float d1 = sub_f32_f16(aw[w] >> 16, fb.y);
    acc = __fmaf_rn(d1, d1, acc);
#else
    __half2 ha = *reinterpret_cast<const __half2*>(&aw[w]);
    float2 fa = __half22float2(ha);
    float d0 = __fsub_rn(fa.x, fb.x);
    acc = __fmaf_rn(d0, d0, acc);
    float d1 = __fsub_rn(fa.y, fb.y);
    acc = __fmaf_rn(d1, d1, acc);
#endif
  }
  return acc;
}

// The two elements (s, s+4) of one chunk that lane s of a 4-lane tile owns
// in the reference's inner-product walk (distance.cuh:95-106: element i goes
// to lane i % 4, in increasing i).
__device__ __forceinline__ float ip_pair(uint32_t qlo, uint32_t qhi, uint32_t rlo,
                                         uint32_t rhi, int s, float acc) {
  const int sh = (s & 1) * 16;
#if JB_MIXED_ADD
  acc = fma_f32_f16(qlo >> sh, rlo >> sh, acc);
  acc = fma_f32_f16(qhi >> sh, rhi >> sh, acc);
#else
  float q0 = __half2float(__ushort_as_half((unsigned short)(qlo >> sh)));
  float r0 = __half2float(__ushort_as_half((unsigned short)(rlo >> sh)));
  acc = __fmaf_rn(q0, r0, acc);
  float q1 = __half2float(__ushort_as_half((unsigned short)(qhi >> sh)));
  float r1 = __half2float(__ushort_as_half((unsigned short)(rhi >> sh)));
  acc = __fmaf_rn(q1, r1, acc);
#endif
  return acc;
}

// Butterfly over a 4-lane tile, identical to cg::reduce(tile, x, plus):
// mask 2 then mask 1, each step out = out + partner
// (cooperative_groups/details/coalesced_reduce.h).
__device__ __forceinline__ float tile4_sum(float x) {
  x = __fadd_rn(x, __shfl_xor_sync(kFull, x, 2));
  x = __fadd_rn(x, __shfl_xor_sync(kFull, x, 1));
  return x;
}

// Same reduction when the tiles of a warp may be on different paths: only
// the 4 lanes of the calling tile synchronise.
__device__ __forceinline__ float tile4_sum_local(float x, int lane) {
  const uint32_t mask = 0xFu << (lane & ~3);
  x = __fadd_rn(x, __shfl_xor_sync(mask, x, 2));
  x = __fadd_rn(x, __shfl_xor_sync(mask, x, 1));
  return x;
}

// Warp-wide bitonic sort of 64 keys held two per lane (element p = r*32+lane).
__device__ __forceinline__ void warp_sort64(uint64_t& v0, uint64_t& v1, int lane) {
#pragma unroll
  for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j == 32) {
        uint64_t lo = v0 < v1 ? v0 : v1, hi = v0 < v1 ? v1 : v0;
        v0 = lo; v1 = hi;
      } else {
#pragma unroll
        for (int r = 0; r < 2; r++) {
          uint64_t& v = r ? v1 : v0;
          const int p = r * 32 + lane;
          uint64_t o = __shfl_xor_sync(kFull, v, j);
          const bool up = (p & k) == 0;
          const bool low = (lane & j) == 0;
          const bool take_min = (low == up);
          v = take_min ? (v < o ? v : o) : (v < o ? o : v);
        }
      }
    }
  }
}

// Warp-wide bitonic sort of 32 keys, one per lane (ascending by lane).
__device__ __forceinline__ uint64_t warp_sort32(uint64_t v, int lane) {
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      uint64_t o = __shfl_xor_sync(kFull, v, j);
      const bool up = (lane & k) == 0;
      const bool low = (lane & j) == 0;
      v = (low == up) ? (v < o ? v : o) : (v < o ? o : v);
    }
  }
  return v;
}

// Bitonic sort of n (power of two, <= 32 * 32) keys in shared memory by one warp.
__device__ __forceinline__ void warp_sort_smem(uint64_t* a, int n, int lane) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = lane; i < n; i += 32) {
        int p = i ^ j;
        if (p > i) {
          uint64_t x = a[i], y = a[p];
          bool up = (i & k) == 0;
          if ((x > y) == up) { a[i] = y; a[p] = x; }
        }
      }
      __syncwarp();
    }
  }
}

// Number of elements of sorted a[0, n) strictly below x.
__device__ __forceinline__ int lower_rank(const uint64_t* a, int n, uint64_t x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (a[mid] < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(uint32_t(b) << 16);
}
__device__ __forceinline__ uint16_t float_to_bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

}  // namespace jb
