// rotate_tc.cu -- prerotation GEMM on the tensor cores (tcgen05, sm_100a).
//
// Y[r][i] = sum_k X[r][k] * M[i][k] for every row r, where X holds the rows
// (fp16, stride dpad, pad lanes zero) and M is the rotation padded to
// dpad x dpad (row i = output coordinate i, K-contiguous, zeros outside
// d x d).  This is the reference's cublasGemmEx(OP_T, OP_N) with fp16 I/O and
// fp32 accumulation (index/construct.cuh:1077-1089, rotation.cuh:122-151);
// the summation order is the tensor core's, so outputs can differ from cuBLAS
// in the last fp16 bit.
//
// Persistent: one CTA per SM walks 128-row x BN-column output tiles (roles
// at rotate_tc_kernel).  TMA brings 64-wide K slices of X and M into a ring
// of SWIZZLE_128B stages (cp.async.bulk.tensor, each CTA its own tiles); one thread
// issues tcgen05.mma kind::f16 (K = 16 each) into one of two fp32 TMEM
// accumulators; four epilogue warps drain the other accumulator with
// tcgen05.ld (TMEM lane = output row), round to fp16, stage 32-row x
// 16-column boxes in shared memory and store them with TMA bulk tensor
// stores, so a tile's epilogue overlaps the next tile's loads and MMAs.
// Every mbarrier wait is bounded: on timeout the CTA records an error code,
// waits (bounded) for its own bulk copies and MMAs, frees its TMEM and
// returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <map>
#include <mutex>
#include <stdexcept>
#include <utility>
#include <string>
#include "rotate.cuh"

namespace jb {
namespace {

constexpr int kBM = 128;          // output rows per CTA (TMEM lanes)
constexpr int kBK = 64;           // K slice per stage: 64 fp16 = one 128-byte swizzle row
constexpr uint64_t kWaitNs = 2000000000ull;  // bound on any single wait

__device__ unsigned int g_tc_rotate_error;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity.  Bounded: gives up (false) after
// about two seconds, or as soon as another CTA has recorded an error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t it = 0;; it++) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 1023) == 0) {
      const uint64_t now = global_ns();
      if (it == 0) t0 = now;
      else if (now - t0 > kWaitNs || *reinterpret_cast<volatile unsigned int*>(&g_tc_rotate_error))
        return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// K-major SWIZZLE_128B operand: rows of 128 bytes, 8-row groups 1024 bytes
// apart (SBO), version 1, layout type 2; LBO is unused for this layout (1).
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
  const uint64_t addr = smem_u32(p);
  return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 accumulator, fp16 A and B, both
// K-major, M = 128, N = bn.
__host__ __device__ constexpr uint32_t f16_idesc(uint32_t bn) {
  return (1u << 4) | ((bn >> 3) << 17) | ((uint32_t(kBM) >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Persistent kernel: one CTA of 192 threads per SM walks the output tiles
// t = blockIdx.x, blockIdx.x + gridDim.x, ... (tile t = row tile t / ncol,
// column tile t % ncol, so consecutive tiles reuse the same rows from L2).
//   warp 0, lane 0  TMA producer: the K slices of every tile, back to back,
//                   into a ring of `stages` SWIZZLE_128B stages;
//   warp 1, lane 0  MMA issuer: a tile's slices accumulate into one of two
//                   TMEM accumulators (tiles alternate), tcgen05.commit frees
//                   each stage and finally marks the accumulator full;
//   warps 2..5      epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (its
//                   rows of the tile), rounds to fp16 into its staging boxes,
//                   hands the accumulator back and issues the boxes' TMA
//                   stores; meanwhile the MMA fills the other accumulator.
// bn: output columns per tile (multiple of 16, <= 256); tmem_cols: power of
// two >= bn (columns per accumulator; two are allocated).
constexpr int kThreads = 192;

__global__ void __launch_bounds__(kThreads, 1)
    rotate_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_m,
                     const __grid_constant__ CUtensorMap map_y, uint32_t n, uint32_t dpad, uint32_t bn,
                     uint32_t tmem_cols, uint32_t stages, uint32_t ksteps, uint32_t ncol,
                     uint32_t ntiles) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte aligned stage ring: A slices [stages][128 x 128 B], then B
  // slices [stages][bn x 128 B]; barriers and the TMEM address after them.
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t a_bytes = kBM * 128, b_bytes = bn * 128;
  unsigned char* a_ring = base;
  unsigned char* b_ring = base + size_t(stages) * a_bytes;
  // epilogue staging: per epilogue warp, bn / 16 boxes of 32 rows x 16 columns
  unsigned char* y_stage = b_ring + size_t(stages) * b_bytes;
  const uint32_t y_warp_bytes = bn * 64;
  uint64_t* full = reinterpret_cast<uint64_t*>(y_stage + size_t(4) * y_warp_bytes);
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;  // [2] MMA -> epilogue
  uint64_t* acc_free = acc_full + 2;    // [2] epilogue -> MMA (4 warp arrivals)
  uint64_t* done = acc_free + 2;        // every MMA of this CTA completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __shared__ volatile uint32_t s_fail;
  if (tid == 0) {
    // a CTA that starts after another one failed does nothing
    s_fail = *reinterpret_cast<volatile unsigned int*>(&g_tc_rotate_error) ? 1u : 0u;
    for (uint32_t s = 0; s < stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_free[b], 4);
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (s_fail) return;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(2 * tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // producer
      uint32_t issued = 0;
      bool ok = true;
      for (uint32_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int row0 = int((t / ncol) * kBM), col0 = int((t % ncol) * bn);
        for (uint32_t k = 0; k < ksteps; k++, issued++) {
          const uint32_t s = issued % stages;
          if (issued >= stages && !mbar_wait(&empty[s], ((issued / stages) - 1) & 1)) {
            atomicExch(&g_tc_rotate_error, 1u);
            s_fail = 1;
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], a_bytes + b_bytes);
          tma_load_2d(a_ring + size_t(s) * a_bytes, &map_x, &full[s], int(k * kBK), row0);
          tma_load_2d(b_ring + size_t(s) * b_bytes, &map_m, &full[s], int(k * kBK), col0);
        }
      }
      // drain: every issued copy has landed before the CTA can leave
      for (uint32_t k = (issued > stages ? issued - stages : 0); k < issued; k++)
        if (!mbar_wait(&full[k % stages], (k / stages) & 1)) atomicExch(&g_tc_rotate_error, 2u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer
      const uint32_t idesc = f16_idesc(bn);
      uint32_t consumed = 0, it = 0;
      bool ok = true;
      for (uint32_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, it++) {
        const uint32_t b = it & 1;
        // the epilogue has read this accumulator's previous tile
        if (it >= 2 && (s_fail || !mbar_wait(&acc_free[b], ((it >> 1) - 1) & 1))) {
          atomicExch(&g_tc_rotate_error, 5u);
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem + b * tmem_cols;
        for (uint32_t k = 0; k < ksteps; k++, consumed++) {
          const uint32_t s = consumed % stages;
          if (!mbar_wait(&full[s], (consumed / stages) & 1)) {
            atomicExch(&g_tc_rotate_error, 3u);
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t ad = sw128_desc(a_ring + size_t(s) * a_bytes);
          const uint64_t bd = sw128_desc(b_ring + size_t(s) * b_bytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; kk++)  // 32 bytes of K per MMA: +2 in the address field
            mma_f16(acc, ad + 2ull * kk, bd + 2ull * kk, idesc, (k | kk) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[b]);
      }
      if (!ok) s_fail = 1;
      mma_commit(done);  // arrives once every MMA issued above has completed
      if (!mbar_wait(done, 0)) atomicExch(&g_tc_rotate_error, 6u);
    }
  } else {
    // epilogue: TMEM lane quadrant of this warp = its rows within the tile
    const uint32_t quad = uint32_t(warp & 3);
    const uint32_t lane_base = (quad * 32) << 16;
    uint32_t it = 0;
    for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x, it++) {
      const uint32_t b = it & 1;
      // warp-uniform wait (tcgen05.ld below is warp-collective)
      int ok = 1;
      if (lane == 0) ok = !s_fail && mbar_wait(&acc_full[b], (it >> 1) & 1);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) atomicExch(&g_tc_rotate_error, 4u);
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int y0 = int((t / ncol) * kBM + quad * 32);
      const int x0 = int((t % ncol) * bn);
      unsigned char* stage_w = y_stage + size_t(warp - 2) * y_warp_bytes;
      // the previous tile's stores have finished reading this warp's staging
      if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      __syncwarp();
      for (uint32_t c = 0; c < bn; c += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + lane_base + b * tmem_cols + c, v);
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const __half2 h2 = __floats2half2_rn(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
          w[j] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        // box c / 16: 32 rows x 16 columns, row `lane` at byte 32 * lane
        uint4* d4 = reinterpret_cast<uint4*>(stage_w + (c / 16) * 1024 + lane * 32);
        d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
        d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
      }
      // TMEM reads done: hand the accumulator back before the stores
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acc_free[b])) : "memory");
        // rows past n and columns past dpad are clipped by the tensor map;
        // x is a multiple of 16 elements (32 bytes), never negative
        for (uint32_t c = 0; c < bn && x0 + int(c) < int(dpad) && y0 < int(n); c += 16)
          asm volatile(
              "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                  reinterpret_cast<uint64_t>(&map_y)),
              "r"(x0 + int(c)), "r"(y0), "r"(smem_u32(stage_w + (c / 16) * 1024))
              : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      }
    }
    // every store of this warp has completed before the CTA leaves
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(2 * tmem_cols)
                 : "memory");
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled is not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D fp16 map over rows x cols (row stride `stride` elements), box of
// box_rows x 64 with 128-byte swizzle; out-of-range elements read as zero.
// box_cols = 64 with the 128-byte swizzle for the operand loads; the output
// map uses unswizzled 16-column boxes.
CUtensorMap make_map(const void* ptr, uint64_t rows, uint64_t cols, uint64_t stride,
                     uint32_t box_rows, uint32_t box_cols = kBK,
                     CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {stride * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr),
                                 dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return m;
}

}  // namespace

void rotate_rows_tc(const uint16_t* Mp, uint32_t dpad, const uint16_t* X, uint16_t* Y, uint64_t n,
                    cudaStream_t st) {
  if (n == 0) return;
  if (dpad % 8 != 0 || dpad == 0) throw std::invalid_argument("rotate: dpad must be a multiple of 8");
  if (n >= (uint64_t(1) << 31)) throw std::invalid_argument("rotate: too many rows");
  if ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(Y) |
       reinterpret_cast<uintptr_t>(Mp)) % 16)
    throw std::invalid_argument("rotate: buffers must be 16-byte aligned");
  // N tiles of at most 256 columns (multiple of 16)
  const uint32_t nsplit = (dpad + 255) / 256;
  uint32_t bn = (dpad + nsplit - 1) / nsplit;
  bn = (bn + 15) / 16 * 16;
  uint32_t tmem_cols = 32;
  while (tmem_cols < bn) tmem_cols <<= 1;
  const uint32_t ksteps = (dpad + kBK - 1) / kBK;
  const size_t stage_bytes = size_t(kBM) * 128 + size_t(bn) * 128;
  // ring depth: up to 6 stages in one CTA's shared memory (one CTA per SM)
  const size_t ystage_bytes = size_t(4) * bn * 64;  // epilogue staging, 4 warps
  uint32_t stages = 6;
  while (stages > 2 && stages * stage_bytes + ystage_bytes + 2048 > 220 * 1024) stages--;
  const size_t smem =
      stages * stage_bytes + ystage_bytes + 1024 /* alignment */ + 8 * (2 * stages + 5) + 16;
  const CUtensorMap mx = make_map(X, n, dpad, dpad, kBM);
  const CUtensorMap mm = make_map(Mp, dpad, dpad, dpad, bn);
  const CUtensorMap my = make_map(Y, n, dpad, dpad, 32, 16, CU_TENSOR_MAP_SWIZZLE_NONE);
  int dev = 0;
  cudaGetDevice(&dev);
  // per device: the SM count, and the largest shared-memory opt-in made so far
  static std::mutex mu;
  static std::map<int, std::pair<int, size_t>> dev_state;
  int sms = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto& st_dev = dev_state[dev];
    if (st_dev.first == 0) cudaDeviceGetAttribute(&st_dev.first, cudaDevAttrMultiProcessorCount, dev);
    if (smem > st_dev.second) {
      cudaFuncSetAttribute(rotate_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      st_dev.second = smem;
    }
    sms = st_dev.first;
  }
  const uint32_t ncol = (dpad + bn - 1) / bn;
  const uint64_t ntiles64 = ((n + kBM - 1) / kBM) * uint64_t(ncol);
  if (ntiles64 >= (uint64_t(1) << 31)) throw std::invalid_argument("rotate: too many tiles");
  const uint32_t ntiles = uint32_t(ntiles64);
  const uint32_t grid = ntiles < uint32_t(sms > 0 ? sms : 1) ? ntiles : uint32_t(sms);
  rotate_tc_kernel<<<grid, kThreads, smem, st>>>(mx, mm, my, uint32_t(n), dpad, bn, tmem_cols,
                                                 stages, ksteps, ncol, ntiles);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("rotate launch: ") + cudaGetErrorString(e));
}

int rotate_tc_error(bool reset) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_rotate_error, sizeof(v));
  if (reset) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_tc_rotate_error, &z, sizeof(z));
  }
  return int(v);
}

}  // namespace jb
