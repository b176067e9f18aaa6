// noalloc.cu -- a search entry point that performs no device allocation.
//
// jb_graph_search takes its per-call device scratch -- the 256-byte work
// counter that hands queries to warps, and a repacked copy of the queries
// when their rows are not 16-byte aligned at the padded stride -- from the
// stream-ordered allocator.  Some callers cannot let a search allocate: code
// that runs under a fixed, pre-reserved device-memory budget, a process whose
// own allocator owns every byte and must not be bypassed, or code that may
// not touch the CUDA allocator while other GPU work is in flight.
// jb_graph_search_noalloc runs the same search kernel with that scratch in the
// fixed device array below, which every GPU that loads this library holds
// until the process exits.
//
// Limits and behaviour:
//  * the array is kNoAllocScratchBytes = 4 MiB: 256 bytes for the work
//    counter, the rest for repacked queries; a call whose queries need
//    repacking (row stride != padded dim, or a base address that is not
//    16-byte aligned) is rejected when n_queries * padded_dim * 2 bytes do not
//    fit in the remainder; queries already at the padded stride have no limit;
//  * every call on a device shares the one array and leaves its contents
//    behind; the counter is cleared at the start of each call, in stream
//    order, so calls that overlap on the GPU (other streams, other threads)
//    race and must be serialised by the caller;
//  * the array's device address is looked up once per device, on the first
//    call made with that device's graph (cudaGetSymbolAddress with that
//    device current); make that first call before any stream capture begins.
#include <cuda_runtime.h>

#include <functional>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>

#include "../../include/jasper_b200.h"
#include "jb_graph.h"
#include "search.cuh"

namespace jb {
std::shared_ptr<Graph> capi_lookup(int64_t h);
int capi_guarded(const std::function<void()>& f);
}  // namespace jb

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
constexpr size_t kCounterBytes = 256;
static_assert(jb::kSearchScratchBytes <= kCounterBytes, "counter region too small");

// In host code this name is only a stand-in; kernels get the address from
// scratch_for_current_device().
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
unsigned char* g_scratch_ptr[kMaxDevices] = {};

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
  }
}

// Device address of the scratch array on the current device (set up once).
unsigned char* scratch_for_current_device() {
  int dev = 0;
  check(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) throw std::runtime_error("device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)");
    g_scratch_ptr[dev] = static_cast<unsigned char*>(p);
  }
  return g_scratch_ptr[dev];
}

struct RestoreDevice {
  int dev = -1;
  ~RestoreDevice() {
    if (dev >= 0) cudaSetDevice(dev);
  }
};

}  // namespace

extern "C" int jb_graph_search_noalloc(int64_t handle, const uint16_t* queries, uint64_t n_queries,
                                       uint32_t row_stride, int32_t* out_idx, float* out_dist,
                                       uint32_t k, uint32_t beam_width, uint32_t limit,
                                       void* stream) {
  return jb::capi_guarded([&] {
    auto g = jb::capi_lookup(handle);
    RestoreDevice restore;
    int prev = -1;
    check(cudaGetDevice(&prev), "cudaGetDevice");
    if (prev != g->device) {
      check(cudaSetDevice(g->device), "cudaSetDevice");
      restore.dev = prev;
    }
    if (n_queries == 0) return;
    if (n_queries > 0x7FFFFFFFull) throw std::invalid_argument("too many queries");
    if (k == 0) throw std::invalid_argument("k must be > 0");
    if (row_stride < g->dim) throw std::invalid_argument("row_stride < dim");
    if (!queries || !out_idx || !out_dist) throw std::invalid_argument("null pointer argument");
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    const uint16_t* q = queries;
    const bool aligned = (reinterpret_cast<uintptr_t>(queries) % 16) == 0;
    const bool repack = row_stride != g->dpad || !aligned;
    const size_t need = repack ? size_t(n_queries) * g->dpad * 2 : 0;
    if (need > kNoAllocScratchBytes - kCounterBytes)
      throw std::invalid_argument(
          "jb_graph_search_noalloc: these queries must be repacked to the padded stride and "
          "need " + std::to_string(need) + " bytes of scratch, more than the fixed " +
          std::to_string(kNoAllocScratchBytes - kCounterBytes) +
          "; pass rows at stride ceil(dim/8)*8 from a 16-byte aligned base, or fewer queries");
    unsigned char* scratch = scratch_for_current_device();
    if (repack) {
      uint16_t* packed = reinterpret_cast<uint16_t*>(scratch + kCounterBytes);
      check(cudaMemsetAsync(packed, 0, need, st), "clear repacked queries");
      check(cudaMemcpy2DAsync(packed, size_t(g->dpad) * 2, queries, size_t(row_stride) * 2,
                              size_t(g->dim) * 2, n_queries, cudaMemcpyDefault, st),
            "repack queries");
      q = packed;
    }
    check(cudaMemsetAsync(scratch, 0, kCounterBytes, st), "clear work counter");
    jb::SearchArgs a{};
    a.g = g->view();
    a.queries = q;
    a.nq = uint32_t(n_queries);
    a.k = k;
    a.bw = beam_width;
    a.limit = limit;
    a.max_result_size = 2048;  // same as jb_graph_search
    a.out_idx = out_idx;
    a.out_dist = out_dist;
    a.work_counter = reinterpret_cast<uint32_t*>(scratch);
    jb::launch_search(a, st);
  });
}
