// Test infrastructure only: runs the reference's own RaBitQ quantizer
// (rabitq_quantize<1>, include/jasper/rabitq/quantize.cuh:296-353) on rows
// read from a file and writes the reference's node store back, so the
// restatement (oracle/jasper_oracle.c) and the device quantizer can be
// checked against it.  Built by oracle/build_ref.sh into oracle/_ref/bin/.
//
// Input file:  u32 n, u32 dim, u32 metric (0 L2, 1 IP), u32 has_rotation,
//              f32 rows[n][dim], f32 centroid[dim],
//              f32 rotation[dim][dim] (column-major) if has_rotation, else identity.
// Output file: the store, n x node_bytes bytes (code bits, f_add, f_rescale).
#include <algorithm>
#include <array>
#include <cstdio>
#include <cstdlib>
#include <vector>
#include "jasper/rabitq/quantize.cuh"

int main(int argc, char** argv) {
  if (argc != 3) {
    std::fprintf(stderr, "usage: %s IN OUT\n", argv[0]);
    return 2;
  }
  FILE* f = std::fopen(argv[1], "rb");
  if (!f) return 3;
  uint32_t hdr[4];
  if (std::fread(hdr, 4, 4, f) != 4) return 4;
  const uint32_t n = hdr[0], dim = hdr[1], metric = hdr[2], has_rot = hdr[3];
  std::vector<float> rows(size_t(n) * dim), cent(dim), rot(size_t(dim) * dim, 0.0f);
  if (std::fread(rows.data(), 4, rows.size(), f) != rows.size()) return 5;
  if (std::fread(cent.data(), 4, cent.size(), f) != cent.size()) return 6;
  if (has_rot) {
    if (std::fread(rot.data(), 4, rot.size(), f) != rot.size()) return 7;
  } else {
    for (uint32_t i = 0; i < dim; i++) rot[i + size_t(i) * dim] = 1.0f;
  }
  std::fclose(f);
  float *d_rows, *d_cent, *d_rot;
  cudaMalloc(&d_rows, rows.size() * 4);
  cudaMalloc(&d_cent, cent.size() * 4);
  cudaMalloc(&d_rot, rot.size() * 4);
  cudaMemcpy(d_rows, rows.data(), rows.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(d_cent, cent.data(), cent.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(d_rot, rot.data(), rot.size() * 4, cudaMemcpyHostToDevice);
  jasper::vector_view<float> view(d_rows, dim, n, false);
  auto store = jasper::rabitq_quantize<1>(view, d_rot, d_cent,
                                          metric ? jasper::METRIC_IP : jasper::METRIC_L2);
  // a rejected launch (e.g. too much dynamic shared memory) is not reported
  // by the synchronisation inside rabitq_quantize: check it here
  const cudaError_t le = cudaGetLastError();
  if (le != cudaSuccess) {
    std::fprintf(stderr, "quantize launch failed: %s\n", cudaGetErrorString(le));
    return 10;
  }
  std::vector<char> out(store.total_bytes());
  cudaMemcpy(out.data(), store.data, out.size(), cudaMemcpyDeviceToHost);
  const cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    std::fprintf(stderr, "cuda error %s\n", cudaGetErrorString(e));
    return 8;
  }
  FILE* o = std::fopen(argv[2], "wb");
  if (!o) return 9;
  std::fwrite(out.data(), 1, out.size(), o);
  std::fclose(o);
  return 0;
}
