// graph.cu -- allocation, upload and the on-disk format of a jasper_b200 graph.
//
// The file format is the reference's, byte for byte
// (include/jasper/index/graph.cuh:1653-1788, save_graph_to_file):
//   [u64 total_file_size][u64 n][u64 medoid][u64 bytes_per_node]
//   n records of: dim x fp16 (unpadded) | u8 edge_count |
//                 R x u32 ids | R x bf16 distances | u32 slot_to_id
//   ceil(n / 8) bytes of deletion bitmask (bit i = slot i), then u64 next_id.
// The loader also accepts the three older record layouts the reference
// reader detects by bytes_per_node (graph.cuh:1460-1479): legacy (no id, no
// deletion), +deleted byte, +deleted byte +id.  Unlike the reference, a bad
// path or a short file raises instead of calling exit().
#include <cuda_runtime.h>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <stdexcept>
#include <vector>
#include "jb_graph.h"

namespace jb {
namespace {

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
  }
}

template <typename T>
T* alloc_array(size_t count, bool on_host, const char* what) {
  void* p = nullptr;
  size_t bytes = count * sizeof(T);
  if (bytes == 0) bytes = 16;
  if (on_host) check(cudaHostAlloc(&p, bytes, cudaHostAllocMapped | cudaHostAllocPortable), what);
  else check(cudaMalloc(&p, bytes), what);
  return static_cast<T*>(p);
}

void free_array(void* p, bool on_host) {
  if (!p) return;
  if (on_host) cudaFreeHost(p); else cudaFree(p);
}

void copy_to(void* dst, const void* src, size_t bytes) {
  check(cudaMemcpy(dst, src, bytes, cudaMemcpyDefault), "graph copy");
}

}  // namespace

void graph_allocate(Graph& g, uint32_t dim, uint32_t R, int metric, uint32_t n, bool on_host) {
  if (dim == 0) throw std::invalid_argument("dim must be > 0");
  if (R == 0 || R > 64) throw std::invalid_argument("n_neighbors must be in [1, 64]");
  if (n >= 0x7FFFFFFFu) throw std::invalid_argument("graphs are limited to 2^31 - 1 rows");
  g = Graph{};
  check(cudaGetDevice(&g.device), "cudaGetDevice");
  g.dim = dim;
  g.dpad = pad_dim(dim);
  g.R = R;
  g.metric = metric;
  g.n = n;
  g.capacity = n;
  g.on_host = on_host;
  g.next_id = n;
  try {
    g.vec = alloc_array<uint16_t>(size_t(n) * g.dpad, on_host, "alloc vectors");
    g.edges = alloc_array<uint32_t>(size_t(n) * R, on_host, "alloc edges");
    g.edist = alloc_array<uint16_t>(size_t(n) * R, on_host, "alloc edge distances");
    g.counts = alloc_array<uint8_t>(n, on_host, "alloc edge counts");
    g.slot_to_id = alloc_array<uint32_t>(n, on_host, "alloc slot ids");
    g.deleted = alloc_array<uint32_t>((size_t(n) + 31) / 32, on_host, "alloc deletion bits");
    if (on_host) {
      memset(g.edges, 0xFF, size_t(n) * R * 4);
      memset(g.edist, 0, size_t(n) * R * 2);
      memset(g.counts, 0, n);
      memset(g.deleted, 0, ((size_t(n) + 31) / 32) * 4);
    } else {
      check(cudaMemset(g.edges, 0xFF, size_t(n) * R * 4), "memset edges");
      check(cudaMemset(g.edist, 0, size_t(n) * R * 2), "memset dists");
      check(cudaMemset(g.counts, 0, n), "memset counts");
      check(cudaMemset(g.deleted, 0, ((size_t(n) + 31) / 32) * 4), "memset deleted");
    }
  } catch (...) {
    graph_free(g);
    throw;
  }
}

void graph_reserve(Graph& g, uint32_t rows) {
  if (rows <= g.capacity) return;
  if (g.on_host) throw std::runtime_error("graph_reserve: graph rows live in host memory");
  if (rows >= 0x7FFFFFFFu) throw std::invalid_argument("graphs are limited to 2^31 - 1 rows");
  const size_t n = g.n, R = g.R, dp = g.dpad;
  const size_t wn = (n + 31) / 32, wc = (size_t(rows) + 31) / 32;
  uint16_t* vec = nullptr; uint32_t* edges = nullptr; uint16_t* edist = nullptr;
  uint8_t* counts = nullptr; uint32_t* ids = nullptr; uint32_t* del = nullptr;
  try {
    vec = alloc_array<uint16_t>(size_t(rows) * dp, false, "grow vectors");
    edges = alloc_array<uint32_t>(size_t(rows) * R, false, "grow edges");
    edist = alloc_array<uint16_t>(size_t(rows) * R, false, "grow edge distances");
    counts = alloc_array<uint8_t>(rows, false, "grow edge counts");
    ids = alloc_array<uint32_t>(rows, false, "grow slot ids");
    del = alloc_array<uint32_t>(wc, false, "grow deletion bits");
    check(cudaMemcpy(vec, g.vec, n * dp * 2, cudaMemcpyDeviceToDevice), "grow copy");
    check(cudaMemcpy(edges, g.edges, n * R * 4, cudaMemcpyDeviceToDevice), "grow copy");
    check(cudaMemset(edges + n * R, 0xFF, (rows - n) * R * 4), "grow memset");
    check(cudaMemcpy(edist, g.edist, n * R * 2, cudaMemcpyDeviceToDevice), "grow copy");
    check(cudaMemset(edist + n * R, 0, (rows - n) * R * 2), "grow memset");
    check(cudaMemcpy(counts, g.counts, n, cudaMemcpyDeviceToDevice), "grow copy");
    check(cudaMemset(counts + n, 0, rows - n), "grow memset");
    check(cudaMemcpy(ids, g.slot_to_id, n * 4, cudaMemcpyDeviceToDevice), "grow copy");
    check(cudaMemset(del, 0, wc * 4), "grow memset");
    check(cudaMemcpy(del, g.deleted, wn * 4, cudaMemcpyDeviceToDevice), "grow copy");
  } catch (...) {
    for (void* p : {static_cast<void*>(vec), static_cast<void*>(edges), static_cast<void*>(edist),
                    static_cast<void*>(counts), static_cast<void*>(ids), static_cast<void*>(del)})
      free_array(p, false);
    throw;
  }
  if (g.eflag) {  // prune flags: the first n rows kept, the new ones zero
    uint64_t* f = nullptr;
    try {
      f = alloc_array<uint64_t>(rows, false, "grow prune flags");
      check(cudaMemcpy(f, g.eflag, n * 8, cudaMemcpyDeviceToDevice), "grow copy");
      check(cudaMemset(f + n, 0, (rows - n) * 8), "grow memset");
    } catch (...) {
      free_array(f, false);
      for (void* p : {static_cast<void*>(vec), static_cast<void*>(edges), static_cast<void*>(edist),
                      static_cast<void*>(counts), static_cast<void*>(ids), static_cast<void*>(del)})
        free_array(p, false);
      throw;
    }
    cudaFree(g.eflag);
    g.eflag = f;
  }
  free_array(g.vec, false); free_array(g.edges, false); free_array(g.edist, false);
  free_array(g.counts, false); free_array(g.slot_to_id, false); free_array(g.deleted, false);
  g.vec = vec; g.edges = edges; g.edist = edist; g.counts = counts; g.slot_to_id = ids;
  g.deleted = del;
  g.capacity = rows;
}

void graph_free_directional(Graph& g) {
  DirArtifacts& d = g.dir;
  if (d.lsh_packed) cudaFree(d.lsh_packed);
  if (d.lsh_mag) cudaFree(d.lsh_mag);
  if (d.pq_centroids) cudaFree(d.pq_centroids);
  if (d.pq_codes) cudaFree(d.pq_codes);
  if (d.norms) cudaFree(d.norms);
  if (d.rotation) cudaFree(d.rotation);
  if (d.rotation_pad) cudaFree(d.rotation_pad);
  if (d.rq_store) cudaFree(d.rq_store);
  if (d.rq_centroid) cudaFree(d.rq_centroid);
  if (d.rq_err) cudaFree(d.rq_err);
  d = DirArtifacts{};
}

void graph_free(Graph& g) {
  graph_free_directional(g);
  free_array(g.vec, g.on_host);
  free_array(g.edges, g.on_host);
  free_array(g.edist, g.on_host);
  free_array(g.counts, g.on_host);
  free_array(g.slot_to_id, g.on_host);
  free_array(g.deleted, g.on_host);
  if (g.eflag) cudaFree(g.eflag);
  g.eflag = nullptr;
  g.vec = nullptr; g.edges = nullptr; g.edist = nullptr; g.counts = nullptr;
  g.slot_to_id = nullptr; g.deleted = nullptr;
  g.n = 0;
  g.capacity = 0;
}

void graph_upload_rows(Graph& g, const uint16_t* rows, uint32_t stride) {
  const size_t n = g.n;
  if (n == 0) return;
  // Padded row array: one 2-D copy puts each dim-element row at stride dpad;
  // the pad lanes are zeroed first so padded distances stay exact.
  if (g.dpad != g.dim) {
    if (g.on_host) memset(g.vec, 0, n * g.dpad * 2);
    else check(cudaMemset(g.vec, 0, n * g.dpad * 2), "memset pad");
  }
  check(cudaMemcpy2D(g.vec, size_t(g.dpad) * 2, rows, size_t(stride) * 2, size_t(g.dim) * 2, n,
                     cudaMemcpyDefault),
        "upload rows");
  std::vector<uint32_t> ids(n);
  for (size_t i = 0; i < n; i++) ids[i] = uint32_t(i);
  copy_to(g.slot_to_id, ids.data(), n * 4);
  g.ids_identity = true;
}

void graph_load_file(Graph& g, const std::string& path, uint32_t dim, uint32_t R, int metric,
                     bool on_host) {
  std::ifstream f(path, std::ios::binary);
  if (!f.is_open()) throw std::runtime_error("Failed to open " + path + " for graph load");
  uint64_t hdr[4];
  f.read(reinterpret_cast<char*>(hdr), sizeof(hdr));
  if (f.gcount() != sizeof(hdr)) throw std::runtime_error("graph file too short: " + path);
  const uint64_t n = hdr[1], medoid = hdr[2], bpn = hdr[3];
  const uint64_t base = 2ull * dim + 1 + 6ull * R;
  const bool bitpacked = bpn == base + 4;
  const bool inline_del = bpn == base + 1 || bpn == base + 5;
  const bool has_id = bpn == base + 5 || bitpacked;
  if (!(bpn == base || bitpacked || inline_del))
    throw std::runtime_error("graph file " + path + ": bytes_per_node " + std::to_string(bpn) +
                             " does not match dim=" + std::to_string(dim) +
                             " n_neighbors=" + std::to_string(R));
  if (n >= 0x7FFFFFFFull) throw std::runtime_error("graph file has too many rows");
  if (n > 0 && medoid >= n)
    throw std::runtime_error("graph file " + path + ": medoid " + std::to_string(medoid) +
                             " is not a row of the file (n=" + std::to_string(n) + ")");
  graph_allocate(g, dim, R, metric, uint32_t(n), on_host);
  g.medoid = uint32_t(medoid);
  try {
    const uint32_t dpad = g.dpad;
    const size_t chunk = size_t(1) << 18;
    std::vector<char> raw(chunk * bpn);
    std::vector<uint16_t> hv(chunk * dpad);
    std::vector<uint32_t> he(chunk * R), hid(chunk);
    std::vector<uint16_t> hd(chunk * R);
    std::vector<uint8_t> hc(chunk);
    std::vector<uint8_t> del_bits((n + 7) / 8, 0);
    bool identity = true;
    for (uint64_t start = 0; start < n; start += chunk) {
      const size_t cnt = size_t(std::min<uint64_t>(chunk, n - start));
      f.read(raw.data(), std::streamsize(cnt * bpn));
      if (size_t(f.gcount()) != cnt * bpn)
        throw std::runtime_error("Short read in graph file " + path);
      std::fill(hv.begin(), hv.begin() + cnt * dpad, 0);
      for (size_t i = 0; i < cnt; i++) {
        const char* p = raw.data() + i * bpn;
        memcpy(&hv[i * dpad], p, 2ull * dim);
        p += 2ull * dim;
        hc[i] = uint8_t(*p);
        p += 1;
        memcpy(&he[i * R], p, 4ull * R);
        p += 4ull * R;
        // Every kernel walks the first count edges of a row and gathers their
        // rows, so a count above R or an id outside the file would read past
        // the arrays: reject the file before anything reaches the device.
        if (hc[i] > R)
          throw std::runtime_error("graph file " + path + ": row " + std::to_string(start + i) +
                                   " has edge count " + std::to_string(hc[i]) + " > n_neighbors " +
                                   std::to_string(R));
        for (uint32_t e = 0; e < hc[i]; e++) {
          const uint32_t id = he[i * R + e];
          if (id != 0xFFFFFFFFu && id >= n)
            throw std::runtime_error("graph file " + path + ": row " + std::to_string(start + i) +
                                     " has neighbour id " + std::to_string(id) + " >= n " +
                                     std::to_string(n));
        }
        memcpy(&hd[i * R], p, 2ull * R);
        p += 2ull * R;
        if (inline_del) {
          if (*p) del_bits[(start + i) >> 3] |= uint8_t(1u << ((start + i) & 7));
          p += 1;
        }
        uint32_t id = uint32_t(start + i);
        if (has_id) memcpy(&id, p, 4);
        hid[i] = id;
        if (id != uint32_t(start + i)) identity = false;
      }
      copy_to(g.vec + start * dpad, hv.data(), cnt * dpad * 2);
      copy_to(g.edges + start * R, he.data(), cnt * R * 4);
      copy_to(g.edist + start * R, hd.data(), cnt * R * 2);
      copy_to(g.counts + start, hc.data(), cnt);
      copy_to(g.slot_to_id + start, hid.data(), cnt * 4);
    }
    if (bitpacked) {
      f.read(reinterpret_cast<char*>(del_bits.data()), std::streamsize(del_bits.size()));
      if (size_t(f.gcount()) != del_bits.size())
        throw std::runtime_error("Short read of deletion bitmask in " + path);
    }
    uint64_t next_id = n;
    if (has_id) {
      f.read(reinterpret_cast<char*>(&next_id), 8);
      if (f.gcount() != 8) next_id = n;
    }
    std::vector<uint32_t> words((n + 31) / 32, 0);
    uint64_t n_del = 0;
    for (uint64_t i = 0; i < n; i++)
      if ((del_bits[i >> 3] >> (i & 7)) & 1u) {
        words[i >> 5] |= 1u << (i & 31);
        n_del++;
      }
    copy_to(g.deleted, words.data(), words.size() * 4);
    g.n_deleted = n_del;
    g.next_id = next_id;
    g.ids_identity = identity;
  } catch (...) {
    graph_free(g);
    throw;
  }
}

void graph_save_file(const Graph& g, const std::string& path) {
  std::ofstream f(path, std::ios::binary);
  if (!f.is_open()) throw std::runtime_error("Failed to open " + path + " for graph save");
  const uint64_t n = g.n, dim = g.dim, R = g.R;
  const uint64_t bpn = 2 * dim + 1 + 6 * R + 4;
  const uint64_t del_bytes = (n + 7) / 8;
  uint64_t hdr[4] = {4 * 8 + n * bpn + del_bytes + 8, n, g.medoid, bpn};
  f.write(reinterpret_cast<const char*>(hdr), sizeof(hdr));
  const size_t chunk = size_t(1) << 18;
  std::vector<uint16_t> hv(chunk * g.dpad), hd(chunk * R);
  std::vector<uint32_t> he(chunk * R), hid(chunk);
  std::vector<uint8_t> hc(chunk);
  std::vector<char> out(chunk * bpn);
  for (uint64_t start = 0; start < n; start += chunk) {
    const size_t cnt = size_t(std::min<uint64_t>(chunk, n - start));
    copy_to(hv.data(), g.vec + start * g.dpad, cnt * g.dpad * 2);
    copy_to(he.data(), g.edges + start * R, cnt * R * 4);
    copy_to(hd.data(), g.edist + start * R, cnt * R * 2);
    copy_to(hc.data(), g.counts + start, cnt);
    copy_to(hid.data(), g.slot_to_id + start, cnt * 4);
    for (size_t i = 0; i < cnt; i++) {
      char* p = out.data() + i * bpn;
      memcpy(p, &hv[i * g.dpad], 2 * dim); p += 2 * dim;
      *p = char(hc[i]); p += 1;
      memcpy(p, &he[i * R], 4 * R); p += 4 * R;
      memcpy(p, &hd[i * R], 2 * R); p += 2 * R;
      memcpy(p, &hid[i], 4);
    }
    f.write(out.data(), std::streamsize(cnt * bpn));
  }
  std::vector<uint32_t> words((n + 31) / 32);
  copy_to(words.data(), g.deleted, words.size() * 4);
  std::vector<uint8_t> bits(del_bytes, 0);
  for (uint64_t i = 0; i < n; i++)
    if ((words[i >> 5] >> (i & 31)) & 1u) bits[i >> 3] |= uint8_t(1u << (i & 7));
  f.write(reinterpret_cast<const char*>(bits.data()), std::streamsize(bits.size()));
  uint64_t next_id = g.next_id;
  f.write(reinterpret_cast<const char*>(&next_id), 8);
  if (!f.good()) throw std::runtime_error("write failed for " + path);
}

// ---------------------------------------------------------------------------
// Directional trailer (include/jasper/index/graph.cuh:1814-2090):
//   u32 magic 0x484C5344 | u32 version 1 | u8 flags (1 lsh, 2 pq, 4 norms)
//   lsh:  u8 k_ranks | u8 packed word size | f32 c[k_ranks] | f32 norm_denom |
//         n records { word[R * k_ranks] | bf16 mag[R] } padded to 4 bytes
//   pq:   u32 M | u32 K (256) | u32 dsub | f32 centroids[M][K][dsub] |
//         n records { u8 code[M * R] } padded to 4 bytes
//   norms: f32[n]
// The trailer follows the complete base section (records, deletion bitmask,
// next_id).  The reference's loader looks for it at 32 + n * (legacy record
// size) instead, which only lands on it for legacy-layout base sections;
// graph_load_directional accepts the trailer at either offset.

namespace {

constexpr uint32_t kTrailerMagic = 0x484C5344u;
constexpr uint32_t kTrailerVersion = 1u;

size_t pad4(size_t x) { return (x + 3) / 4 * 4; }

}  // namespace

void graph_save_directional(const Graph& g, const std::string& path) {
  graph_save_file(g, path);
  const DirArtifacts& d = g.dir;
  if (g.n == 0) return;
  const bool has_lsh = d.has_lsh, has_pq = d.has_pq, has_norms = d.norms != nullptr;
  if (!has_lsh && !has_pq && !has_norms) return;
  std::ofstream f(path, std::ios::binary | std::ios::app);
  if (!f.is_open()) throw std::runtime_error("cannot reopen " + path + " for the trailer");
  const uint8_t flags = uint8_t((has_lsh ? 1 : 0) | (has_pq ? 2 : 0) | (has_norms ? 4 : 0));
  f.write(reinterpret_cast<const char*>(&kTrailerMagic), 4);
  f.write(reinterpret_cast<const char*>(&kTrailerVersion), 4);
  f.write(reinterpret_cast<const char*>(&flags), 1);
  const size_t n = g.n, R = g.R;
  if (has_lsh) {
    const uint8_t kr = uint8_t(d.k_ranks), ps = uint8_t(d.packed_bytes);
    f.write(reinterpret_cast<const char*>(&kr), 1);
    f.write(reinterpret_cast<const char*>(&ps), 1);
    f.write(reinterpret_cast<const char*>(d.lsh_c), 4 * d.k_ranks);
    f.write(reinterpret_cast<const char*>(&d.norm_denom), 4);
    const size_t wbytes = R * d.k_ranks * d.packed_bytes, rec = pad4(wbytes + 2 * R);
    std::vector<char> words(n * wbytes), mags(n * R * 2), out(n * rec, 0);
    copy_to(words.data(), d.lsh_packed, words.size());
    copy_to(mags.data(), d.lsh_mag, mags.size());
    for (size_t i = 0; i < n; i++) {
      memcpy(&out[i * rec], &words[i * wbytes], wbytes);
      memcpy(&out[i * rec + wbytes], &mags[i * R * 2], R * 2);
    }
    f.write(out.data(), std::streamsize(out.size()));
  }
  if (has_pq) {
    const uint32_t hdr[3] = {d.pq_m, 256u, d.pq_dsub};
    f.write(reinterpret_cast<const char*>(hdr), sizeof(hdr));
    std::vector<float> cent(size_t(d.pq_m) * 256 * d.pq_dsub);
    copy_to(cent.data(), d.pq_centroids, cent.size() * 4);
    f.write(reinterpret_cast<const char*>(cent.data()), std::streamsize(cent.size() * 4));
    const size_t cbytes = R * d.pq_m, rec = pad4(cbytes);
    std::vector<char> codes(n * cbytes), out(n * rec, 0);
    copy_to(codes.data(), d.pq_codes, codes.size());
    for (size_t i = 0; i < n; i++) memcpy(&out[i * rec], &codes[i * cbytes], cbytes);
    f.write(out.data(), std::streamsize(out.size()));
  }
  if (has_norms) {
    std::vector<float> nr(n);
    copy_to(nr.data(), d.norms, n * 4);
    f.write(reinterpret_cast<const char*>(nr.data()), std::streamsize(n * 4));
  }
  if (!f.good()) throw std::runtime_error("write failed for " + path);
}

namespace {

template <typename T>
void read_exact(std::ifstream& f, T* dst, size_t bytes, const std::string& path) {
  f.read(reinterpret_cast<char*>(dst), std::streamsize(bytes));
  if (size_t(f.gcount()) != bytes)
    throw std::runtime_error("short read in the directional trailer of " + path);
}

template <typename T>
T* device_copy(const void* src, size_t bytes, const char* what) {
  void* p = nullptr;
  check(cudaMalloc(&p, bytes + 16), what);
  check(cudaMemcpy(p, src, bytes, cudaMemcpyHostToDevice), what);
  return static_cast<T*>(p);
}

}  // namespace

int graph_load_directional(Graph& g, const std::string& path, uint32_t k_ranks) {
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  if (!f.is_open()) throw std::runtime_error("Failed to open " + path);
  const uint64_t size = uint64_t(f.tellg());
  f.seekg(0);
  uint64_t hdr[4];
  read_exact(f, hdr, sizeof(hdr), path);
  const uint64_t n = hdr[1], bpn = hdr[3];
  const uint64_t legacy = 2ull * g.dim + 1 + 6ull * g.R;
  const bool has_id = bpn == legacy + 4 || bpn == legacy + 5;
  uint64_t full_end = 32 + n * bpn;
  if (bpn == legacy + 4) full_end += (n + 7) / 8;
  if (has_id) full_end += 8;
  const uint64_t offsets[2] = {full_end, 32 + n * legacy};
  int64_t at = -1;
  for (uint64_t off : offsets) {
    if (off + 9 > size) continue;
    f.seekg(std::streamoff(off));
    uint32_t mv[2];
    read_exact(f, mv, 8, path);
    if (mv[0] == kTrailerMagic && mv[1] == kTrailerVersion) { at = int64_t(off); break; }
  }
  if (at < 0 || n == 0) return 0;
  f.seekg(std::streamoff(at + 8));
  uint8_t flags = 0;
  read_exact(f, &flags, 1, path);
  DirArtifacts& d = g.dir;
  const size_t R = g.R;
  if (flags & 1) {
    uint8_t kr = 0, ps = 0;
    read_exact(f, &kr, 1, path);
    read_exact(f, &ps, 1, path);
    const uint32_t want_ps = g.dpad <= 128 ? 1u : 2u;
    if (kr != k_ranks || ps != want_ps)
      throw std::runtime_error("directional trailer of " + path + ": k_ranks/packed word size " +
                               std::to_string(kr) + "/" + std::to_string(ps) +
                               " do not match the requested " + std::to_string(k_ranks) + "/" +
                               std::to_string(want_ps));
    float c[17] = {};
    read_exact(f, c, 4 * (size_t(kr) + 1), path);
    const size_t wbytes = R * kr * ps, rec = pad4(wbytes + 2 * R);
    std::vector<char> in(n * rec), words(n * wbytes), mags(n * R * 2);
    read_exact(f, in.data(), in.size(), path);
    for (size_t i = 0; i < n; i++) {
      memcpy(&words[i * wbytes], &in[i * rec], wbytes);
      memcpy(&mags[i * R * 2], &in[i * rec + wbytes], R * 2);
    }
    if (d.lsh_packed) cudaFree(d.lsh_packed);
    if (d.lsh_mag) cudaFree(d.lsh_mag);
    d.lsh_packed = device_copy<void>(words.data(), words.size(), "upload lsh words");
    d.lsh_mag = device_copy<uint16_t>(mags.data(), mags.size(), "upload lsh magnitudes");
    for (uint32_t r = 0; r < 16; r++) d.lsh_c[r] = r < kr ? c[r] : 0.f;
    d.norm_denom = c[kr];
    d.k_ranks = kr;
    d.packed_bytes = ps;
    d.has_lsh = true;
  }
  if (flags & 2) {
    uint32_t ph[3];
    read_exact(f, ph, sizeof(ph), path);
    if (ph[0] != k_ranks || ph[1] != 256u || ph[0] == 0 || ph[0] * ph[2] != g.dpad)
      throw std::runtime_error("directional trailer of " + path + ": PQ M/K/dsub " +
                               std::to_string(ph[0]) + "/" + std::to_string(ph[1]) + "/" +
                               std::to_string(ph[2]) + " do not match this graph");
    std::vector<float> cent(size_t(ph[0]) * 256 * ph[2]);
    read_exact(f, cent.data(), cent.size() * 4, path);
    const size_t cbytes = R * ph[0], rec = pad4(cbytes);
    std::vector<char> in(n * rec), codes(n * cbytes);
    read_exact(f, in.data(), in.size(), path);
    for (size_t i = 0; i < n; i++) memcpy(&codes[i * cbytes], &in[i * rec], cbytes);
    if (d.pq_centroids) cudaFree(d.pq_centroids);
    if (d.pq_codes) cudaFree(d.pq_codes);
    d.pq_centroids = device_copy<float>(cent.data(), cent.size() * 4, "upload centroids");
    d.pq_codes = device_copy<uint8_t>(codes.data(), codes.size(), "upload codes");
    d.pq_m = ph[0];
    d.pq_dsub = ph[2];
    d.has_pq = true;
  }
  if (flags & 4) {
    std::vector<float> nr(n);
    read_exact(f, nr.data(), n * 4, path);
    if (d.norms) cudaFree(d.norms);
    d.norms = device_copy<float>(nr.data(), n * 4, "upload norms");
  }
  return flags;
}

}  // namespace jb
