// jb_graph.h -- graph storage of jasper_b200.
//
// The reference keeps a graph in 2^20-row segments reached through a device
// array of segment structs (include/jasper/index/graph.cuh:92-496, 829-1066),
// so every gather first loads a segment pointer.  Here a graph is a handful of
// flat, 256-byte-aligned device arrays sized for the whole shard (a 12.5 M-row
// shard at D = 128, R = 64 is ~8 GB, far below 180 GB of HBM):
//   vec     [n][dpad]  fp16 rows, dpad = ceil(dim / 8) * 8, pad lanes zero
//   edges   [n][R]     uint32 neighbour ids (global ids)
//   edist   [n][R]     bf16 distance per edge (reference edge_list::dist)
//   counts  [n]        uint8 edge count
//   slot_to_id [n]     stable id per slot (identity unless a file says otherwise)
//   deleted [ceil(n/32)] soft-delete bitmask, bit i = slot i
// Ids and distances live in separate arrays so the search streams only the
// R x 4-byte id list of an expanded node (256 B at R = 64).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace jb {

enum Metric : int { kL2 = 0, kIP = 1 };

struct GraphView {
  const uint16_t* vec;
  uint32_t* edges;
  uint16_t* edist;
  uint8_t* counts;
  const uint32_t* slot_to_id;
  const uint32_t* deleted;
  uint32_t n;
  uint32_t dim;
  uint32_t dpad;
  uint32_t R;
  uint32_t medoid;
  uint32_t global_offset;
  int metric;
  int ids_identity;
  // Build only (null elsewhere): per row, bit e set when edge slot e was
  // kept by a RobustPrune that tested it with exactly the distance stored
  // for it (its bf16 value).  Lets a later re-prune of the row skip the
  // pairs of two such edges (construct.cu, incremental prune).
  uint64_t* eflag;
};

// Directional artifacts (reference: edge_lsh_list / edge_pq_list / lsh_globals
// / pq_codebooks / graph::d_vector_norms, include/jasper/lsh/edge_lsh.cuh,
// include/jasper/pq/edge_pq.cuh, include/jasper/index/graph.cuh:520-525).
struct DirArtifacts {
  bool has_lsh = false;
  uint32_t k_ranks = 0;       // LSH ranks per edge (4 or 16)
  uint32_t packed_bytes = 0;  // 1 (dim <= 128) or 2
  void* lsh_packed = nullptr; // [n][R * k_ranks] words: sign in the MSB, coord below
  uint16_t* lsh_mag = nullptr;// [n][R] bf16 |v - u|^2
  float lsh_c[16] = {};
  float norm_denom = 0.f;
  bool has_pq = false;
  uint32_t pq_m = 0, pq_dsub = 0;
  float* pq_centroids = nullptr;  // [M][256][dsub]
  uint8_t* pq_codes = nullptr;    // [n][M * R], code of edge e in subspace j at j * R + e
  float* norms = nullptr;         // [n] exact |x|^2
  bool has_rabitq = false;
  uint32_t rq_code_bytes = 0, rq_node_bytes = 0;
  uint8_t* rq_store = nullptr;    // [n][rq_node_bytes]: code bits, f_add, f_rescale (f32)
  float* rq_centroid = nullptr;   // [dim] column mean of the rows the codes were made from
  float* rq_err = nullptr;        // [n] error scale of each row's estimate (search filter)
  bool prerotate = false;
  uint64_t rotation_seed = 0;
  uint16_t* rotation = nullptr;   // [dim][dim] fp16, column-major P (rows rotate as x^T P)
  uint16_t* rotation_pad = nullptr;  // [dpad][dpad] fp16, row i = column i of P, zero padded
};

struct Graph {
  uint32_t dim = 0, dpad = 0, R = 0;
  int metric = kL2;
  uint32_t n = 0;
  uint32_t capacity = 0;       // rows the arrays hold (>= n; grows on append)
  uint32_t medoid = 0;
  uint32_t global_offset = 0;
  bool on_host = false;        // rows live in mapped pinned host memory
  bool ids_identity = true;
  uint64_t n_deleted = 0;
  uint64_t next_id = 0;
  int device = 0;
  uint16_t* vec = nullptr;
  uint32_t* edges = nullptr;
  uint16_t* edist = nullptr;
  uint8_t* counts = nullptr;
  uint32_t* slot_to_id = nullptr;
  uint32_t* deleted = nullptr;
  uint64_t* eflag = nullptr;   // build-time prune flags [capacity] (GraphView::eflag)
  DirArtifacts dir;

  GraphView view() const {
    return GraphView{vec, edges, edist, counts, slot_to_id, deleted, n, dim, dpad, R,
                     medoid, global_offset, metric, ids_identity ? 1 : 0, eflag};
  }
};

inline uint32_t pad_dim(uint32_t d) { return (d + 7u) / 8u * 8u; }

// Host-side graph lifecycle (graph.cu).  All throw std::runtime_error.
void graph_allocate(Graph& g, uint32_t dim, uint32_t R, int metric, uint32_t n, bool on_host);
void graph_free(Graph& g);
// Device-resident graphs: grow every per-row array to hold `rows` rows (the
// first n rows kept; new edge counts and deletion bits zero).
void graph_reserve(Graph& g, uint32_t rows);
// Copy [n][dim] fp16 rows with row stride `stride` elements (host or device
// pointer) into the padded row array.
void graph_upload_rows(Graph& g, const uint16_t* rows, uint32_t stride);
void graph_load_file(Graph& g, const std::string& path, uint32_t dim, uint32_t R, int metric,
                     bool on_host);
void graph_save_file(const Graph& g, const std::string& path);
void graph_free_directional(Graph& g);
// Base file plus the directional trailer (LSH / PQ / norms present in g.dir).
void graph_save_directional(const Graph& g, const std::string& path);
// Read the directional trailer of `path` into g.dir (g already loaded from the
// same file).  Returns the trailer flags (0 when the file has none).
int graph_load_directional(Graph& g, const std::string& path, uint32_t k_ranks);

}  // namespace jb
