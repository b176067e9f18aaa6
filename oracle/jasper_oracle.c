/*
 * jasper_oracle.c -- CPU restatement of Jasper's batched Vamana beam-search
 * path.  TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may call it, as the checker.  The product
 * (jasper_b200/) never links or calls anything in this directory.
 *
 * Every routine restates the reference algorithm literally (not the GPU
 * design of jasper_b200): a sorted entry buffer that is re-sorted, deduped
 * and clipped after each expansion, exactly as the reference kernel does.
 * Citations are to saltsystemslab/Jasper paths.
 *
 * Parity pins: the distance routines are checked against the known answers
 * of tests/test_distance.cu:32-136, and search/build outputs against golden
 * fixtures produced by the reference's own CUDA build (tests/golden/).
 *
 * Numeric contract (include/jasper/distance/distance.cuh:32-106):
 *   L2  : lane t (t = 0..3) of a 4-lane tile walks 16-byte chunks t, t+4, ...
 *         (loads_per_round = 2 only changes load grouping, not order), and
 *         accumulates (float(a_i) - float(b_i))^2 with a fused multiply-add,
 *         in element order; then cg::reduce over the tile, which is the
 *         butterfly (s0 + s2) + (s1 + s3)
 *         (cooperative_groups/details/coalesced_reduce.h: mask 2 then 1).
 *   IP  : lane t walks elements t, t+4, ... with sum = fma(a, b, sum), same
 *         reduce, result negated.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

#define ORC_INVALID 0xFFFFFFFFu
#define ORC_EMPTY_IDX 0x7FFFFFFFu

/* --------------------------------------------------------- thread pool */

/* Minimal parallel-for over [0, n) with dynamic chunking (the image's gcc
 * has no OpenMP runtime).  Each iteration is independent, so results do not
 * depend on the thread count. */
typedef void (*orc_body)(void *ctx, long i);
typedef struct { orc_body fn; void *ctx; long n; long next; pthread_mutex_t mu; } orc_pf;

static int g_threads = 0;

int orc_max_threads(void) {
  long c = sysconf(_SC_NPROCESSORS_ONLN);
  return c > 0 ? (int)c : 1;
}

void orc_set_threads(int n) { g_threads = n; }

static void *pf_worker(void *arg) {
  orc_pf *p = (orc_pf *)arg;
  for (;;) {
    pthread_mutex_lock(&p->mu);
    long i = p->next++;
    pthread_mutex_unlock(&p->mu);
    if (i >= p->n) break;
    p->fn(p->ctx, i);
  }
  return NULL;
}

static void parallel_for(long n, orc_body fn, void *ctx) {
  int nt = g_threads > 0 ? g_threads : orc_max_threads();
  if (nt > 256) nt = 256;
  if (nt <= 1 || n <= 1) { for (long i = 0; i < n; i++) fn(ctx, i); return; }
  orc_pf p = {fn, ctx, n, 0, PTHREAD_MUTEX_INITIALIZER};
  pthread_t th[256];
  int started = 0;
  for (int t = 0; t < nt - 1; t++)
    if (pthread_create(&th[started], NULL, pf_worker, &p) == 0) started++;
  pf_worker(&p);
  for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
}

/* ---------------------------------------------------------------- numbers */

/* IEEE binary16 -> binary32 (exact). */
float orc_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1F;
  uint32_t man = h & 0x3FF;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do { man <<= 1; e++; } while (!(man & 0x400));
      man &= 0x3FF;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* binary32 -> bfloat16, round to nearest even (what a __nv_bfloat16
 * conversion from float does; graph.cuh:491-495). */
uint16_t orc_float_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return (uint16_t)(u >> 16);
}

float orc_bf16_to_float(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* ------------------------------------------------------------- distances */

/* L2 over float-converted elements, `epc` elements per 16-byte chunk (8 for
 * fp16 rows, 4 for the f32 rows used by the reference's own distance tests),
 * `n_chunks` = dim / epc (distance.cuh:108-110). */
static float l2_lanes(const float *a, const float *b, int n_chunks, int epc) {
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  for (int t = 0; t < 4; t++) {
    float acc = 0.f;
    for (int c = t; c < n_chunks; c += 4) {
      for (int e = 0; e < epc; e++) {
        float d = a[c * epc + e] - b[c * epc + e];
        acc = fmaf(d, d, acc);
      }
    }
    s[t] = acc;
  }
  return (s[0] + s[2]) + (s[1] + s[3]);
}

static float ip_lanes(const float *a, const float *b, int dim) {
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  for (int t = 0; t < 4; t++) {
    float acc = 0.f;
    for (int i = t; i < dim; i += 4) acc = fmaf(a[i], b[i], acc);
    s[t] = acc;
  }
  return -((s[0] + s[2]) + (s[1] + s[3]));
}

/* Known-answer entry for f32 rows (tests/test_distance.cu uses float data). */
float orc_distance_f32(int metric, const float *a, const float *b, int dim) {
  if (metric == 0) return l2_lanes(a, b, dim / 4, 4);
  return ip_lanes(a, b, dim);
}

/* fp16 rows.  `dim` is the element count handed to compute_distance: the
 * padded dim in the search kernel (device_kernels.cuh:42-49) and the raw
 * graph dim in the prune kernels (construct.cuh:437-439). */
float orc_distance_f16(int metric, const uint16_t *a, const uint16_t *b, int dim) {
  float fa[4096], fb[4096];
  if (dim > 4096) return NAN;
  for (int i = 0; i < dim; i++) {
    fa[i] = orc_half_to_float(a[i]);
    fb[i] = orc_half_to_float(b[i]);
  }
  if (metric == 0) return l2_lanes(fa, fb, dim / 8, 8);
  return ip_lanes(fa, fb, dim);
}

/* ----------------------------------------------------------------- graph */

typedef struct {
  uint32_t n;            /* rows                                    */
  uint32_t dim, dpad;    /* dim and row stride (multiple of 8)      */
  uint32_t R;            /* degree                                  */
  int metric;            /* 0 = L2, 1 = IP                          */
  uint32_t medoid;
  uint32_t global_offset;
  const uint16_t *vec;   /* [n * dpad] fp16 bits                    */
  uint32_t *edges;       /* [n * R]                                 */
  uint16_t *edist;       /* [n * R] bf16 bits                       */
  uint8_t *counts;       /* [n]                                     */
  const uint32_t *deleted; /* [ceil(n/32)] or NULL                  */
} orc_graph;

static inline const uint16_t *row(const orc_graph *g, uint32_t gid) {
  return g->vec + (size_t)(gid - g->global_offset) * g->dpad;
}

/* Entry: (index, distance, visited), ordered as CustomPairLess
 * (device_kernels.cuh:132-151): distance, then 31-bit index. */
typedef struct { uint32_t idx; float dist; int visited; } orc_entry;

static int entry_less(const orc_entry *a, const orc_entry *b) {
  if (a->dist < b->dist) return 1;
  if (a->dist == b->dist && (a->idx & 0x7FFFFFFFu) < (b->idx & 0x7FFFFFFFu)) return 1;
  return 0;
}

/* Stable merge sort (cub::BlockMergeSort::Sort is stable: StableSort simply
 * calls Sort, cub/block/block_merge_sort.cuh). */
static void stable_sort(orc_entry *v, int n, orc_entry *tmp) {
  for (int w = 1; w < n; w *= 2) {
    for (int lo = 0; lo < n; lo += 2 * w) {
      int mid = lo + w < n ? lo + w : n, hi = lo + 2 * w < n ? lo + 2 * w : n;
      int i = lo, j = mid, k = lo;
      while (i < mid && j < hi) tmp[k++] = entry_less(&v[j], &v[i]) ? v[j++] : v[i++];
      while (i < mid) tmp[k++] = v[i++];
      while (j < hi) tmp[k++] = v[j++];
    }
    memcpy(v, tmp, sizeof(orc_entry) * n);
  }
}

static int is_deleted(const orc_graph *g, uint32_t gid) {
  if (!g->deleted) return 0;
  uint32_t l = gid - g->global_offset;
  return (g->deleted[l >> 5] >> (l & 31)) & 1u;
}

/* One query of beam_search_kernel (include/jasper/beam_search/beam_search.cuh:
 * 25-259).  `q` is a padded fp16 row.  Writes k (id, dist) pairs; unfilled
 * slots get (UINT32_MAX, 1e30f) (beam_search.cuh:218-221).  When `visited`
 * is non-NULL records the expansion order (beam_search.cuh:157-166).
 * Returns the number of expansions. */
static void rabitq_query_prep(const uint16_t *q, uint32_t dim, const float *c, int ip,
                              uint32_t *planes, float *vl_out, float *delta_out, int *S_out,
                              float *gadd_out, float *qcn_out);
static float rabitq_estimate(const uint8_t *node, uint32_t code_bytes, uint32_t dim,
                             const uint32_t *planes, float vl, float delta, int S, float gadd,
                             int ip);

/* RaBitQ candidate filter of the exact beam search (no reference
 * counterpart): with the beam full, a new neighbour v is skipped -- its row
 * never read -- when est(v) - margin * |q - c| * err(v) > the beam's worst
 * exact distance; otherwise the search is the reference's exactly. */
typedef struct {
  const uint8_t *store;     /* [n][node_bytes]: code bits, f_add, f_rescale */
  uint32_t node_bytes, code_bytes;
  const float *centroid;    /* [dim] */
  const float *err;         /* [n] */
  float margin;
} orc_rq;

static const orc_rq *g_rq = NULL;  /* filter for orc_search_one (test infrastructure) */

uint32_t orc_search_one(const orc_graph *g, const uint16_t *q, uint32_t k,
                        uint32_t bw, uint32_t limit, uint32_t max_result_size,
                        uint32_t *out_idx, float *out_dist,
                        uint32_t *visited_idx, float *visited_dist,
                        uint64_t *n_dist_evals) {
  const orc_rq *rq = g_rq;
  uint32_t *rq_planes = NULL;
  float rq_vl = 0.f, rq_delta = 0.f, rq_gadd = 0.f, rq_qcn = 0.f, rq_lq = 0.f;
  int rq_S = 0;
  if (rq) {
    rq_planes = (uint32_t *)calloc((size_t)4 * ((g->dim + 31) / 32), sizeof(uint32_t));
    rabitq_query_prep(q, g->dim, rq->centroid, g->metric == 1, rq_planes, &rq_vl, &rq_delta,
                      &rq_S, &rq_gadd, &rq_qcn);
    rq_lq = rq->margin * rq_qcn;
  }
  uint32_t cap = bw + 64 + 64;
  orc_entry *buf = (orc_entry *)malloc(sizeof(orc_entry) * cap);
  orc_entry *tmp = (orc_entry *)malloc(sizeof(orc_entry) * cap);
  uint32_t count = 1;
  uint64_t evals = 0;
  buf[0].idx = g->medoid; buf[0].visited = 0;
  buf[0].dist = orc_distance_f16(g->metric, q, row(g, g->medoid), g->dpad);
  evals++;
  uint32_t visited_counter = 0, loop_count = 0;
  uint32_t lo = g->global_offset, hi = g->global_offset + g->n;
  while (loop_count <= limit) {
    loop_count++;
    /* choose_new_frontier: first unvisited (device_kernels.cuh:60-92) */
    int f = -1;
    for (uint32_t i = 0; i < count; i++) if (!buf[i].visited) { f = (int)i; break; }
    if (f < 0) break;
    buf[f].visited = 1;
    if (visited_idx) {
      visited_idx[visited_counter] = buf[f].idx;
      visited_dist[visited_counter] = buf[f].dist;
    }
    visited_counter++;
    if (visited_counter == max_result_size) break;
    /* add_frontier_out (device_kernels.cuh:95-129) */
    uint32_t u = buf[f].idx;
    uint32_t ne = g->counts[u - g->global_offset];
    uint32_t off = count;
    const int filter = rq != NULL && count >= bw;
    const float tau = filter ? buf[bw - 1].dist : 0.0f;
    uint32_t added = 0;
    for (uint32_t i = 0; i < ne; i++) {
      uint32_t nb = g->edges[(size_t)(u - g->global_offset) * g->R + i];
      orc_entry e;
      if (nb >= lo && nb < hi) { e.idx = nb; e.dist = 3.402823466e+38f; e.visited = 0; }
      else { e.idx = ORC_EMPTY_IDX; e.dist = 3.402823466e+38f; e.visited = 1; }
      if (filter && e.idx != ORC_EMPTY_IDX) {
        const size_t l = nb - g->global_offset;
        const float est = rabitq_estimate(rq->store + l * rq->node_bytes, rq->code_bytes, g->dim,
                                          rq_planes, rq_vl, rq_delta, rq_S, rq_gadd,
                                          g->metric == 1);
        if (est - rq_lq * rq->err[l] > tau) continue;
      }
      buf[off + added++] = e;
    }
    count += added;
    /* populate_distances from offset (device_kernels.cuh:23-57) */
    for (uint32_t i = off; i < count; i++) {
      if (buf[i].idx != ORC_EMPTY_IDX) {
        buf[i].dist = orc_distance_f16(g->metric, q, row(g, buf[i].idx), g->dpad);
        evals++;
      }
    }
    stable_sort(buf, (int)count, tmp);
    /* dedup_results: keep the first of each run of equal index
     * (device_kernels.cuh:197-288) */
    uint32_t w = 0;
    for (uint32_t i = 0; i < count; i++) {
      if (i > 0 && (buf[i].idx & 0x7FFFFFFFu) == (buf[i - 1].idx & 0x7FFFFFFFu)) continue;
      buf[w++] = buf[i];
    }
    /* the predecessor test above looks at the unfiltered neighbour, as the
     * reference does (it compares with the previous element's index). */
    count = w;
    if (count > bw) count = bw; /* clip_k */
  }
  uint32_t out = 0;
  for (uint32_t i = 0; i < count && out < k; i++) {
    uint32_t idx = buf[i].idx & 0x7FFFFFFFu;
    if (idx == ORC_EMPTY_IDX || idx < lo || idx >= hi) continue; /* is_valid */
    if (is_deleted(g, idx)) continue;
    out_idx[out] = idx;
    out_dist[out] = buf[i].dist;
    out++;
  }
  for (; out < k; out++) { out_idx[out] = ORC_INVALID; out_dist[out] = 1e30f; }
  free(buf);
  free(tmp);
  free(rq_planes);
  if (n_dist_evals) *n_dist_evals = evals;
  return visited_counter;
}

void orc_set_rabitq_filter(const uint8_t *store, uint32_t node_bytes, const float *centroid,
                           const float *err, float margin, int enable) {
  static orc_rq rq;
  if (!enable) { g_rq = NULL; return; }
  rq.store = store; rq.node_bytes = node_bytes; rq.code_bytes = node_bytes - 8;
  rq.centroid = centroid; rq.err = err; rq.margin = margin;
  g_rq = &rq;
}

/* Batch of independent queries (one CUDA block each in the reference). */
typedef struct {
  const orc_graph *g; const uint16_t *queries; uint32_t k, bw, limit, mrs;
  uint32_t *out_idx; float *out_dist; uint32_t *n_expanded; uint64_t *n_dist_evals;
} search_ctx;

static void search_body(void *vctx, long qi) {
  search_ctx *c = (search_ctx *)vctx;
  uint64_t ev = 0;
  uint32_t e = orc_search_one(c->g, c->queries + (size_t)qi * c->g->dpad, c->k, c->bw,
                              c->limit, c->mrs, c->out_idx + (size_t)qi * c->k,
                              c->out_dist + (size_t)qi * c->k, NULL, NULL, &ev);
  if (c->n_expanded) c->n_expanded[qi] = e;
  if (c->n_dist_evals) c->n_dist_evals[qi] = ev;
}

void orc_search(const orc_graph *g, const uint16_t *queries, uint32_t nq,
                uint32_t k, uint32_t bw, uint32_t limit, uint32_t max_result_size,
                uint32_t *out_idx, float *out_dist, uint32_t *n_expanded,
                uint64_t *n_dist_evals) {
  search_ctx c = {g, queries, k, bw, limit, max_result_size, out_idx, out_dist,
                  n_expanded, n_dist_evals};
  parallel_for((long)nq, search_body, &c);
}

/* ----------------------------------------------------------------- build */

typedef struct { uint32_t id; float d; } orc_pair;

static int pair_less(const orc_pair *a, const orc_pair *b) {
  if (a->d != b->d) return a->d < b->d;
  return a->id < b->id;
}

static void sort_pairs(orc_pair *v, int n) { /* insertion sort, n <= ~400 */
  for (int i = 1; i < n; i++) {
    orc_pair x = v[i];
    int j = i - 1;
    while (j >= 0 && pair_less(&x, &v[j])) { v[j + 1] = v[j]; j--; }
    v[j + 1] = x;
  }
}

/* RobustPrune over sorted candidates (construct.cuh:419-463 and 686-726):
 * keep c unless some selected s has d(c, s) * alpha < d(p, c); stop at R. */
static uint32_t robust_prune(const orc_graph *g, uint32_t self, const orc_pair *c,
                             uint32_t nc, float alpha, uint32_t *sel, float *sel_d) {
  uint32_t ns = 0;
  for (uint32_t i = 0; i < nc; i++) {
    if (ns >= g->R) break;
    if (c[i].id == self || c[i].id == ORC_INVALID) continue;
    int pruned = 0;
    for (uint32_t j = 0; j < ns && !pruned; j++) {
      float d = orc_distance_f16(g->metric, row(g, c[i].id), row(g, sel[j]), (int)g->dim);
      if (d * alpha < c[i].d) pruned = 1;
    }
    if (!pruned) { sel[ns] = c[i].id; sel_d[ns] = c[i].d; ns++; }
  }
  return ns;
}

static void write_row(orc_graph *g, uint32_t gid, const uint32_t *sel, const float *sel_d, uint32_t ns) {
  size_t l = gid - g->global_offset;
  for (uint32_t i = 0; i < ns; i++) {
    g->edges[l * g->R + i] = sel[i];
    g->edist[l * g->R + i] = orc_float_to_bf16(sel_d[i]);
  }
  g->counts[l] = (uint8_t)ns;
}

typedef struct { uint32_t src, sink; } orc_rev;

static int rev_cmp(const void *a, const void *b) {
  const orc_rev *x = (const orc_rev *)a, *y = (const orc_rev *)b;
  if (x->src != y->src) return x->src < y->src ? -1 : 1;
  if (x->sink != y->sink) return x->sink < y->sink ? -1 : 1;
  return 0;
}

#define ORC_BUILD_L 64
#define ORC_BUILD_LIMIT 256
#define ORC_BUILD_MAX_RESULT 256

typedef struct {
  orc_graph *g; uint32_t off; float alpha;
  uint32_t *vis_idx; float *vis_dist; uint32_t *vis_cnt;
  const orc_rev *rev; const size_t *gstart;
} batch_ctx;

/* (a) greedy search from the medoid for one batch row */
static void batch_search_body(void *vctx, long b) {
  batch_ctx *c = (batch_ctx *)vctx;
  uint32_t tk[ORC_BUILD_L];
  float td[ORC_BUILD_L];
  c->vis_cnt[b] = orc_search_one(c->g, row(c->g, c->off + (uint32_t)b), ORC_BUILD_L,
                                 ORC_BUILD_L, ORC_BUILD_LIMIT, ORC_BUILD_MAX_RESULT, tk, td,
                                 c->vis_idx + (size_t)b * ORC_BUILD_MAX_RESULT,
                                 c->vis_dist + (size_t)b * ORC_BUILD_MAX_RESULT, NULL);
}

/* (b)+(c) merge_candidates_kernel (construct.cuh:280-377) + robust_prune_kernel
 * (construct.cuh:379-473) for one batch row */
static void batch_prune_body(void *vctx, long b) {
  batch_ctx *c = (batch_ctx *)vctx;
  orc_graph *g = c->g;
  const uint32_t R = g->R, maxc = ORC_BUILD_MAX_RESULT + R;
  uint32_t gid = c->off + (uint32_t)b;
  orc_pair *cand = (orc_pair *)malloc(sizeof(orc_pair) * maxc);
  uint32_t nc = 0;
  size_t l = gid - g->global_offset;
  for (uint32_t i = 0; i < g->counts[l]; i++) {
    uint32_t nb = g->edges[l * R + i];
    if (nb == ORC_INVALID) continue;
    if (nc < maxc) { cand[nc].id = nb; cand[nc].d = orc_bf16_to_float(g->edist[l * R + i]); nc++; }
  }
  for (uint32_t i = 0; i < c->vis_cnt[b]; i++) {
    uint32_t v = c->vis_idx[(size_t)b * ORC_BUILD_MAX_RESULT + i];
    if (v == gid || v == ORC_INVALID) continue;
    if (nc < maxc) {
      cand[nc].id = v;
      cand[nc].d = c->vis_dist[(size_t)b * ORC_BUILD_MAX_RESULT + i];
      nc++;
    }
  }
  sort_pairs(cand, (int)nc);
  uint32_t sel[256];
  float sel_d[256];
  uint32_t ns = robust_prune(g, gid, cand, nc, c->alpha, sel, sel_d);
  write_row(g, gid, sel, sel_d, ns);
  free(cand);
}

/* (e) process_reverse_edges_kernel (construct.cuh:560-741) for one target.
 * Candidates are the target's existing edges (stored bf16 distances) and the
 * reverse sinks with fresh distances, at most MAX_CANDS = 256 + R of them.
 * When there are more, the reference keeps whichever ones its shared-memory
 * atomics place first, which is the existing edges (one cheap pass) and then
 * the sinks roughly in group order; this restatement keeps exactly that: the
 * existing edges, then sinks in (target, sink) order until the cap.  Below the
 * cap both are identical. */
static void batch_reverse_body(void *vctx, long gi) {
  batch_ctx *c = (batch_ctx *)vctx;
  orc_graph *g = c->g;
  const uint32_t R = g->R, maxc = ORC_BUILD_MAX_RESULT + R;
  uint32_t t = c->rev[c->gstart[gi]].src;
  size_t nr = c->gstart[gi + 1] - c->gstart[gi];
  size_t l = t - g->global_offset;
  orc_pair *cand = (orc_pair *)malloc(sizeof(orc_pair) * maxc);
  uint32_t nc = 0;
  for (uint32_t i = 0; i < g->counts[l]; i++) {
    uint32_t nb = g->edges[l * R + i];
    if (nb == ORC_INVALID) continue;
    cand[nc].id = nb; cand[nc].d = orc_bf16_to_float(g->edist[l * R + i]); nc++;
  }
  for (size_t i = 0; i < nr && nc < maxc; i++) {
    uint32_t s = c->rev[c->gstart[gi] + i].sink;
    if (s == ORC_INVALID || s == t) continue;
    cand[nc].id = s;
    cand[nc].d = orc_distance_f16(g->metric, row(g, t), row(g, s), (int)g->dim);
    nc++;
  }
  sort_pairs(cand, (int)nc);
  uint32_t sel[256];
  float sel_d[256];
  uint32_t ns = robust_prune(g, t, cand, nc, c->alpha, sel, sel_d);
  write_row(g, t, sel, sel_d, ns);
  free(cand);
}

/* process_batch (construct.cuh:743-911) for rows [off, off + bs). */
static void process_batch(orc_graph *g, uint32_t off, uint32_t bs, float alpha,
                          uint32_t *vis_idx, float *vis_dist, uint32_t *vis_cnt) {
  const uint32_t R = g->R;
  batch_ctx c = {g, off, alpha, vis_idx, vis_dist, vis_cnt, NULL, NULL};
  parallel_for((long)bs, batch_search_body, &c);
  parallel_for((long)bs, batch_prune_body, &c);
  /* (d) reverse edges grouped by target (fill_reverse_edges + semisort) */
  size_t nrev = 0;
  orc_rev *rev = (orc_rev *)malloc(sizeof(orc_rev) * ((size_t)bs * R + 1));
  for (uint32_t b = 0; b < bs; b++) {
    uint32_t gid = off + b;
    size_t l = gid - g->global_offset;
    for (uint32_t i = 0; i < g->counts[l]; i++) {
      rev[nrev].src = g->edges[l * R + i];
      rev[nrev].sink = gid;
      nrev++;
    }
  }
  qsort(rev, nrev, sizeof(orc_rev), rev_cmp);
  size_t ngroups = 0;
  size_t *gstart = (size_t *)malloc(sizeof(size_t) * (nrev + 1));
  for (size_t i = 0; i < nrev; i++)
    if (i == 0 || rev[i].src != rev[i - 1].src) gstart[ngroups++] = i;
  gstart[ngroups] = nrev;
  c.rev = rev;
  c.gstart = gstart;
  parallel_for((long)ngroups, batch_reverse_body, &c);
  free(gstart);
  free(rev);
}

/* construct_graph -> construction_round (construct.cuh:913-958, 992-1160):
 * batches in id order, sizes 1, 2, 4, ... capped at max_batch_size.  The
 * graph's edge counts must be zero on entry. */
void orc_build(orc_graph *g, float alpha, uint32_t max_batch_size) {
  if (max_batch_size == 0) max_batch_size = 1;
  uint32_t *vis_idx = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)max_batch_size * ORC_BUILD_MAX_RESULT);
  float *vis_dist = (float *)malloc(sizeof(float) * (size_t)max_batch_size * ORC_BUILD_MAX_RESULT);
  uint32_t *vis_cnt = (uint32_t *)malloc(sizeof(uint32_t) * max_batch_size);
  uint32_t count = 0, bs = 1;
  while (count < g->n) {
    if (bs > g->n - count) bs = g->n - count;
    if (bs > max_batch_size) bs = max_batch_size;
    process_batch(g, g->global_offset + count, bs, alpha, vis_idx, vis_dist, vis_cnt);
    count += bs;
    if (bs < max_batch_size) bs = (bs * 2 < max_batch_size) ? bs * 2 : max_batch_size;
  }
  free(vis_idx);
  free(vis_dist);
  free(vis_cnt);
}

/* Live append (append_batch, include/jasper/index/construct.cuh:1169-1265):
 * rows [start, start + count) already sit in g with zero edge counts; they
 * are wired in batches of max_batch rows starting at `start` -- no ramp,
 * unlike the build (construct.cuh:1229-1240) -- with the construction's own
 * process_batch. */
void orc_append_range(orc_graph *g, uint32_t start, uint32_t count, float alpha,
                      uint32_t max_batch) {
  if (count == 0) return;
  if (max_batch == 0) max_batch = count < 100000 ? count : 100000;
  uint32_t *vis_idx = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)max_batch * ORC_BUILD_MAX_RESULT);
  float *vis_dist = (float *)malloc(sizeof(float) * (size_t)max_batch * ORC_BUILD_MAX_RESULT);
  uint32_t *vis_cnt = (uint32_t *)malloc(sizeof(uint32_t) * max_batch);
  for (uint32_t off = start; off < start + count;) {
    uint32_t bs = start + count - off < max_batch ? start + count - off : max_batch;
    process_batch(g, off, bs, alpha, vis_idx, vis_dist, vis_cnt);
    off += bs;
  }
  free(vis_idx);
  free(vis_dist);
  free(vis_cnt);
}

/* ----------------------------------------------------- exact brute force */

/* Multi-threaded exact kNN over fp16 rows (the CPU baseline named by the
 * benchmark plan).  Distances use the same arithmetic as the search. */
typedef struct {
  const uint16_t *base; uint32_t n; const uint16_t *queries; uint32_t dpad;
  int metric; uint32_t k; uint32_t *out_idx; float *out_dist;
} bf_ctx;

static void bf_body(void *vctx, long qi) {
  bf_ctx *c = (bf_ctx *)vctx;
  const uint16_t *q = c->queries + (size_t)qi * c->dpad;
  float qf[4096], vf[4096];
  for (uint32_t i = 0; i < c->dpad; i++) qf[i] = orc_half_to_float(q[i]);
  uint32_t k = c->k;
  orc_pair *best = (orc_pair *)malloc(sizeof(orc_pair) * (k + 1));
  uint32_t nb = 0;
  for (uint32_t v = 0; v < c->n; v++) {
    const uint16_t *r = c->base + (size_t)v * c->dpad;
    for (uint32_t i = 0; i < c->dpad; i++) vf[i] = orc_half_to_float(r[i]);
    orc_pair p;
    p.id = v;
    p.d = c->metric == 0 ? l2_lanes(qf, vf, (int)c->dpad / 8, 8) : ip_lanes(qf, vf, (int)c->dpad);
    if (nb == k && !pair_less(&p, &best[k - 1])) continue;
    int j = (int)(nb < k ? nb : k - 1) - 1;
    if (nb < k) nb++;
    while (j >= 0 && pair_less(&p, &best[j])) { best[j + 1] = best[j]; j--; }
    best[j + 1] = p;
  }
  for (uint32_t i = 0; i < k; i++) {
    c->out_idx[(size_t)qi * k + i] = i < nb ? best[i].id : ORC_INVALID;
    c->out_dist[(size_t)qi * k + i] = i < nb ? best[i].d : 1e30f;
  }
  free(best);
}

void orc_bruteforce(const uint16_t *base, uint32_t n, const uint16_t *queries,
                    uint32_t nq, uint32_t dpad, int metric, uint32_t k,
                    uint32_t *out_idx, float *out_dist) {
  if (dpad > 4096 || k == 0) return;
  bf_ctx c = {base, n, queries, dpad, metric, k, out_idx, out_dist};
  parallel_for((long)nq, bf_body, &c);
}

/* ============================================================ directional */

/* Round a double (holding an exact fp16 sum/difference/product) to fp16
 * bits, round-to-nearest-even -- what __hsub2 / __hmul2 produce. */
static uint16_t double_to_half_bits(double x) {
  uint16_t sign = 0;
  if (x < 0 || (x == 0 && signbit(x))) { sign = 0x8000; x = -x; }
  if (x == 0) return sign;
  if (x >= 65520.0) return sign | 0x7C00;               /* overflow -> inf */
  int e;
  double m = frexp(x, &e);                               /* x = m * 2^e, m in [0.5,1) */
  int exp16 = e - 1 + 15;                                /* biased exponent of 1.xxx */
  double scaled;
  if (exp16 >= 1) scaled = ldexp(x, 10 - (e - 1));       /* mantissa incl. hidden bit */
  else scaled = ldexp(x, 24);                            /* subnormal: units of 2^-24 */
  double fl = floor(scaled);
  double rem = scaled - fl;
  uint64_t q = (uint64_t)fl;
  if (rem > 0.5 || (rem == 0.5 && (q & 1))) q++;
  (void)m;
  if (exp16 >= 1) {
    if (q == 2048) { q = 1024; exp16++; }
    if (exp16 >= 31) return sign | 0x7C00;
    return sign | (uint16_t)(exp16 << 10) | (uint16_t)(q & 0x3FF);
  }
  return sign | (uint16_t)q;                             /* q may reach 1024 = min normal */
}

/* Contraction variants of the reference's float expressions (which fused
 * multiply-adds nvcc forms); the golden fixtures decide.  Bit 0-1: visit term
 * `local += f0*f0 + f1*f1` (0: fma(f0,f0,f1*f1), 1: fma(f1,f1,f0*f0),
 * 2: unfused); bit 2: LSH rank term fused; bit 3: L2 estimate fused. */
static int g_dir_mode = 0 | 4 | 8;
void orc_set_dir_mode(int m) { g_dir_mode = m; }

/* Reduction of 128 per-thread partials as the reference's 128-thread blocks
 * do it: xor butterfly (16, 8, 4, 2, 1) per warp, then the same butterfly
 * over the 4 warp sums padded with zeros (beam_search_common.cuh:133-153). */
static float block128_reduce(const float *part) {
  float ws[32] = {0};
  for (int w = 0; w < 4; w++) {
    float v[32];
    for (int l = 0; l < 32; l++) v[l] = part[w * 32 + l];
    for (int d = 16; d > 0; d >>= 1) {
      float nv[32];
      for (int l = 0; l < 32; l++) nv[l] = v[l] + v[l ^ d];
      memcpy(v, nv, sizeof(v));
    }
    ws[w] = v[0];
  }
  for (int d = 16; d > 0; d >>= 1) {
    float nv[32];
    for (int l = 0; l < 32; l++) nv[l] = ws[l] + ws[l ^ d];
    memcpy(ws, nv, sizeof(ws));
  }
  return ws[0];
}

static float warp_reduce32(float *v) {
  for (int d = 16; d > 0; d >>= 1) {
    float nv[32];
    for (int l = 0; l < 32; l++) nv[l] = v[l] + v[l ^ d];
    memcpy(v, nv, 32 * sizeof(float));
  }
  return v[0];
}

typedef struct {
  int kind;                 /* 0 = LSH, 1 = PQ */
  uint32_t k_ranks;         /* LSH */
  uint32_t packed_bytes;    /* 1 or 2 */
  const void *packed;       /* [n][R * k_ranks] */
  const uint16_t *mag_sq;   /* [n][R] bf16 */
  const float *c;           /* [k_ranks] */
  float norm_denom;
  uint32_t pq_m, pq_dsub;   /* PQ */
  const float *centroids;   /* [M][256][dsub] */
  const uint8_t *codes;     /* [n][M * R] subspace-major */
  const float *norms;       /* [n] */
} orc_dir;

/* compute_qu_diff_and_exact (beam_search_common.cuh:87-154); fills qu (fp16
 * bits of q - u) for L2. */
static float dir_visit_exact(const orc_graph *g, const uint16_t *q, uint32_t u, int ip,
                             uint16_t *qu) {
  float part[128];
  memset(part, 0, sizeof(part));
  const uint16_t *ur = row(g, u);
  const uint32_t nv4 = g->dpad / 8;
  for (uint32_t i = 0; i < nv4; i++) {
    float local = part[i % 128];
    for (int j = 0; j < 4; j++) {
      double a0 = orc_half_to_float(q[8 * i + 2 * j]), a1 = orc_half_to_float(q[8 * i + 2 * j + 1]);
      double b0 = orc_half_to_float(ur[8 * i + 2 * j]), b1 = orc_half_to_float(ur[8 * i + 2 * j + 1]);
      if (!ip) {
        uint16_t h0 = double_to_half_bits(a0 - b0), h1 = double_to_half_bits(a1 - b1);
        if (qu) { qu[8 * i + 2 * j] = h0; qu[8 * i + 2 * j + 1] = h1; }
        float f0 = orc_half_to_float(h0), f1 = orc_half_to_float(h1), t;
        switch (g_dir_mode & 3) {
          case 0: t = fmaf(f0, f0, f1 * f1); break;
          case 1: t = fmaf(f1, f1, f0 * f0); break;
          default: t = f0 * f0 + f1 * f1; break;
        }
        local = local + t;
      } else {
        float p0 = orc_half_to_float(double_to_half_bits(a0 * b0));
        float p1 = orc_half_to_float(double_to_half_bits(a1 * b1));
        local = local + (p0 + p1);
      }
    }
    part[i % 128] = local;
  }
  return block128_reduce(part);
}

static void fr_insert(orc_entry *fr, uint32_t *fc, uint32_t k, uint32_t idx, float d) {
  /* frontier_insert_sorted (beam_search_common.cuh:158-185): strict '>' */
  uint32_t c = *fc;
  int j;
  if (c < k) {
    j = (int)c;
    while (j > 0 && fr[j - 1].dist > d) { fr[j] = fr[j - 1]; j--; }
    fr[j].idx = idx; fr[j].dist = d;
    *fc = c + 1;
    return;
  }
  if (d >= fr[k - 1].dist) return;
  j = (int)k - 1;
  while (j > 0 && fr[j - 1].dist > d) { fr[j] = fr[j - 1]; j--; }
  fr[j].idx = idx; fr[j].dist = d;
}

/* ---- RaBitQ (1 bit per dimension) ------------------------------------- */

/* Query side of the RaBitQ estimator (no reference counterpart; the device
 * kernel computes the same values in the same order).  q = fp16 query in the
 * rotated space, first `dim` coordinates:
 *   vl = min q_i, delta = (max q_i - vl) / 15, qq_i = clamp(rint((q_i - vl) *
 *   15 / (max - vl)), 0, 15), S = sum qq_i, plane p bit i = (qq_i >> p) & 1;
 *   gadd = sum (q_i - c_i)^2 (L2) or -sum c_i q_i (IP), summed lane-strided
 *   over 32 lanes (i = l, l + 32, ...; fma) and reduced by the warp butterfly. */
static void rabitq_query_prep(const uint16_t *q, uint32_t dim, const float *c, int ip,
                              uint32_t *planes, float *vl_out, float *delta_out, int *S_out,
                              float *gadd_out, float *qcn_out) {
  float vl = orc_half_to_float(q[0]), vr = vl;
  for (uint32_t i = 1; i < dim; i++) {
    float x = orc_half_to_float(q[i]);
    if (x < vl) vl = x;
    if (x > vr) vr = x;
  }
  const float range = vr - vl;
  const float delta = range / 15.0f;
  const float inv = range > 0.0f ? 15.0f / range : 0.0f;
  int S = 0;
  for (uint32_t i = 0; i < dim; i++) {
    float x = orc_half_to_float(q[i]);
    int qq = (int)rintf((x - vl) * inv);
    if (qq < 0) qq = 0;
    if (qq > 15) qq = 15;
    S += qq;
    for (int p = 0; p < 4; p++)
      if ((qq >> p) & 1) planes[(size_t)p * ((dim + 31) / 32) + i / 32] |= 1u << (i % 32);
  }
  float v[32];
  for (int l = 0; l < 32; l++) {
    float acc = 0.f;
    for (uint32_t i = (uint32_t)l; i < dim; i += 32) {
      float x = orc_half_to_float(q[i]);
      if (ip) acc = fmaf(c[i], x, acc);
      else { float d = x - c[i]; acc = fmaf(d, d, acc); }
    }
    v[l] = acc;
  }
  float gsum = warp_reduce32(v);
  for (int l = 0; l < 32; l++) {
    float acc = 0.f;
    for (uint32_t i = (uint32_t)l; i < dim; i += 32) {
      float d = orc_half_to_float(q[i]) - c[i];
      acc = fmaf(d, d, acc);
    }
    v[l] = acc;
  }
  float qc2 = warp_reduce32(v);
  *vl_out = vl; *delta_out = delta; *S_out = S;
  *gadd_out = ip ? -gsum : gsum;
  *qcn_out = sqrtf(qc2);
}

/* est = f_add + f_rescale * <code - 1/2, q~> + gadd (IP: minus 1, the
 * distance being -<o, q> while f_add carries 1 - <o, q>), with
 * <code - 1/2, q~> = 0.5 vl (2 popc(b) - dim) + 0.5 delta (2 A - S) and
 * A = sum_p 2^p popc(b & plane_p). */
static float rabitq_estimate(const uint8_t *node, uint32_t code_bytes, uint32_t dim,
                             const uint32_t *planes, float vl, float delta, int S, float gadd,
                             int ip) {
  const uint32_t nw = (dim + 31) / 32;
  int A = 0, pb = 0;
  for (uint32_t w = 0; w < nw; w++) {
    uint32_t b;
    memcpy(&b, node + 4 * w, 4);
    pb += __builtin_popcount(b);
    for (int p = 0; p < 4; p++) A += __builtin_popcount(b & planes[(size_t)p * nw + w]) << p;
  }
  float f_add, f_rescale;
  memcpy(&f_add, node + code_bytes, 4);
  memcpy(&f_rescale, node + code_bytes + 4, 4);
  const float t1 = (float)(2 * pb - (int)dim) * (0.5f * vl);
  const float ipx = fmaf((float)(2 * A - S), 0.5f * delta, t1);
  float est = fmaf(f_rescale, ipx, f_add) + gadd;
  return ip ? est - 1.0f : est;
}

/* rabitq_quantize_kernel<1, TILE_SIZE = 4> (rabitq/quantize.cuh:184-290) for
 * every row of `rows` ([n][stride] floats, first `dim` used): residual
 * r = x - c, partial sums by thread j % 4 with fma, the tile's xor-butterfly
 * (mask 2 then 1); code bit = r >= 0; f_add / f_rescale as the reference
 * writes them.  Output: the reference's array-of-structs node layout. */
static void rabitq_row(const float *x, const float *c, uint32_t dim, int ip, uint8_t *node,
                       uint32_t code_bytes, float *err) {
  float part[4] = {0, 0, 0, 0};
  for (uint32_t j = 0; j < dim; j++) { float r = x[j] - c[j]; part[j % 4] = fmaf(r, r, part[j % 4]); }
  const float l2_sqr = (part[0] + part[2]) + (part[1] + part[3]);
  const float l2_norm = sqrtf(l2_sqr);
  float pn[4] = {0, 0, 0, 0};
  for (uint32_t j = 0; j < dim; j++) {
    float r = x[j] - c[j];
    float abs_o = fabsf(r / l2_norm);
    pn[j % 4] = fmaf(0.5f, abs_o, pn[j % 4]);
  }
  const float ip_norm = (pn[0] + pn[2]) + (pn[1] + pn[3]);
  float ipnorm_inv = 1.0f / ip_norm;
  if (isnan(ipnorm_inv)) ipnorm_inv = 1.0f;
  float a[4] = {0, 0, 0, 0}, b[4] = {0, 0, 0, 0}, cc[4] = {0, 0, 0, 0};
  memset(node, 0, code_bytes);
  for (uint32_t j = 0; j < dim; j++) {
    float r = x[j] - c[j];
    int bit = r >= 0.0f;
    if (bit) node[j / 8] |= (uint8_t)(1u << (j % 8));
    float xu = (float)bit + (-0.5f);
    a[j % 4] = fmaf(r, xu, a[j % 4]);
    b[j % 4] = fmaf(c[j], xu, b[j % 4]);
    cc[j % 4] = fmaf(r, c[j], cc[j % 4]);
  }
  float ip_resi_xucb = (a[0] + a[2]) + (a[1] + a[3]);
  const float ip_cent_xucb = (b[0] + b[2]) + (b[1] + b[3]);
  const float ip_resi_cent = (cc[0] + cc[2]) + (cc[1] + cc[3]);
  if (ip_resi_xucb == 0.0f) ip_resi_xucb = INFINITY;
  float f_add, f_rescale;
  if (!ip) {
    f_add = l2_sqr + ((2.0f * l2_sqr) * ip_cent_xucb) / ip_resi_xucb;
    f_rescale = (ipnorm_inv * -2.0f) * l2_norm;
  } else {
    f_add = (1.0f - ip_resi_cent) + (l2_sqr * ip_cent_xucb) / ip_resi_xucb;
    f_rescale = ipnorm_inv * -l2_norm;
  }
  memcpy(node + code_bytes, &f_add, 4);
  memcpy(node + code_bytes + 4, &f_rescale, 4);
  if (err) {
    /* error scale of the estimate (no reference counterpart): with
     * a = <o_bar, o> = 2 ipn / sqrt(dim), the 1-bit estimate of <r, q - c>
     * has standard error |r| |q - c| sqrt(1 - a^2) / (a sqrt(dim - 1)); err
     * holds that without |q - c|, times 2 for L2 (the term enters as -2<r, q>). */
    const float a = (2.0f * ip_norm) / sqrtf((float)dim);
    const float num = (ip ? 1.0f : 2.0f) * l2_norm * sqrtf(fmaxf(0.0f, 1.0f - a * a));
    *err = num / (a * sqrtf((float)(dim - 1)));
  }
}

uint32_t orc_rabitq_code_bytes(uint32_t dim) { return ((dim + 7) / 8 + 3) / 4 * 4; }

typedef struct { const float *rows; uint64_t stride; const float *c; uint32_t dim; int ip; uint8_t *out; float *err; } rq_ctx;

static void rq_body(void *vctx, long i) {
  rq_ctx *c = (rq_ctx *)vctx;
  const uint32_t cb = orc_rabitq_code_bytes(c->dim);
  rabitq_row(c->rows + (size_t)i * c->stride, c->c, c->dim, c->ip, c->out + (size_t)i * (cb + 8), cb,
             c->err ? c->err + i : NULL);
}

/* err may be NULL (the reference's quantizer has no error output). */
void orc_rabitq_quantize(const float *rows, uint64_t n, uint64_t stride, uint32_t dim,
                         const float *centroid, int ip, uint8_t *out, float *err) {
  rq_ctx c = {rows, stride, centroid, dim, ip, out, err};
  parallel_for((long)n, rq_body, &c);
}

/* Column means of n fp16 rows (dpad stride) accumulated in double in row
 * order, rounded to float: the centroid the graph's RaBitQ codes use. */
void orc_rabitq_centroid(const uint16_t *vec, uint64_t n, uint32_t dim, uint32_t dpad, float *out) {
  for (uint32_t j = 0; j < dim; j++) {
    double s = 0.0;
    for (uint64_t i = 0; i < n; i++) s += (double)orc_half_to_float(vec[i * dpad + j]);
    out[j] = (float)(s / (double)n);
  }
}

/* graph_beam_search_kernel (graph_beam_search.cuh:55-270) with the LSH
 * (directional_beam_search.cuh:31-192) or PQ (pq_beam_search.cuh:31-201)
 * estimator, for one query.  Unfilled outputs are (0x7FFFFFFF, FLT_MAX). */
void orc_dir_search_one(const orc_graph *g, const orc_dir *dd, const uint16_t *q, uint32_t k,
                        uint32_t bw, uint32_t limit, uint32_t max_result_size,
                        uint32_t *out_idx, float *out_dist) {
  const int ip = g->metric == 1;
  const uint32_t R = g->R;
  uint32_t cap = bw + 2 * R + 8;
  orc_entry *buf = (orc_entry *)malloc(sizeof(orc_entry) * cap);
  orc_entry *tmp = (orc_entry *)malloc(sizeof(orc_entry) * cap);
  orc_entry *fr = (orc_entry *)malloc(sizeof(orc_entry) * (k + 1));
  uint16_t *qu = (uint16_t *)calloc(g->dpad, sizeof(uint16_t));
  float *lut = NULL;
  float q_sq = 0.f, inv_nd = 0.f;
  uint32_t fc = 0, count = 1;
  buf[0].idx = g->medoid; buf[0].dist = 0.0f; buf[0].visited = 0;
  if (dd->kind == 0) {
    inv_nd = 1.0f / dd->norm_denom;
  } else {
    const uint32_t M = dd->pq_m, dsub = dd->pq_dsub;
    lut = (float *)malloc(sizeof(float) * M * 256);
    for (uint32_t e = 0; e < M * 256; e++) {       /* pq_build_lut: warp per centroid */
      uint32_t j = e / 256;
      float v[32];
      for (int l = 0; l < 32; l++) {
        float acc = 0.f;
        for (uint32_t t = (uint32_t)l; t < dsub; t += 32)
          acc = fmaf(orc_half_to_float(q[j * dsub + t]), dd->centroids[(size_t)e * dsub + t], acc);
        v[l] = acc;
      }
      lut[e] = warp_reduce32(v);
    }
    if (!ip) {                                       /* ||q||^2, 128-thread block */
      float part[128];
      memset(part, 0, sizeof(part));
      for (uint32_t i = 0; i < g->dpad; i++) {
        float x = orc_half_to_float(q[i]);
        part[i % 128] = fmaf(x, x, part[i % 128]);
      }
      q_sq = block128_reduce(part);
    }
  }
  uint32_t visited_counter = 0, loop_count = 0;
  const uint32_t lo = g->global_offset, hi = g->global_offset + g->n;
  while (loop_count <= limit) {
    loop_count++;
    int f = -1;
    for (uint32_t i = 0; i < count; i++) if (!buf[i].visited) { f = (int)i; break; }
    if (f < 0) break;
    buf[f].visited = 1;
    const uint32_t u = buf[f].idx;
    float exact_u, dist_u;
    if (dd->kind == 0) {
      exact_u = dir_visit_exact(g, q, u, ip, ip ? NULL : qu);
      dist_u = ip ? -exact_u : exact_u;
    } else {
      exact_u = dir_visit_exact(g, q, u, 1, NULL);   /* <q, u> */
      dist_u = ip ? -exact_u : (q_sq - 2.0f * exact_u) + dd->norms[u - g->global_offset];
    }
    fr_insert(fr, &fc, k, u, dist_u);
    visited_counter++;
    if (visited_counter == max_result_size) break;
    const size_t lu = u - g->global_offset;
    const uint32_t ne = g->counts[lu];
    const uint32_t off = count;
    for (uint32_t e = 0; e < ne; e++) {
      uint32_t nb = g->edges[lu * R + e];
      orc_entry en;
      if (nb >= lo && nb < hi) { en.idx = nb; en.dist = 3.402823466e+38f; en.visited = 0; }
      else { en.idx = ORC_EMPTY_IDX; en.dist = 3.402823466e+38f; en.visited = 1; }
      buf[off + e] = en;
    }
    count += ne;
    for (uint32_t e = 0; e < ne; e++) {
      orc_entry *en = &buf[off + e];
      if (en->idx == ORC_EMPTY_IDX) continue;
      float est;
      if (dd->kind == 0) {
        float dot = 0.f;
        for (uint32_t r = 0; r < dd->k_ranks; r++) {
          uint32_t word, coord, neg;
          if (dd->packed_bytes == 1) {
            word = ((const uint8_t *)dd->packed)[lu * R * dd->k_ranks + e * dd->k_ranks + r];
            coord = word & 0x7F; neg = word & 0x80;
          } else {
            word = ((const uint16_t *)dd->packed)[lu * R * dd->k_ranks + e * dd->k_ranks + r];
            coord = word & 0x7FFF; neg = word & 0x8000;
          }
          float x = orc_half_to_float(ip ? q[coord] : qu[coord]);
          float cs = dd->c[r] * (neg ? -1.0f : 1.0f);
          dot = (g_dir_mode & 4) ? fmaf(cs, x, dot) : dot + cs * x;
        }
        float dot_est = dot * inv_nd;
        float mag_sq = orc_bf16_to_float(dd->mag_sq[lu * R + e]);
        float mag = sqrtf(mag_sq);
        if (!ip) {
          float base = exact_u + mag_sq;
          est = (g_dir_mode & 8) ? fmaf(-(2.0f * mag), dot_est, base) : base - (2.0f * mag) * dot_est;
        } else {
          float ipv = fmaf(mag, dot_est, exact_u);
          est = -ipv;
        }
      } else {
        float acc = exact_u;
        for (uint32_t j = 0; j < dd->pq_m; j++)
          acc = acc + lut[j * 256 + dd->codes[lu * dd->pq_m * R + j * R + e]];
        est = ip ? -acc : (q_sq - 2.0f * acc) + dd->norms[en->idx - g->global_offset];
      }
      en->dist = est;
    }
    stable_sort(buf, (int)count, tmp);
    uint32_t w = 0;
    for (uint32_t i = 0; i < count; i++) {
      if (i > 0 && (buf[i].idx & 0x7FFFFFFFu) == (buf[i - 1].idx & 0x7FFFFFFFu)) continue;
      buf[w++] = buf[i];
    }
    count = w;
    if (count > bw) count = bw;
  }
  uint32_t out = 0;
  for (uint32_t i = 0; i < fc && out < k; i++) {
    uint32_t idx = fr[i].idx;
    if (idx < lo || idx >= hi) continue;
    if (is_deleted(g, idx)) continue;
    out_idx[out] = idx; out_dist[out] = fr[i].dist; out++;
  }
  for (; out < k; out++) { out_idx[out] = ORC_EMPTY_IDX; out_dist[out] = 3.402823466e+38f; }
  free(buf); free(tmp); free(fr); free(qu); free(lut);
}

typedef struct {
  const orc_graph *g; const orc_dir *dd; const uint16_t *queries;
  uint32_t k, bw, limit; uint32_t *oi; float *od;
} dir_ctx;

static void dir_body(void *vctx, long qi) {
  dir_ctx *c = (dir_ctx *)vctx;
  orc_dir_search_one(c->g, c->dd, c->queries + (size_t)qi * c->g->dpad, c->k, c->bw, c->limit,
                     2048, c->oi + (size_t)qi * c->k, c->od + (size_t)qi * c->k);
}

void orc_dir_search(const orc_graph *g, const orc_dir *dd, const uint16_t *queries, uint32_t nq,
                    uint32_t k, uint32_t bw, uint32_t limit, uint32_t *oi, float *od) {
  dir_ctx c = {g, dd, queries, k, bw, limit, oi, od};
  parallel_for((long)nq, dir_body, &c);
}

/* ---- directional artifact builders (exact parts) ----------------------- */

/* populate_lsh (include/jasper/lsh/lsh_kernels.cuh:9-131), 128 threads:
 * Δ = v − u in fp16; key = |Δ| half bits << (B+1) | sign << B | coord with
 * B = 7 (packed_bytes 1) or 15; Σ float(Δ)² with thread t (= i mod 128)
 * accumulating fmaf(f, f, acc) and the two-level block butterfly; k_ranks
 * rounds of argmax, the winner's low B+1 bits stored, then zeroed.  Only edge
 * slots below the edge count are written. */
typedef struct { const orc_graph *g; uint32_t k_ranks; int pb; void *packed; uint16_t *mag; } lsh_ctx;

static void lsh_body(void *vctx, long l) {
  lsh_ctx *c = (lsh_ctx *)vctx;
  const orc_graph *g = c->g;
  const uint32_t B = c->pb == 1 ? 7u : 15u, cmask = (1u << B) - 1u;
  const uint16_t *u = g->vec + (size_t)l * g->dpad;
  uint32_t *keys = (uint32_t *)malloc(sizeof(uint32_t) * g->dpad);
  for (uint32_t e = 0; e < g->counts[l]; e++) {
    const uint32_t nb = g->edges[(size_t)l * g->R + e];
    const uint16_t *v = row(g, nb);
    float part[128] = {0};
    for (uint32_t i = 0; i < g->dpad; i++) {
      uint16_t h = double_to_half_bits((double)orc_half_to_float(v[i]) - (double)orc_half_to_float(u[i]));
      keys[i] = ((uint32_t)(h & 0x7FFFu) << (B + 1)) | ((uint32_t)((h >> 15) & 1u) << B) | (i & cmask);
      float f = orc_half_to_float(h);
      part[i % 128] = fmaf(f, f, part[i % 128]);
    }
    float m2 = block128_reduce(part);
    for (uint32_t r = 0; r < c->k_ranks; r++) {
      uint32_t best = 0;
      for (uint32_t i = 0; i < g->dpad; i++) if (keys[i] > best) best = keys[i];
      size_t w = ((size_t)l * g->R + e) * c->k_ranks + r;
      if (c->pb == 1) ((uint8_t *)c->packed)[w] = (uint8_t)best;
      else ((uint16_t *)c->packed)[w] = (uint16_t)best;
      keys[best & cmask] = 0;
    }
    c->mag[(size_t)l * g->R + e] = orc_float_to_bf16(m2);
  }
  free(keys);
}

void orc_lsh_edges(const orc_graph *g, uint32_t k_ranks, int packed_bytes, void *packed,
                   uint16_t *mag) {
  lsh_ctx c = {g, k_ranks, packed_bytes, packed, mag};
  parallel_for((long)g->n, lsh_body, &c);
}

/* pq_populate (include/jasper/pq/pq_kernels.cuh:252-295): residual
 * float(fp16(v − u)); per subspace, d_c = Σ_t fmaf(r_t − C_t, ·, d) in t
 * order; the lowest (d, c) wins (pq_block_argmin, :25-58). */
typedef struct { const orc_graph *g; uint32_t M; const float *cent; uint8_t *codes; } pqc_ctx;

static void pqc_body(void *vctx, long l) {
  pqc_ctx *c = (pqc_ctx *)vctx;
  const orc_graph *g = c->g;
  const uint32_t dsub = g->dpad / c->M;
  const uint16_t *u = g->vec + (size_t)l * g->dpad;
  float *res = (float *)malloc(sizeof(float) * g->dpad);
  for (uint32_t e = 0; e < g->counts[l]; e++) {
    const uint16_t *v = row(g, g->edges[(size_t)l * g->R + e]);
    for (uint32_t i = 0; i < g->dpad; i++)
      res[i] = orc_half_to_float(double_to_half_bits((double)orc_half_to_float(v[i]) -
                                                     (double)orc_half_to_float(u[i])));
    for (uint32_t j = 0; j < c->M; j++) {
      float best = 0; int bi = -1;
      for (int cc = 0; cc < 256; cc++) {
        const float *C = c->cent + ((size_t)j * 256 + cc) * dsub;
        float d = 0.0f;
        for (uint32_t t = 0; t < dsub; t++) { float df = res[j * dsub + t] - C[t]; d = fmaf(df, df, d); }
        if (bi < 0 || d < best) { best = d; bi = cc; }
      }
      c->codes[(size_t)l * c->M * g->R + (size_t)j * g->R + e] = (uint8_t)bi;
    }
  }
  free(res);
}

void orc_pq_codes(const orc_graph *g, uint32_t M, const float *cent, uint8_t *codes) {
  pqc_ctx c = {g, M, cent, codes};
  parallel_for((long)g->n, pqc_body, &c);
}

/* pq_compute_vector_norms (pq_kernels.cuh:218-247), 128 threads. */
void orc_row_norms(const orc_graph *g, float *norms) {
  for (uint32_t l = 0; l < g->n; l++) {
    float part[128] = {0};
    for (uint32_t i = 0; i < g->dpad; i++) {
      float v = orc_half_to_float(g->vec[(size_t)l * g->dpad + i]);
      part[i % 128] = fmaf(v, v, part[i % 128]);
    }
    norms[l] = block128_reduce(part);
  }
}
