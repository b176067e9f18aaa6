/* Exact brute-force k-nearest-neighbour search on the host cores.
 *
 * TEST / MEASUREMENT INFRASTRUCTURE ONLY: the multi-threaded CPU baseline the
 * benchmark reports beside the GPU search (fp16 rows widened to fp32 by the
 * caller, every query compared with every row, per-thread top-k).  Nothing
 * in the product links it.
 *
 * Distances: L2 = |q|^2 + |x|^2 - 2<q,x> (fp32), inner product = -<q,x>, the
 * reference's conventions (distance/distance.cuh:32-106: smaller is nearer,
 * IP negated).  Result order: distance ascending, then id ascending.
 *
 * Work split: threads take blocks of QB queries; for each block the rows are
 * walked in blocks of RB rows (RB rows x dim fp32 stay in L2) with a 4 x 4
 * register tile of dot products, so each row is read from memory once per
 * query block, not once per query.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QB 64
#define RB 512
#define MAXK 256

typedef float v8f __attribute__((vector_size(32)));

typedef struct {
  const float* base;
  const float* bnorm;
  const float* queries;
  uint64_t n, nq;
  uint32_t dim, k;
  int metric;
  int32_t* out_idx;
  float* out_dist;
  uint64_t next;           /* next query block (shared, atomic) */
} bf_job;

/* Insert (d, id) into a sorted top-k list of length *len (capacity k). */
static inline void topk_insert(float* td, int32_t* ti, uint32_t* len, uint32_t k, float d,
                               int32_t id) {
  uint32_t m = *len;
  if (m == k) {
    if (d > td[k - 1] || (d == td[k - 1] && id > ti[k - 1])) return;
    m = k - 1;
  }
  uint32_t p = m;
  while (p > 0 && (td[p - 1] > d || (td[p - 1] == d && ti[p - 1] > id))) {
    td[p] = td[p - 1];
    ti[p] = ti[p - 1];
    p--;
  }
  td[p] = d;
  ti[p] = id;
  if (*len < k) (*len)++;
}

/* out[a][r] = <q_a, row_r> for a < nqb, r < nrb: 4 queries x 4 rows per
 * register tile (8 loads feed 16 multiply-adds), the dim loop vectorised. */
__attribute__((target_clones("arch=x86-64-v4", "arch=x86-64-v3", "default")))
static void dots_tile(const float* q, uint32_t nqb, const float* rows, uint32_t nrb, uint32_t dim,
                      float* out /* [QB][RB] */) {
  for (uint32_t r = 0; r < nrb; r += 4) {
    const uint32_t nr = nrb - r < 4 ? nrb - r : 4;
    const float* x0 = rows + (size_t)r * dim;
    const float* x1 = nr > 1 ? x0 + dim : x0;
    const float* x2 = nr > 2 ? x0 + 2 * dim : x0;
    const float* x3 = nr > 3 ? x0 + 3 * dim : x0;
    for (uint32_t a = 0; a < nqb; a += 4) {
      const uint32_t na = nqb - a < 4 ? nqb - a : 4;
      const float* q0 = q + (size_t)a * dim;
      const float* q1 = na > 1 ? q0 + dim : q0;
      const float* q2 = na > 2 ? q0 + 2 * dim : q0;
      const float* q3 = na > 3 ? q0 + 3 * dim : q0;
      float s[4][4];
      if ((dim & 7) == 0) {
        /* 8-wide vector chains, one per (query, row) pair */
        v8f acc[4][4];
        for (int i = 0; i < 4; i++)
          for (int t = 0; t < 4; t++) acc[i][t] = (v8f){0};
        for (uint32_t j = 0; j < dim; j += 8) {
          v8f u0, u1, u2, u3, w0, w1, w2, w3;
          memcpy(&u0, x0 + j, 32); memcpy(&u1, x1 + j, 32);
          memcpy(&u2, x2 + j, 32); memcpy(&u3, x3 + j, 32);
          memcpy(&w0, q0 + j, 32); memcpy(&w1, q1 + j, 32);
          memcpy(&w2, q2 + j, 32); memcpy(&w3, q3 + j, 32);
          acc[0][0] += w0 * u0; acc[0][1] += w0 * u1; acc[0][2] += w0 * u2; acc[0][3] += w0 * u3;
          acc[1][0] += w1 * u0; acc[1][1] += w1 * u1; acc[1][2] += w1 * u2; acc[1][3] += w1 * u3;
          acc[2][0] += w2 * u0; acc[2][1] += w2 * u1; acc[2][2] += w2 * u2; acc[2][3] += w2 * u3;
          acc[3][0] += w3 * u0; acc[3][1] += w3 * u1; acc[3][2] += w3 * u2; acc[3][3] += w3 * u3;
        }
        for (int i = 0; i < 4; i++)
          for (int t = 0; t < 4; t++) {
            const v8f v = acc[i][t];
            s[i][t] = ((v[0] + v[4]) + (v[1] + v[5])) + ((v[2] + v[6]) + (v[3] + v[7]));
          }
      } else {
        for (int i = 0; i < 4; i++)
          for (int t = 0; t < 4; t++) s[i][t] = 0.f;
        const float* qq[4] = {q0, q1, q2, q3};
        const float* xx[4] = {x0, x1, x2, x3};
        for (uint32_t j = 0; j < dim; j++)
          for (int i = 0; i < 4; i++)
            for (int t = 0; t < 4; t++) s[i][t] += qq[i][j] * xx[t][j];
      }
      for (uint32_t i = 0; i < na; i++)
        for (uint32_t t = 0; t < nr; t++) out[(size_t)(a + i) * RB + r + t] = s[i][t];
    }
  }
}

static void* bf_worker(void* arg) {
  bf_job* J = (bf_job*)arg;
  float* dots = (float*)malloc(sizeof(float) * QB * RB);
  float td[QB][MAXK];
  int32_t ti[QB][MAXK];
  uint32_t len[QB];
  for (;;) {
    const uint64_t q0 = __atomic_fetch_add(&J->next, QB, __ATOMIC_RELAXED);
    if (q0 >= J->nq) break;
    const uint32_t nqb = (uint32_t)(J->nq - q0 < QB ? J->nq - q0 : QB);
    const float* q = J->queries + q0 * J->dim;
    float qn[QB];
    for (uint32_t a = 0; a < nqb; a++) {
      float s = 0.f;
      for (uint32_t j = 0; j < J->dim; j++) s += q[(size_t)a * J->dim + j] * q[(size_t)a * J->dim + j];
      qn[a] = s;
      len[a] = 0;
    }
    for (uint64_t r0 = 0; r0 < J->n; r0 += RB) {
      const uint32_t nrb = (uint32_t)(J->n - r0 < RB ? J->n - r0 : RB);
      dots_tile(q, nqb, J->base + r0 * J->dim, nrb, J->dim, dots);
      for (uint32_t a = 0; a < nqb; a++) {
        const float* o = dots + (size_t)a * RB;
        for (uint32_t r = 0; r < nrb; r++) {
          const float d = J->metric == 0 ? qn[a] + J->bnorm[r0 + r] - 2.f * o[r] : -o[r];
          if (len[a] < J->k || d <= td[a][J->k - 1])
            topk_insert(td[a], ti[a], &len[a], J->k, d, (int32_t)(r0 + r));
        }
      }
    }
    for (uint32_t a = 0; a < nqb; a++)
      for (uint32_t i = 0; i < J->k; i++) {
        J->out_idx[(q0 + a) * J->k + i] = i < len[a] ? ti[a][i] : -1;
        J->out_dist[(q0 + a) * J->k + i] = i < len[a] ? td[a][i] : INFINITY;
      }
  }
  free(dots);
  return NULL;
}

/* base [n][dim] fp32, queries [nq][dim] fp32; metric 0 = L2, 1 = inner
 * product; k <= 256; nthreads >= 1.  Returns 0, or -1 on bad arguments. */
int orc_bruteforce_knn(const float* base, uint64_t n, const float* queries, uint64_t nq,
                       uint32_t dim, uint32_t k, int metric, int nthreads, int32_t* out_idx,
                       float* out_dist) {
  if (k == 0 || k > MAXK || nthreads < 1 || dim == 0) return -1;
  float* bnorm = (float*)malloc(sizeof(float) * (n ? n : 1));
  for (uint64_t i = 0; i < n; i++) {
    float s = 0.f;
    for (uint32_t j = 0; j < dim; j++) s += base[i * dim + j] * base[i * dim + j];
    bnorm[i] = s;
  }
  bf_job J = {base, bnorm, queries, n, nq, dim, k, metric, out_idx, out_dist, 0};
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
  for (int t = 0; t < nthreads; t++) pthread_create(&th[t], NULL, bf_worker, &J);
  for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
  free(th);
  free(bnorm);
  return 0;
}
