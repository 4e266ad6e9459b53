/*
 * CPU oracle for the LDLQ loop's floating-point arithmetic — TEST
 * INFRASTRUCTURE ONLY (tests/ and bench.py's CPU legs; never linked by the
 * product).
 *
 * The reference loop (exl3_quant/ldlq.py:163-309) is, per span of `buf` rows
 * (bottom-up) and 16-row block (bottom-up):
 *   comp  = prod_cache[blk] + L[below, blk]^T (W - W_q)[below]    (addmm_)
 *   rows  = W[blk] + comp
 *   tiles = rows cut into 16x16 tiles, tensor-core order   -> encoder
 * and after each span
 *   prod_cache += L[span]^T (W - W_q)[span]                       (addmm_)
 * The reference leaves the summation order of its two products to the BLAS
 * of the device it runs on. This restatement fixes one order, the one the
 * device loop uses: every output is a sequential fmaf chain from 0 over the
 * contracted rows in ascending order, added once to the cached product. With
 * the same encoder the device loop then agrees bit for bit.
 *
 * Compiled with -ffp-contract=off: the only fused operations are the
 * explicit fmaf calls.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <unistd.h>

#define EXPORT __attribute__((visibility("default")))

/* Runs fn(arg, i0, i1) over [0, n) split into one contiguous range per host
 * thread; each output is computed by exactly one thread, so the split does
 * not change any result. */
typedef void (*range_fn)(void* arg, int64_t i0, int64_t i1);
typedef struct {
  range_fn fn;
  void* arg;
  int64_t i0, i1;
} range_job;

static void* range_run(void* p) {
  range_job* j = (range_job*)p;
  j->fn(j->arg, j->i0, j->i1);
  return NULL;
}

static void parallel_ranges(range_fn fn, void* arg, int64_t n) {
  long nt = sysconf(_SC_NPROCESSORS_ONLN);
  if (nt < 1) nt = 1;
  if (nt > 256) nt = 256;
  if (nt > n) nt = (long)(n > 0 ? n : 1);
  pthread_t th[256];
  range_job jobs[256];
  for (long t = 0; t < nt; ++t) {
    jobs[t].fn = fn;
    jobs[t].arg = arg;
    jobs[t].i0 = n * t / nt;
    jobs[t].i1 = n * (t + 1) / nt;
  }
  for (long t = 1; t < nt; ++t) pthread_create(&th[t], NULL, range_run, &jobs[t]);
  range_run(&jobs[0]);
  for (long t = 1; t < nt; ++t) pthread_join(th[t], NULL);
}

/*
 * One block's encoder input.
 *   W, Wq, prod: (k, n) row-major; L: (k, k) row-major.
 *   r0: first row of the block; rows [below0, below1) are the quantized rows
 *   of the same span under it.
 *   tiles: out (n/16, 256) in encoder order (perm_inv maps tile position
 *   r*16+c to the encoder position).
 */
typedef struct {
  const float *W, *Wq, *L, *prod;
  int64_t k, n, r0, below0, below1;
  const int16_t* perm_inv;
  float* tiles;
} prep_args;

static void prep_range(void* p, int64_t t0, int64_t t1) {
  const prep_args* a = (const prep_args*)p;
  const int64_t nb = a->below1 - a->below0, n = a->n;
  for (int64_t tc = t0; tc < t1; ++tc) {
    for (int r = 0; r < 16; ++r) {
      for (int c = 0; c < 16; ++c) {
        const int64_t col = tc * 16 + c;
        float acc = 0.0f;
        for (int64_t s = 0; s < nb; ++s) {
          const int64_t row = a->below0 + s;
          const float e = a->W[row * n + col] - a->Wq[row * n + col];
          acc = fmaf(a->L[row * a->k + a->r0 + r], e, acc);
        }
        const int64_t off = (a->r0 + r) * n + col;
        const float comp = a->prod[off] + acc;
        a->tiles[tc * 256 + a->perm_inv[r * 16 + c]] = a->W[off] + comp;
      }
    }
  }
}

EXPORT void ldlq_oracle_prep(const float* W, const float* Wq, const float* L, const float* prod,
                             int64_t k, int64_t n, int64_t r0, int64_t below0, int64_t below1,
                             const int16_t* perm_inv, float* tiles) {
  prep_args a = {W, Wq, L, prod, k, n, r0, below0, below1, perm_inv, tiles};
  parallel_ranges(prep_range, &a, n / 16);
}

/*
 * Trailing update after the span [span0, span0 + span_rows):
 *   prod[rr, :] += sum_s L[span0 + s, rr] * (W - Wq)[span0 + s, :]
 * for rr < rows_above, the sum a sequential fmaf chain over ascending s.
 */
typedef struct {
  const float *E, *L;
  float* prod;
  int64_t k, n, span0, span_rows;
} span_args;

__attribute__((target_clones("arch=x86-64-v3", "default")))
static void span_range(void* p, int64_t r0, int64_t r1) {
  const span_args* a = (const span_args*)p;
  const int64_t n = a->n;
  float* acc = (float*)malloc(sizeof(float) * (size_t)n);
  for (int64_t rr = r0; rr < r1; ++rr) {
    for (int64_t c = 0; c < n; ++c) acc[c] = 0.0f;
    for (int64_t s = 0; s < a->span_rows; ++s) {
      const float l = a->L[(a->span0 + s) * a->k + rr];
      const float* e = a->E + s * n;
      for (int64_t c = 0; c < n; ++c) acc[c] = fmaf(l, e[c], acc[c]);
    }
    float* q = a->prod + rr * n;
    for (int64_t c = 0; c < n; ++c) q[c] = q[c] + acc[c];
  }
  free(acc);
}

EXPORT void ldlq_oracle_span(const float* W, const float* Wq, const float* L, float* prod,
                             int64_t k, int64_t n, int64_t span0, int64_t span_rows,
                             int64_t rows_above) {
  float* E = (float*)malloc(sizeof(float) * (size_t)(span_rows * n));
  for (int64_t s = 0; s < span_rows; ++s)
    for (int64_t c = 0; c < n; ++c) {
      const int64_t off = (span0 + s) * n + c;
      E[s * n + c] = W[off] - Wq[off];
    }
  span_args a = {E, L, prod, k, n, span0, span_rows};
  parallel_ranges(span_range, &a, rows_above);
  free(E);
}
