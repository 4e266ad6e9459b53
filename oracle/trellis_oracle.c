/*
 * CPU oracle for the EXL3 trellis encoder — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference encoder's algorithm, used by the
 * tests, by __graft_entry__.smoke() and by bench.py's CPU baseline as the
 * checker. Nothing in the product path links or calls it.
 *
 * Followed, function by function (paths inside alpha2beta/EXL3_Intel_Arc_quantizer):
 *   codebook      exl3_quant/trellis_format.py:41-81   (codebook_lut)
 *   forward       exl3_quant/reference_encoder.py:130-204
 *   argmin        exl3_quant/reference_encoder.py:206-214
 *   backward      exl3_quant/reference_encoder.py:216-251
 *   encode_tile   exl3_quant/reference_encoder.py:253-324
 *   pack          exl3_quant/trellis_format.py:120-174 (pack_trellis + swap16_storage)
 *
 * fp16 semantics: every fp16 result is the exact real result rounded once to
 * binary16 (round to nearest, ties to even). Differences and products of
 * binary16 values are exact in binary64, and the binary64 sum d*d + c is
 * either exact or cannot land on a binary16 rounding boundary, so computing
 * in double and rounding once equals a fused fp16 multiply-add.
 *
 * Build: see oracle/Makefile (gcc -O2 -pthread -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>
#include <stdatomic.h>

#define H_INF 0x7C00u

/* binary16 bits -> double (exact). */
static double h2d(uint16_t h) {
  const int s = (h >> 15) & 1, e = (h >> 10) & 0x1F, m = h & 0x3FF;
  double v;
  if (e == 0) v = ldexp((double)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = ldexp((double)(m | 0x400), e - 25);
  return s ? -v : v;
}

/* double -> binary16 bits, round to nearest, ties to even. */
static uint16_t d2h(double x) {
  uint64_t b;
  memcpy(&b, &x, 8);
  const uint16_t s = (uint16_t)((b >> 48) & 0x8000u);
  const uint64_t a = b & 0x7FFFFFFFFFFFFFFFull;
  /* Normal binary16 range [2^-14, 2^16): round the 52-bit fraction to 10 bits
   * (ties to even) with one add; a carry out of the fraction bumps the
   * exponent, and 2^16 lands on the +inf encoding. */
  if (a >= 0x3F10000000000000ull && a < 0x40F0000000000000ull) {
    const uint64_t r = a + ((1ull << 41) - 1) + ((a >> 42) & 1);
    return (uint16_t)(s | ((r >> 42) - (1008ull << 10)));
  }
  if (a >= 0x7FF0000000000000ull) return (uint16_t)(s | (a > 0x7FF0000000000000ull ? 0x7E00u : 0x7C00u));
  if (a == 0) return s;
  const int e = (int)(a >> 52) - 1023; /* unbiased exponent; doubles here are normal */
  const uint64_t m = (a & ((1ull << 52) - 1)) | (1ull << 52);
  if (e > 15) return (uint16_t)(s | 0x7C00u);
  int shift; /* bits of m dropped */
  int ee;    /* biased half exponent for the normal case */
  if (e >= -14) {
    shift = 42;
    ee = e + 15;
  } else {
    /* subnormal: units of 2^-24; value = m * 2^(e-52) */
    shift = 52 - (e + 24);
    if (shift > 63) return s;
    ee = 0;
  }
  uint64_t q = m >> shift;
  const uint64_t rem = m & ((1ull << shift) - 1), half = 1ull << (shift - 1);
  if (rem > half || (rem == half && (q & 1))) q++;
  if (ee == 0) return (uint16_t)(s | q); /* q <= 1024; 1024 is the smallest normal */
  if (q == 2048) {
    q = 1024;
    ee++;
  }
  if (ee >= 31) return (uint16_t)(s | 0x7C00u);
  return (uint16_t)(s | (ee << 10) | (q - 1024));
}

/* binary16 -> double for all 65536 bit patterns, filled once. */
static double g_h2d[65536];
static pthread_once_t g_h2d_once = PTHREAD_ONCE_INIT;
static void h2d_table_init(void) {
  for (uint32_t i = 0; i < 65536; ++i) g_h2d[i] = h2d((uint16_t)i);
}
static inline double H(uint16_t h) { return g_h2d[h]; }

static int h_isnan(uint16_t h) { return (h & 0x7C00u) == 0x7C00u && (h & 0x3FFu); }
static int h_isfinite(uint16_t h) { return (h & 0x7C00u) != 0x7C00u; }

/* strict a < b on binary16 values (false if either is NaN) */
static int h_lt(uint16_t a, uint16_t b) { return H(a) < H(b); }

uint16_t ora_f32_to_h(float f) { return d2h((double)f); }
double ora_h_to_d(uint16_t h) { return h2d(h); }
uint16_t ora_d_to_h(double d) { return d2h(d); }

void ora_codebook(int cb, uint16_t* lut) {
  for (uint32_t s = 0; s < 65536; ++s) {
    if (cb == 2) {
      const uint32_t x = s * 0x83DCD12Du;
      const uint32_t bsum = (x & 0xFF) + ((x >> 8) & 0xFF) + ((x >> 16) & 0xFF) + (x >> 24);
      const double h = (double)(1024 + bsum);
      lut[s] = d2h(h * h2d(0x1EEE) + h2d(0xC931));
    } else {
      uint32_t x = (cb == 0) ? (s * 89226354u + 64248484u) : (s * 0xCBAC1FEDu);
      x = (x & 0x8FFF8FFFu) ^ 0x3B603B60u;
      lut[s] = d2h(h2d((uint16_t)(x & 0xFFFF)) + h2d((uint16_t)(x >> 16)));
    }
  }
}

/*
 * Forward ACS pass over a ring of L fp16 weights rotated by `roll`.
 * pre_state >= 0 masks, at step 0 only, every branch whose predecessor is not
 * pre_state to +inf. edges (L x S, indexed by ring position) may be NULL.
 * costs receives the S final costs.
 */
void ora_forward(const uint16_t* w, int L, int K, const uint16_t* lut, int roll, int pre_state,
                 uint16_t* edges, uint16_t* costs) {
  const int S = 65536 >> K, Q = 1 << K, Kr = 16 - K;
  pthread_once(&g_h2d_once, h2d_table_init);
  uint16_t* prev = (uint16_t*)malloc(sizeof(uint16_t) * S);
  uint16_t* cur = (uint16_t*)malloc(sizeof(uint16_t) * S);
  for (int i = 0; i < L; ++i) {
    int ri = i + roll;
    if (ri >= L) ri -= L;
    const double wi = H(w[ri]);
    for (int e = 0; e < S; ++e) {
      uint16_t best = H_INF, bpred = 0;
      for (int k = 0; k < Q; ++k) {
        const uint32_t st = ((uint32_t)k << Kr) | (uint32_t)e;
        const uint16_t pred = (uint16_t)(st >> K);
        const double dh = H(d2h(H(lut[st]) - wi));
        uint16_t err;
        if (i == 0) {
          err = d2h(dh * dh);
          if (pre_state >= 0 && (int)pred != pre_state) err = H_INF;
        } else {
          err = d2h(dh * dh + H(prev[pred]));
        }
        if (k == 0 || h_lt(err, best)) {
          best = err;
          bpred = pred;
        }
      }
      cur[e] = best;
      if (edges) edges[(size_t)ri * S + e] = bpred;
    }
    uint16_t* t = prev;
    prev = cur;
    cur = t;
  }
  memcpy(costs, prev, sizeof(uint16_t) * S);
  free(prev);
  free(cur);
}

/* numpy-semantics argmin: 0 if no finite cost or all +inf; else the first
 * NaN if any, else the first minimum. */
int ora_argmin(const uint16_t* c, int S) {
  pthread_once(&g_h2d_once, h2d_table_init);
  int any_finite = 0, all_inf = 1, first_nan = -1, best = -1;
  for (int e = 0; e < S; ++e) {
    if (h_isfinite(c[e])) any_finite = 1;
    if (c[e] != H_INF) all_inf = 0;
    if (h_isnan(c[e]) && first_nan < 0) first_nan = e;
  }
  if (!any_finite || all_inf) return 0;
  if (first_nan >= 0) return first_nan;
  for (int e = 0; e < S; ++e)
    if (best < 0 || h_lt(c[e], c[best])) best = e;
  return best;
}

/* pack_trellis (16 spans x 16 elements, low K bits MSB-first) + SWAP16. */
void ora_pack(const uint16_t* states, int K, uint16_t* out) {
  const int n16 = 16 * K;
  uint16_t tmp[128];
  for (int t = 0; t < 16; ++t) {
    int j = K * t, k = 32;
    uint32_t buf = 0;
    for (int i = 16 * t; i < 16 * t + 16; ++i) {
      const uint32_t v = states[i] & ((1u << K) - 1u);
      k -= K;
      buf |= v << k;
      if (k <= 16) {
        tmp[j++] = (uint16_t)(buf >> 16);
        buf <<= 16;
        k += 16;
      }
    }
  }
  for (int m = 0; m < n16; m += 2) {
    out[m] = tmp[m + 1];
    out[m + 1] = tmp[m];
  }
}

/*
 * Full two-pass tail-biting encode of one tile whose elements are already in
 * encoder order (pre_permute = False in the reference).
 * Outputs: idx[L] states, recon[L] fp16 bits, end_state, path cost fp16 bits,
 * packed[16K] (only when L == 256 and packed != NULL).
 */
void ora_encode_tile(const float* tile, int L, int K, const uint16_t* lut, uint16_t* idx,
                     uint16_t* recon, int32_t* end_state, uint16_t* path_cost,
                     uint16_t* packed) {
  const int S = 65536 >> K;
  uint16_t* w = (uint16_t*)calloc((size_t)L, sizeof(uint16_t));
  uint16_t* edges = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)L * S);
  uint16_t* costs = (uint16_t*)malloc(sizeof(uint16_t) * S);
  for (int i = 0; i < L; ++i) w[i] = d2h((double)tile[i]);

  ora_forward(w, L, K, lut, L / 2, -1, edges, costs);
  int edge = ora_argmin(costs, S);
  for (int i = L - 1; i >= 0; --i) {
    int ri = i + L / 2;
    if (ri >= L) ri -= L;
    edge = edges[(size_t)ri * S + edge];
    if (ri == 0) break;
  }
  const int es = edge;
  ora_forward(w, L, K, lut, 0, es, edges, costs);
  edge = es;
  for (int i = L - 1; i >= 0; --i) {
    const int prev = edges[(size_t)i * S + edge];
    const uint16_t st = (uint16_t)((prev << K) | edge);
    edge = prev;
    idx[i] = st;
    recon[i] = lut[st];
  }
  *end_state = es;
  *path_cost = costs[es];
  if (packed && L == 256) ora_pack(idx, K, packed);
  free(w);
  free(edges);
  free(costs);
}

/* Batch encode, tiles distributed dynamically over `threads` POSIX threads
 * (threads <= 0: one). Returns the thread count used. */
typedef struct {
  const float* tiles;
  int64_t n;
  int L, K;
  const uint16_t* lut;
  uint16_t *idx, *recon, *path_cost, *packed;
  int32_t* end_state;
  atomic_llong next;
} batch_job;

static void* batch_worker(void* arg) {
  batch_job* j = (batch_job*)arg;
  for (;;) {
    const int64_t t = atomic_fetch_add(&j->next, 1);
    if (t >= j->n) break;
    ora_encode_tile(j->tiles + t * j->L, j->L, j->K, j->lut, j->idx + t * j->L,
                    j->recon + t * j->L, j->end_state + t, j->path_cost + t,
                    j->packed ? j->packed + t * 16 * j->K : NULL);
  }
  return NULL;
}

int ora_encode_batch(const float* tiles, int64_t n, int L, int K, int cb, uint16_t* idx,
                     uint16_t* recon, int32_t* end_state, uint16_t* path_cost,
                     uint16_t* packed, int threads) {
  uint16_t* lut = (uint16_t*)malloc(sizeof(uint16_t) * 65536);
  ora_codebook(cb, lut);
  if (threads < 1) threads = 1;
  if (threads > 1024) threads = 1024;
  batch_job job = {tiles, n, L, K, lut, idx, recon, path_cost, packed, end_state, 0};
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * threads);
  int started = 0;
  for (int i = 1; i < threads; ++i)
    if (pthread_create(&th[started], NULL, batch_worker, &job) == 0) started++;
  batch_worker(&job);
  for (int i = 0; i < started; ++i) pthread_join(th[i], NULL);
  free(th);
  free(lut);
  return started + 1;
}
