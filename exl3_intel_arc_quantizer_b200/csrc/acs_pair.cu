// Tile-pair ACS encoder (K = 2..8): two tiles share one CTA, one per fp16
// half2 lane, with cost-vector checkpoints instead of per-step backpointers.
//
// Both tiles walk the same trellis, so a candidate's codebook value is one
// scalar shared by the two lanes; everything per-tile (weight, accumulated
// cost) is a lane of one 32-bit register:
//   * the cost vector is stored as {cost_A, cost_B} words in natural edge
//     order: a predecessor cost is read as one word that already holds both
//     lanes, and a result is written as one word;
//   * threads take edges chunk-major (consecutive threads own consecutive
//     chunks) so a warp's shared-memory stores are contiguous.
//
// Forward passes only compute minima (sub, fma on the fp16 FMA pipe, one
// min on the ALU pipe per candidate): recording which branch won costs a
// compare and a select per candidate on the ALU pipe, which bounded the
// earlier tracked steps. Instead, the cost vector of every R-th step is also
// copied to HBM as a checkpoint (R = 2 at K=2, every step above) by one bulk
// copy from shared memory (ck_issue), which costs the warps nothing. The traceback walks the
// path back from its end, recomputing from the nearest checkpoint only the
// costs of the path's ancestors (Q^R loads and Q^R candidate evaluations per
// R steps) with the same fp16 operations and the same first-minimum rule, so
// the branches it finds are the ones a tracked forward pass would record.
//
// The arithmetic, tie-breaking and NaN behaviour are those of encoder.cu
// (reference_encoder.py:130-324): strict < over ascending k, a NaN at k=0
// sticks, later NaNs never win; a tile pair with a NaN input runs
// compare-and-select instead of min for its costs.
#include "common.cuh"
#include "encoder_shared.cuh"

namespace exl3 {

template <int K>
struct PGeo {
  static constexpr int S = 1 << (16 - K);
  static constexpr int Kr = 16 - K;
  static constexpr int GB = 16 - 2 * K;
  static constexpr int Q = 1 << K;
  static constexpr bool SPLIT = (K == 8);              // two lanes per edge
  static constexpr int E = SPLIT ? 1 : S / kPairNT;     // edges per thread
  static constexpr int QT = SPLIT ? Q / 2 : Q;          // branches per thread
  static constexpr int CE = SPLIT ? 1 : (E < 8 ? E : 8);  // edges per chunk
  static constexpr int NCH = E / CE;                    // chunks per step
  static constexpr int NGC = SPLIT ? 1 : (((CE >> K) > 0) ? (CE >> K) : 1);
  static constexpr int KB = QT < 8 ? QT : 8;            // branches per load batch
  static constexpr int R = ck_stride(K);               // checkpoint stride
  static constexpr int CKB = S * 4;                     // bytes per pair checkpoint
  static_assert(E * QT == 128, "codebook register budget: 128 values per thread");
};

// Checkpointed steps. Pass 1 (roll L/2): steps half-1, half-1+R, ... <= L-2,
// the ones the end-state traceback over [half, L) needs. Pass 2 (roll 0):
// steps R-1, 2R-1, ... <= L-2 (step -1 is the all-zero start).
__host__ __device__ constexpr int ck_slots_pass1(int K, int L) {
  return (L - L / 2 - 1) / ck_stride(K) + 1;
}
__host__ __device__ constexpr int ck_slots_pass2(int K, int L) { return (L - 1) / ck_stride(K); }

int pair_ck_bytes_per_step_slot(int K) { return (65536 >> K) * 4; }

size_t pair_ck_bytes(int K, int L) {
  const int s1 = ck_slots_pass1(K, L), s2 = ck_slots_pass2(K, L);
  const size_t b = (size_t)(s1 > s2 ? s1 : s2) * (size_t)pair_ck_bytes_per_step_slot(K);
  return (b + 255) / 256 * 256;
}

size_t pair_tile_ws_bytes(int K, int L) { return pair_ck_bytes(K, L) / 2 + 8; }

// Global edge of the thread's local edge le (chunk-major mapping).
template <int K>
__host__ __device__ __forceinline__ int pair_edge_of(int t, int le) {
  using G = PGeo<K>;
  if constexpr (G::SPLIT) {
    return t >> 1;
  } else {
    const int c = le / G::CE, j = le % G::CE;
    return (c * kPairNT + t) * G::CE + j;
  }
}

// 128 codebook values per thread, two per register: candidate
// m = le * QT + kk sits in lane (m & 1) of cbv[m >> 1].
template <int K>
__device__ __forceinline__ void pair_init_codebook(uint32_t (&cbv)[64], int cb, int t) {
  using G = PGeo<K>;
#pragma unroll
  for (int le = 0; le < G::E; ++le) {
    const uint32_t e = (uint32_t)pair_edge_of<K>(t, le);
#pragma unroll
    for (int kk = 0; kk < G::QT; kk += 2) {
      const uint32_t k = (G::SPLIT ? (uint32_t)((t & 1) * G::QT) : 0u) + kk;
      const uint32_t s0 = (k << G::Kr) | e, s1 = ((k + 1) << G::Kr) | e;
      cbv[(le * G::QT + kk) >> 1] = (uint32_t)cb_state_bits(cb, s0) |
                                    ((uint32_t)cb_state_bits(cb, s1) << 16);
    }
  }
}

// One ACS step over both lanes.
//   FIRST : step 0; pre2 = {pre_A, pre_B} wrap constraint (-1 = none)
//   EXACT : compare-and-select for the cost (NaN-faithful) instead of min
template <int K, bool FIRST, bool EXACT>
__device__ __forceinline__ void pair_step(const uint32_t (&cbv)[64], uint32_t w2,
                                          const uint32_t* __restrict__ cin,
                                          uint32_t* __restrict__ cout, int t, int preA,
                                          int preB) {
  using G = PGeo<K>;
  if constexpr (!G::SPLIT) {
#pragma unroll
    for (int c = 0; c < G::NCH; ++c) {
      const int e0 = (c * kPairNT + t) * G::CE;
      const int g0 = e0 >> K;
      uint32_t best[G::CE];
#pragma unroll
      for (int kb = 0; kb < G::QT; kb += G::KB) {
        uint32_t P[G::KB][G::NGC];
        if constexpr (!FIRST) {
#pragma unroll
          for (int q = 0; q < G::KB; ++q) {
            const uint32_t* src = cin + ((kb + q) << G::GB) + g0;
            if constexpr (G::NGC == 2) {
              const uint2 v = *reinterpret_cast<const uint2*>(src);
              P[q][0] = v.x;
              P[q][1] = v.y;
            } else {
              P[q][0] = *src;
            }
          }
        }
#pragma unroll
        for (int j = 0; j < G::CE; ++j) {
          const int le = c * G::CE + j;
          const int gi = (G::NGC > 1) ? (j >> K) : 0;
#pragma unroll
          for (int q = 0; q < G::KB; ++q) {
            const int k = kb + q;
            const int m = le * G::QT + k;
            const uint32_t d = (m & 1) ? h2_sub_bcast<true>(cbv[m >> 1], w2)
                                       : h2_sub_bcast<false>(cbv[m >> 1], w2);
            uint32_t cst = h2_fma(d, d, FIRST ? 0u : P[q][gi]);
            if constexpr (FIRST) {
              const int pred = (k << G::GB) | ((e0 + j) >> K);
              const uint32_t keep = (pred == preA ? 0x0000FFFFu : 0u) |
                                    (pred == preB ? 0xFFFF0000u : 0u);
              if (preA >= 0 || preB >= 0) {
                const uint32_t allow = keep | (preA < 0 ? 0x0000FFFFu : 0u) |
                                       (preB < 0 ? 0xFFFF0000u : 0u);
                cst = bsel(allow, cst, kHInf2);
              }
            }
            if (k == 0) {
              best[j] = cst;
            } else if constexpr (EXACT) {
              best[j] = bsel(h2_lt_mask(cst, best[j]), cst, best[j]);
            } else {
              best[j] = h2_min(best[j], cst);
            }
          }
        }
      }
      // results: CE words at edges [e0, e0 + CE)
      uint32_t* dst = cout + e0;
      if constexpr (G::CE % 4 == 0) {
#pragma unroll
        for (int q = 0; q < G::CE / 4; ++q)
          reinterpret_cast<uint4*>(dst)[q] =
              make_uint4(best[4 * q], best[4 * q + 1], best[4 * q + 2], best[4 * q + 3]);
      } else if constexpr (G::CE == 2) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(best[0], best[1]);
      } else {
        dst[0] = best[0];
      }
    }
  } else {
    // K = 8: lanes t and t^1 split the 256 branches of edge t >> 1.
    const int e = t >> 1, r = t & 1;
    const int k0 = r * G::QT;
    uint32_t best = kHInf2;
#pragma unroll
    for (int kb = 0; kb < G::QT; kb += 8) {
      uint32_t P[8];
      if constexpr (!FIRST) {
        const uint4 v0 = *reinterpret_cast<const uint4*>(cin + k0 + kb);
        const uint4 v1 = *reinterpret_cast<const uint4*>(cin + k0 + kb + 4);
        P[0] = v0.x; P[1] = v0.y; P[2] = v0.z; P[3] = v0.w;
        P[4] = v1.x; P[5] = v1.y; P[6] = v1.z; P[7] = v1.w;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int kk = kb + q, k = k0 + kk;
        const uint32_t d = (kk & 1) ? h2_sub_bcast<true>(cbv[kk >> 1], w2)
                                    : h2_sub_bcast<false>(cbv[kk >> 1], w2);
        uint32_t cst = h2_fma(d, d, FIRST ? 0u : P[q]);
        if constexpr (FIRST) {
          if (preA >= 0 || preB >= 0) {
            const uint32_t allow = ((k == preA || preA < 0) ? 0x0000FFFFu : 0u) |
                                   ((k == preB || preB < 0) ? 0xFFFF0000u : 0u);
            cst = bsel(allow, cst, kHInf2);
          }
        }
        if (kk == 0) {
          // the lower range starts from its k = 0 candidate (a NaN there
          // sticks); the upper range starts from +inf and skips NaNs
          const uint32_t msk = h2_lt_mask(cst, best) | (r == 0 ? 0xFFFFFFFFu : 0u);
          best = bsel(msk, cst, best);
        } else if constexpr (EXACT) {
          best = bsel(h2_lt_mask(cst, best), cst, best);
        } else {
          best = h2_min(best, cst);
        }
      }
    }
    // lower branch range (r = 0) wins ties
    const uint32_t ob = __shfl_xor_sync(0xFFFFFFFFu, best, 1);
    const uint32_t lo_c = r ? ob : best, hi_c = r ? best : ob;
    if (r == 0) cout[e] = bsel(h2_lt_mask(hi_c, lo_c), hi_c, lo_c);
  }
}

template <int K>
struct PSmem {
  static constexpr size_t costs = 2ull * PGeo<K>::S * sizeof(uint32_t);
  static constexpr size_t bytes = costs + 256 * sizeof(uint32_t);
};

// Both tiles of pair `tp` into {w_A, w_B} words; returns nonzero if either
// holds a NaN. A missing B tile (odd count) repeats A.
__device__ __forceinline__ int pair_load(const float* __restrict__ in, int n, int L, int tp,
                                         uint32_t* wt, int t) {
  const int ta = 2 * tp, tb = (2 * tp + 1 < n) ? 2 * tp + 1 : 2 * tp;
  int nan = 0;
  for (int i = t; i < L; i += kPairNT) {
    const __half a = __float2half_rn(in[(size_t)ta * L + i]);
    const __half b = __float2half_rn(in[(size_t)tb * L + i]);
    nan |= (__hisnan(a) || __hisnan(b)) ? 1 : 0;
    wt[i] = (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
  }
  return __syncthreads_or(nan);
}

// Per-lane argmin of the final costs (minimum, lowest edge on ties,
// non-finite skipped, none finite -> 0).
template <int K>
__device__ __forceinline__ void pair_argmin(const uint32_t* costs, uint32_t* red, int t,
                                            int* outA, int* outB) {
  using G = PGeo<K>;
  uint32_t ka = 0xFFFFFFFFu, kb = 0xFFFFFFFFu;
  for (int e = t; e < G::S; e += kPairNT) {
    const uint32_t w = costs[e];
    const uint32_t a = w & 0xFFFFu, b = w >> 16;
    if ((a & 0x7C00u) != 0x7C00u) ka = min(ka, (a << 16) | (uint32_t)e);
    if ((b & 0x7C00u) != 0x7C00u) kb = min(kb, (b << 16) | (uint32_t)e);
  }
  ka = __reduce_min_sync(0xFFFFFFFFu, ka);
  kb = __reduce_min_sync(0xFFFFFFFFu, kb);
  if ((t & 31) == 0) {
    red[t >> 5] = ka;
    red[32 + (t >> 5)] = kb;
  }
  __syncthreads();
  if (t < 32) {
    uint32_t va = (t < kPairNT / 32) ? red[t] : 0xFFFFFFFFu;
    uint32_t vb = (t < kPairNT / 32) ? red[32 + t] : 0xFFFFFFFFu;
    va = __reduce_min_sync(0xFFFFFFFFu, va);
    vb = __reduce_min_sync(0xFFFFFFFFu, vb);
    if (t == 0) {
      red[0] = va;
      red[32] = vb;
    }
  }
  __syncthreads();
  const uint32_t va = red[0], vb = red[32];
  __syncthreads();
  *outA = va == 0xFFFFFFFFu ? 0 : (int)(va & 0xFFFFu);
  *outB = vb == 0xFFFFFFFFu ? 0 : (int)(vb & 0xFFFFu);
}

// Checkpoints leave shared memory through the bulk-copy engine: after the
// step's barrier one thread issues a single cp.async.bulk of the finished
// cost vector (S x 4 bytes, 16-byte aligned) to its HBM slot; no warp spends
// an instruction or an LSU slot on it. Writers order their shared-memory
// stores for the async proxy first (ck_fence, before the barrier). The
// buffer is rewritten two steps later, so the issuing thread waits until the
// copy has finished reading it (ck_wait_read) before the next barrier.
__device__ __forceinline__ void ck_fence() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void ck_issue(uint8_t* gdst, const uint32_t* ssrc, uint32_t bytes) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(ssrc));
  asm volatile(
      "cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n\t"
      "cp.async.bulk.commit_group;" ::"l"(gdst), "r"(s), "r"(bytes)
      : "memory");
}
__device__ __forceinline__ void ck_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void ck_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

template <int K, bool EXACT>
__device__ __forceinline__ void pair_pass1(const uint32_t (&cbv)[64], const uint32_t* wt,
                                           uint32_t* c0, uint32_t* c1, uint8_t* ckp, int L,
                                           int t) {
  using G = PGeo<K>;
  const int half = L / 2;
  pair_step<K, true, EXACT>(cbv, wt[half], nullptr, c0, t, -1, -1);
  __syncthreads();
  for (int i = 1; i < L; ++i) {
    const uint32_t* cin = (i & 1) ? c0 : c1;
    uint32_t* cout = (i & 1) ? c1 : c0;
    pair_step<K, false, EXACT>(cbv, wt[i < half ? i + half : i - half], cin, cout, t, -1, -1);
    const int rel = i - (half - 1);
    const bool ckpt = rel >= 0 && rel % G::R == 0 && i <= L - 2;
    if (ckpt) ck_fence();
    if (t == 0) ck_wait_read();  // the copy of step i-1 read the buffer step i+1 rewrites
    __syncthreads();
    if (ckpt && t == 0) ck_issue(ckp + (size_t)(rel / G::R) * G::CKB, cout, G::CKB);
  }
  if (t == 0) ck_wait_read();
}

template <int K, bool EXACT>
__device__ __forceinline__ void pair_pass2(const uint32_t (&cbv)[64], const uint32_t* wt,
                                           uint32_t* c0, uint32_t* c1, uint8_t* ckp, int L,
                                           int t, int preA, int preB) {
  using G = PGeo<K>;
  pair_step<K, true, EXACT>(cbv, wt[0], nullptr, c0, t, preA, preB);
  const bool ck0 = G::R == 1 && L >= 2;
  if (ck0) ck_fence();
  __syncthreads();
  if (ck0 && t == 0) ck_issue(ckp, c0, G::CKB);
  for (int i = 1; i < L; ++i) {
    const uint32_t* cin = (i & 1) ? c0 : c1;
    uint32_t* cout = (i & 1) ? c1 : c0;
    pair_step<K, false, EXACT>(cbv, wt[i], cin, cout, t, -1, -1);
    const bool ckpt = (i + 1) % G::R == 0 && i <= L - 2;
    if (ckpt) ck_fence();
    if (t == 0) ck_wait_read();
    __syncthreads();
    if (ckpt && t == 0) ck_issue(ckp + (size_t)((i + 1) / G::R - 1) * G::CKB, cout, G::CKB);
  }
  if (t == 0) ck_wait_read();
}

template <int K, int PASS>
__global__ void __launch_bounds__(kPairNT, 1)
acs_pair_kernel(const float* __restrict__ in, int n, int L, int cb, uint8_t* __restrict__ ck,
                size_t ck_pair_bytes, int32_t* __restrict__ best_edge,
                const int32_t* __restrict__ end_state, float* __restrict__ path_cost) {
  using G = PGeo<K>;
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* c0 = reinterpret_cast<uint32_t*>(smem);
  uint32_t* c1 = c0 + G::S;
  uint32_t* wt = reinterpret_cast<uint32_t*>(smem + PSmem<K>::costs);
  __shared__ uint32_t red[64];
  const int t = threadIdx.x;
  uint32_t cbv[64];
  pair_init_codebook<K>(cbv, cb, t);
  const int npairs = (n + 1) / 2;
  for (int tp = blockIdx.x; tp < npairs; tp += gridDim.x) {
    const int nan = pair_load(in, n, L, tp, wt, t);
    uint8_t* pck = ck + (size_t)tp * ck_pair_bytes;
    const uint32_t* fin = ((L - 1) & 1) ? c1 : c0;
    const int ta = 2 * tp, tb = 2 * tp + 1;
    if constexpr (PASS == 1) {
      if (nan) pair_pass1<K, true>(cbv, wt, c0, c1, pck, L, t);
      else     pair_pass1<K, false>(cbv, wt, c0, c1, pck, L, t);
      int ea, eb;
      pair_argmin<K>(fin, red, t, &ea, &eb);
      if (t == 0) {
        best_edge[ta] = ea;
        if (tb < n) best_edge[tb] = eb;
      }
    } else {
      const int preA = end_state[ta];
      const int preB = (tb < n) ? end_state[tb] : preA;
      if (nan) pair_pass2<K, true>(cbv, wt, c0, c1, pck, L, t, preA, preB);
      else     pair_pass2<K, false>(cbv, wt, c0, c1, pck, L, t, preA, preB);
      if (t == 0 && path_cost) {
        path_cost[ta] = half_bits_to_float((uint16_t)(fin[preA] & 0xFFFFu));
        if (tb < n) path_cost[tb] = half_bits_to_float((uint16_t)(fin[preB] >> 16));
      }
    }
    __syncthreads();
  }
  if (t == 0) ck_wait_all();
}

// ---------------------------------------------------------------------------
// Traceback from checkpoints (one warp per tile)
// ---------------------------------------------------------------------------

// Ordering key of candidate k with cost bits v under the sequential rule
// (strict < over ascending k; a NaN at k = 0 wins; later NaNs never win):
// the smallest key is the candidate a forward pass keeps. Costs are >= +0,
// so their bits order as unsigned integers.
__device__ __forceinline__ uint32_t cand_key(int k, uint16_t v) {
  const bool nan = (v & 0x7C00u) == 0x7C00u && (v & 0x03FFu) != 0u;
  if (nan) return k == 0 ? 0u : 0xFFFFFFFFu;
  return (((uint32_t)v + 1u) << 16) | (uint32_t)k;
}

// Cost of candidate k into edge x at step s. prev = predecessor's cost after
// step s-1 (0 before step 0); at step 0 of a constrained pass, a candidate
// whose predecessor is not `pre` costs +inf.
// cand_diff is the part that does not depend on prev (codebook value minus
// the weight), cand_finish the rest.
template <int K>
__device__ __forceinline__ uint16_t cand_diff(int cb, int k, int x, uint16_t w) {
  using G = PGeo<K>;
  return h_sub(cb_state_bits(cb, ((uint32_t)k << G::Kr) | (uint32_t)x), w);
}
template <int K>
__device__ __forceinline__ uint16_t cand_finish(uint16_t d, uint16_t prev, int k, int x,
                                                bool first, int pre) {
  using G = PGeo<K>;
  uint16_t c = h_fma(d, d, prev);
  if (first && pre >= 0 && (((k << G::GB) | (x >> K)) != pre)) c = 0x7C00u;
  return c;
}
template <int K>
__device__ __forceinline__ uint16_t cand_cost(int cb, int k, int x, uint16_t w, uint16_t prev,
                                              bool first, int pre) {
  return cand_finish<K>(cand_diff<K>(cb, k, x, w), prev, k, x, first, pre);
}

// The cost bits a winning key was made from (cand_key inverted). Key 0 is a
// NaN at k = 0: any NaN stands for it, since later keys see only NaN-ness.
__device__ __forceinline__ uint16_t key_cost(uint32_t key) {
  return key == 0u ? (uint16_t)0x7FFFu : (uint16_t)((key >> 16) - 1u);
}

constexpr int kSingleR = 4;  // the single-tile K=1 encoder checkpoints every 4th step
constexpr size_t kTbDeepBytes = size_t(64) << 20;  // checkpoints of a call beyond L2

// The pair walk without shared-memory levels. K >= 3 (a checkpoint every
// step, one level): lane k loads the checkpoint cost of branch k's
// predecessor and evaluates candidate k itself; its codebook value does not
// depend on the load, so it is computed while the load is in flight.
// K = 2 (a checkpoint every 2nd step; with L even every segment spans two
// steps): the Q^2 level-2 nodes (costs at the checkpoint) are spread
// over the lanes, node (kb << K) | j1 in register r of lane
// ((kb << K) | j1) & 31; each lane evaluates branch kb of level-1 node j1
// for its nodes, keeps the lowest key, and lanes holding the same j1 combine
// by xor shuffles of the keys alone (a key holds its cost bits). Step i then
// takes the minimum over branch kq = lane & (Q-1) of node kq; step i-1's
// candidates are the level-1 candidates of the node step i picked, so their
// keys are reused rather than evaluated again. The candidate costs, the ordering
// keys (cand_key) and the first-minimum rule are those of the forward pass,
// so the path is the one a tracked forward pass would record.
template <int K, int PASS, int D>
__device__ int ck_walk_reg(const uint8_t* __restrict__ pck, int b, int cb, const uint16_t* w,
                           int L, int e_top, int pre, uint16_t* st, int lane) {
  using G = PGeo<K>;
  constexpr int R = G::R;  // checkpoint stride; D = steps per segment
  constexpr int Q = G::Q;
  static_assert(D % R == 0 && (D == 1 || D == 2), "a segment spans 1 or 2 checkpoint strides");
  const int half = L / 2;
  const int i_stop = PASS == 1 ? half : 0;
  auto wt = [&](int s) { return w[PASS == 1 ? (s < half ? s + half : s - half) : s]; };
  auto cost_of = [&](const uint32_t* ckb, int x) -> uint16_t {
    return ckb ? (uint16_t)((__ldg(ckb + x) >> (16 * b)) & 0xFFFFu) : (uint16_t)0;
  };
  auto pick = [&](uint32_t bk) { return (bk == 0u || bk == 0xFFFFFFFFu) ? 0 : (int)(bk & 0xFFFFu); };
  int i = L - 1, e = e_top;
  while (i >= i_stop) {
    int c, slot;
    if (PASS == 1) {
      const int rel = ((i - 1) - (half - 1)) / D;
      c = (half - 1) + rel * D;
      slot = rel * (D / R);
    } else {
      c = (i / D) * D - 1;
      slot = (c + 1) / R - 1;
    }
    const uint32_t* ckb =
        c >= 0 ? reinterpret_cast<const uint32_t*>(pck + (size_t)slot * G::CKB) : nullptr;
    if constexpr (D == 1) {
      const uint16_t ws = wt(i);
      const bool first = PASS == 2 && i == 0;
      constexpr int NPL = (Q + 31) / 32;  // branches per lane, all loads issued first
      uint16_t prev[NPL];
#pragma unroll
      for (int r = 0; r < NPL; ++r) {
        const int k = lane + 32 * r;
        prev[r] = k < Q ? cost_of(ckb, (k << G::GB) | (e >> K)) : (uint16_t)0;
      }
      uint32_t bk = 0xFFFFFFFFu;
#pragma unroll
      for (int r = 0; r < NPL; ++r) {
        const int k = lane + 32 * r;
        if (k < Q) {
          const uint32_t key = cand_key(k, cand_cost<K>(cb, k, e, ws, prev[r], first, pre));
          bk = key < bk ? key : bk;
        }
      }
      const int k = pick(__reduce_min_sync(0xFFFFFFFFu, bk));
      if (PASS == 2 && lane == 0) st[i] = (uint16_t)((k << G::Kr) | e);
      e = (k << G::GB) | (e >> K);
    } else {
      static_assert(Q * Q <= 256, "two-level register walk: Q^2 <= 256");
      constexpr int NPL = (Q * Q + 31) / 32;  // level-2 nodes per lane
      const int s1 = i - 1;
      const uint16_t ws1 = wt(s1);
      uint16_t v2[NPL];
#pragma unroll
      for (int r = 0; r < NPL; ++r) {  // every load in flight before the candidates
        const int node = (lane + 32 * r) & (Q * Q - 1);
        v2[r] = cost_of(ckb, (node << (G::Kr - 2 * K)) | (e >> (2 * K)));
      }
      // step i, branch kq = lane & (Q-1): its difference needs no load
      const int kq = lane & (Q - 1);
      const uint16_t d0 = cand_diff<K>(cb, kq, e, wt(i));
      // level 1: node (kb << K) | j1 is branch kb of step i-1 into the edge
      // that step i leaves when it picks j1; own[r] keeps that candidate's key
      uint32_t own[NPL], key1 = 0xFFFFFFFFu;
#pragma unroll
      for (int r = 0; r < NPL; ++r) {
        const int node = (lane + 32 * r) & (Q * Q - 1);
        const int j1 = node & (Q - 1), kb = node >> K;
        const int x1 = (j1 << (G::Kr - K)) | (e >> K);
        own[r] = cand_key(kb, cand_finish<K>(cand_diff<K>(cb, kb, x1, ws1), v2[r], kb, x1,
                                             PASS == 2 && s1 == 0, pre));
        key1 = min(key1, own[r]);
      }
#pragma unroll
      for (int h = Q; h < 32; h <<= 1)  // lanes with the same j1 = lane & (Q-1)
        key1 = min(key1, __shfl_xor_sync(0xFFFFFFFFu, key1, h));
      // step i: branch kq from level-1 node kq, whose minimum this lane holds
      const uint32_t bk = cand_key(kq, cand_finish<K>(d0, key_cost(key1), kq, e,
                                                      PASS == 2 && i == 0, pre));
      const int k0 = pick(__reduce_min_sync(0xFFFFFFFFu, bk));
      if (PASS == 2 && lane == 0) st[i] = (uint16_t)((k0 << G::Kr) | e);
      e = (k0 << G::GB) | (e >> K);
      if (s1 >= i_stop) {
        // step i - 1: the candidates of level-1 node k0 are its branches
        uint32_t bk2 = 0xFFFFFFFFu;
#pragma unroll
        for (int r = 0; r < NPL; ++r)
          if (((lane + 32 * r) & (Q - 1)) == k0) bk2 = min(bk2, own[r]);
        const int k1 = pick(__reduce_min_sync(0xFFFFFFFFu, bk2));
        if (PASS == 2 && lane == 0) st[s1] = (uint16_t)((k1 << G::Kr) | e);
        e = (k1 << G::GB) | (e >> K);
      }
    }
    i = c;
  }
  return e;
}

// The K = 1 single-tile walk in registers (checkpoints hold one fp16 cost
// per edge every kSingleR = 4 steps; with L a multiple of 4 every segment
// spans four steps). Lane j < 16 loads level-4 node j (the 16 ancestors of
// the path edge four steps up); level m < 4 node j lives in every lane with
// lane & (2^m - 1) == j: such a lane evaluates branch k = (lane >> m) & 1
// from its own level-(m+1) cost and the two branches meet by one xor
// shuffle of their keys (a key holds its cost bits). The path steps below
// the top reuse those keys: step i - tt's candidates are the level-tt
// candidates of the node the steps before it picked. Costs, keys
// (cand_key) and the first-minimum rule are the forward pass's.
template <int PASS>
__device__ int ck_walk_single_reg(const uint8_t* __restrict__ pck, int cb, const uint16_t* w,
                                  int L, int e_top, int pre, uint16_t* st, int lane) {
  using G = PGeo<1>;
  constexpr int R = kSingleR;
  constexpr int CKB = G::S * 2;
  const int half = L / 2;
  const int i_stop = PASS == 1 ? half : 0;
  auto wt = [&](int s) { return w[PASS == 1 ? (s < half ? s + half : s - half) : s]; };
  auto pick = [&](uint32_t bk) { return (bk == 0u || bk == 0xFFFFFFFFu) ? 0 : (int)(bk & 0xFFFFu); };
  int i = L - 1, e = e_top;
  while (i >= i_stop) {
    int c, slot;
    if (PASS == 1) {
      const int rel = ((i - 1) - (half - 1)) / R;
      c = (half - 1) + rel * R;
      slot = rel;
    } else {
      c = (i / R) * R - 1;
      slot = (c + 1) / R - 1;
    }
    const int Lv = i - c;  // 4
    const uint16_t* ckb =
        c >= 0 ? reinterpret_cast<const uint16_t*>(pck + (size_t)slot * CKB) : nullptr;
    uint32_t cost[5];  // cost[m]: this lane's level-m node
    {
      const int node = lane & ((1 << Lv) - 1);
      cost[4] = ckb ? (uint32_t)__ldg(ckb + ((node << (G::Kr - Lv)) | (e >> Lv))) : 0u;
    }
    // step i, branch lane & 1: its difference needs no load
    const uint16_t d0 = cand_diff<1>(cb, lane & 1, e, wt(i));
    uint32_t own[4];  // own[m]: this lane's branch of level-m node lane & (2^m - 1)
#pragma unroll
    for (int m = 3; m >= 1; --m) {
      if (m >= Lv) {
        cost[m] = cost[m + 1];  // levels above the segment's top are not used
        own[m] = 0xFFFFFFFFu;
        continue;
      }
      const int j = lane & ((1 << m) - 1), kb = (lane >> m) & 1;
      const int s = i - m;
      const int x = (j << (G::Kr - m)) | (e >> m);
      own[m] = cand_key(kb, cand_finish<1>(cand_diff<1>(cb, kb, x, wt(s)), (uint16_t)cost[m + 1],
                                           kb, x, PASS == 2 && s == 0, pre));
      cost[m] = key_cost(min(own[m], __shfl_xor_sync(0xFFFFFFFFu, own[m], 1 << m)));
    }
    // the path: steps i .. c+1. Step i: branch lane & 1 from level-1 node
    // lane & 1 (this lane's cost[1]); step i - tt (tt >= 1): the level-tt
    // candidates of the node the steps before picked (j), keys reused.
    int j = 0;
#pragma unroll
    for (int tt = 0; tt < 4; ++tt) {
      if (tt >= Lv || i - tt < i_stop) break;
      const int s = i - tt;
      uint32_t bk;
      if (tt == 0)
        bk = cand_key(lane & 1, cand_finish<1>(d0, (uint16_t)cost[1], lane & 1, e,
                                               PASS == 2 && s == 0, pre));
      else
        bk = (lane & ((1 << tt) - 1)) == j ? own[tt] : 0xFFFFFFFFu;
      const int k = pick(__reduce_min_sync(0xFFFFFFFFu, bk));
      if (PASS == 2 && lane == 0) st[s] = (uint16_t)((k << G::Kr) | e);
      j |= k << tt;
      e = (k << G::GB) | (e >> 1);
    }
    i = c;
  }
  return e;
}

template <int K>
__device__ __forceinline__ void tb_load_weights(const float* __restrict__ in, int tile, int L,
                                                uint16_t* w, int lane) {
  for (int i = lane; i < L; i += 32)
    w[i] = __half_as_ushort(__float2half_rn(in[(size_t)tile * L + i]));
  __syncwarp();
}

template <int K, int D>
__global__ void __launch_bounds__(32 * kTbWarps)
pair_tb1_kernel(const float* __restrict__ in, const uint8_t* __restrict__ ck, size_t ck_pair_bytes,
                int n, int L, int cb, const int32_t* __restrict__ best_edge,
                int32_t* __restrict__ end_state) {
  __shared__ uint16_t w[kTbWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x * kTbWarps + warp;
  if (tile >= n) return;
  tb_load_weights<K>(in, tile, L, w[warp], lane);
  const int e = ck_walk_reg<K, 1, D>(ck + (size_t)(tile >> 1) * ck_pair_bytes, tile & 1, cb, w[warp],
                                  L, best_edge[tile], -1, nullptr, lane);
  if (lane == 0) end_state[tile] = e;
}

template <int K, int D>
__global__ void __launch_bounds__(32 * kTbWarps)
pair_tb2_kernel(const float* __restrict__ in, const uint8_t* __restrict__ ck, size_t ck_pair_bytes,
                int n, int L, int cb, const int32_t* __restrict__ end_state,
                float* __restrict__ out_w, int16_t* __restrict__ out_idx,
                int16_t* __restrict__ out_packed) {
  __shared__ uint16_t w[kTbWarps][256];
  __shared__ uint16_t st[kTbWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x * kTbWarps + warp;
  if (tile >= n) return;
  tb_load_weights<K>(in, tile, L, w[warp], lane);
  const int pre = end_state[tile];
  ck_walk_reg<K, 2, D>(ck + (size_t)(tile >> 1) * ck_pair_bytes, tile & 1, cb, w[warp], L, pre, pre,
                    st[warp], lane);
  __syncwarp();
  for (int i = lane; i < L; i += 32) {
    const uint16_t s = st[warp][i];
    out_idx[(size_t)tile * L + i] = (int16_t)s;
    out_w[(size_t)tile * L + i] = half_bits_to_float(cb_state_bits(cb, s));
  }
  if (out_packed && L == 256 && lane < 16)
    pack_span(st[warp], K, lane, out_packed + (size_t)tile * 16 * K);
}

template <int K>
int pair_encode_chunks(const float* in, float* out_w, int16_t* out_idx, int16_t* out_packed,
                       float* out_cost, int64_t n, int cb, int L, uint8_t* ws, size_t ws_bytes,
                       cudaStream_t stream) {
  static DeviceBits attr_done;
  int dev = 0;
  EXL3_CUDA(cudaGetDevice(&dev));
  if (!attr_done.has(dev)) {
    EXL3_CUDA(cudaFuncSetAttribute(acs_pair_kernel<K, 1>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)PSmem<K>::bytes));
    EXL3_CUDA(cudaFuncSetAttribute(acs_pair_kernel<K, 2>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)PSmem<K>::bytes));
    attr_done.set(dev);
  }
  const size_t per_tile = pair_tile_ws_bytes(K, L);
  const size_t ck_pair = pair_ck_bytes(K, L);
  int64_t cap = (int64_t)(ws_bytes / per_tile) & ~(int64_t)1;  // whole pairs
  EXL3_REQUIRE(cap >= 2, "workspace of %zu bytes is smaller than one tile pair (%zu bytes)",
               ws_bytes, 2 * per_tile);
  if (cap > n) cap = (n + 1) & ~(int64_t)1;
  if (cap > (1 << 30)) cap = 1 << 30;
  uint8_t* ck = ws;
  int32_t* best_edge = reinterpret_cast<int32_t*>(ws + (size_t)(cap / 2) * ck_pair);
  int32_t* end_state = best_edge + cap;
  const int sms = sm_count();
  for (int64_t start = 0; start < n; start += cap) {
    const int m = (int)((n - start) < cap ? (n - start) : cap);
    const int pairs = (m + 1) / 2;
    const float* cin = in + start * L;
    const int tb_grid = (m + kTbWarps - 1) / kTbWarps;
    // few pairs: every pair split over a cluster; more than one wave: whole
    // waves one pair per CTA, and the last partial wave, if it is small
    // enough, split over clusters (it would otherwise leave most SMs idle
    // for a whole wave)
    int csize = 1, cpairs = 1;
    cluster_choice(K, pairs, &csize, &cpairs);
    int bulk = pairs, tail = 0, tail_c = 1, tail_p = 1;
    if (csize == 1 && pairs > sms && pairs % sms) {
      cluster_choice(K, pairs % sms, &tail_c, &tail_p);
      if (tail_c > 1) {
        tail = pairs % sms;
        bulk = pairs - tail;
      }
    }
    const int mb = 2 * bulk < m ? 2 * bulk : m;  // tiles of the whole waves
    // Tracebacks at K = 3 (a checkpoint every step) take two steps per
    // segment in calls of at most one wave of pairs whose checkpoints do not
    // fit in L2: each segment is then a round trip to HBM on the path's
    // critical chain, and halving their number outweighs evaluating 64
    // ancestors per segment (measured: 256 tiles 1.000 -> 0.916 ms per call).
    // Larger calls keep one step per segment, and so does K = 4, whose 256
    // ancestors per segment made its tracebacks twice as slow. Outputs are
    // identical either way.
    constexpr int RD = PGeo<K>::R;
    constexpr bool kDeepOk = K == 3 && RD == 1;
    const bool deep = kDeepOk && pairs <= sms && (size_t)pairs * ck_pair > kTbDeepBytes;
    auto acs_pass = [&](int pass) -> int {
      LaunchTimer lt(stream, 0);
      int32_t* be = pass == 1 ? best_edge : nullptr;
      const int32_t* es = pass == 2 ? end_state : nullptr;
      float* pc = (pass == 2 && out_cost) ? out_cost + start : nullptr;
      if (csize > 1)
        return cluster_acs_pass(K, csize, cpairs, pass, stream, cin, m, L, cb, ck, ck_pair, be, es,
                                pc);
      const int g = bulk < sms ? bulk : sms;
      if (pass == 1)
        acs_pair_kernel<K, 1><<<g, kPairNT, PSmem<K>::bytes, stream>>>(cin, mb, L, cb, ck, ck_pair,
                                                                      be, es, pc);
      else
        acs_pair_kernel<K, 2><<<g, kPairNT, PSmem<K>::bytes, stream>>>(cin, mb, L, cb, ck, ck_pair,
                                                                      be, es, pc);
      EXL3_LAUNCHED();
      if (!tail) return EXL3_OK;
      return cluster_acs_pass(K, tail_c, tail_p, pass, stream, cin + (size_t)mb * L, m - mb, L, cb,
                              ck + (size_t)bulk * ck_pair, ck_pair, be ? be + mb : nullptr,
                              es ? es + mb : nullptr, pc ? pc + mb : nullptr);
    };
    if (int rc = acs_pass(1)) return rc;
    EXL3_LAUNCHED();
    {
      LaunchTimer lt(stream, 1);
      if (deep)
        pair_tb1_kernel<K, kDeepOk ? 2 : RD><<<tb_grid, 32 * kTbWarps, 0, stream>>>(
            cin, ck, ck_pair, m, L, cb, best_edge, end_state);
      else
        pair_tb1_kernel<K, RD><<<tb_grid, 32 * kTbWarps, 0, stream>>>(cin, ck, ck_pair, m, L, cb,
                                                                     best_edge, end_state);
    }
    EXL3_LAUNCHED();
    if (int rc = acs_pass(2)) return rc;
    EXL3_LAUNCHED();
    {
      LaunchTimer lt(stream, 1);
      int16_t* pk = out_packed ? out_packed + start * 16 * K : nullptr;
      if (deep)
        pair_tb2_kernel<K, kDeepOk ? 2 : RD><<<tb_grid, 32 * kTbWarps, 0, stream>>>(
            cin, ck, ck_pair, m, L, cb, end_state, out_w + start * L, out_idx + start * L, pk);
      else
        pair_tb2_kernel<K, RD><<<tb_grid, 32 * kTbWarps, 0, stream>>>(
            cin, ck, ck_pair, m, L, cb, end_state, out_w + start * L, out_idx + start * L, pk);
    }
    EXL3_LAUNCHED();
  }
  return EXL3_OK;
}


// ---------------------------------------------------------------------------
// K = 1: one tile per CTA. A tile pair's two 32,768-word cost vectors would
// take 256 KiB, above a CTA's shared memory; one tile's fp16 vectors take
// 128 KiB. The fp16 lanes hold the two edges 2g and 2g+1 that share both
// predecessors g and g + 2^14, so a step is the pair kernel's step with
// edges instead of tiles in the lanes: per edge pair two sub + two fma on
// the FMA pipe and one min on the ALU pipe, min-only, cost checkpoints every
// kSingleR steps by bulk copy, the same recomputing traceback.
// ---------------------------------------------------------------------------
struct SGeo {
  static constexpr int S = 32768;               // edges
  static constexpr int NP = S / 2 / kPairNT;    // 32 edge pairs per thread
  static constexpr int CP = 8;                  // pairs per chunk
  static constexpr int NCH = NP / CP;           // 4 chunks per step
  static constexpr int R = kSingleR;
  static constexpr int CKB = S * 2;             // fp16 per edge
};

__host__ __device__ constexpr int single_slots_pass1(int L) { return (L - L / 2 - 1) / kSingleR + 1; }
__host__ __device__ constexpr int single_slots_pass2(int L) { return (L - 1) / kSingleR; }

size_t single_ck_bytes(int L) {
  const int s1 = single_slots_pass1(L), s2 = single_slots_pass2(L);
  const size_t b = (size_t)(s1 > s2 ? s1 : s2) * SGeo::CKB;
  return (b + 255) / 256 * 256;
}

size_t single_tile_ws_bytes(int L) { return single_ck_bytes(L) + 8; }

// edge pair g = (c * 512 + t) * CP + j: cbv[(c * CP + j) * 2 + k] holds the
// codebook values of states (k << 15) | 2g and (k << 15) | (2g + 1)
__device__ __forceinline__ void single_init_codebook(uint32_t (&cbv)[64], int cb, int t) {
#pragma unroll
  for (int c = 0; c < SGeo::NCH; ++c)
#pragma unroll
    for (int j = 0; j < SGeo::CP; ++j) {
      const uint32_t g = (uint32_t)((c * kPairNT + t) * SGeo::CP + j);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const uint32_t s0 = ((uint32_t)k << 15) | (2 * g);
        cbv[(c * SGeo::CP + j) * 2 + k] =
            (uint32_t)cb_state_bits(cb, s0) | ((uint32_t)cb_state_bits(cb, s0 + 1) << 16);
      }
    }
}

// cin: fp16 per edge; cout: {cost(2g), cost(2g+1)} words per edge pair (the
// same bytes read as fp16 per edge); w2 = {w, w}
template <bool FIRST, bool EXACT>
__device__ __forceinline__ void single_step(const uint32_t (&cbv)[64], uint32_t w2,
                                            const uint16_t* __restrict__ cin,
                                            uint32_t* __restrict__ cout, int t, int pre) {
#pragma unroll
  for (int c = 0; c < SGeo::NCH; ++c) {
    const int g0 = (c * kPairNT + t) * SGeo::CP;
    uint32_t p0[4], p1[4];
    if constexpr (!FIRST) {
      const uint4 a = *reinterpret_cast<const uint4*>(cin + g0);
      const uint4 b = *reinterpret_cast<const uint4*>(cin + (1 << 14) + g0);
      p0[0] = a.x; p0[1] = a.y; p0[2] = a.z; p0[3] = a.w;
      p1[0] = b.x; p1[1] = b.y; p1[2] = b.z; p1[3] = b.w;
    }
    uint32_t best[SGeo::CP];
#pragma unroll
    for (int j = 0; j < SGeo::CP; ++j) {
      uint32_t c0, c1;
      {
        const uint32_t d0 = h2_sub(cbv[(c * SGeo::CP + j) * 2], w2);
        const uint32_t d1 = h2_sub(cbv[(c * SGeo::CP + j) * 2 + 1], w2);
        uint32_t q0 = 0u, q1 = 0u;
        if constexpr (!FIRST) {
          q0 = (j & 1) ? h2_hi2(p0[j >> 1]) : h2_lo2(p0[j >> 1]);
          q1 = (j & 1) ? h2_hi2(p1[j >> 1]) : h2_lo2(p1[j >> 1]);
        }
        c0 = h2_fma(d0, d0, q0);
        c1 = h2_fma(d1, d1, q1);
      }
      if constexpr (FIRST) {
        if (pre >= 0) {
          const int g = g0 + j;
          c0 = (g == pre) ? c0 : kHInf2;                 // pred (0 << 14) | g
          c1 = (((1 << 14) | g) == pre) ? c1 : kHInf2;   // pred (1 << 14) | g
        }
      }
      best[j] = EXACT ? bsel(h2_lt_mask(c1, c0), c1, c0) : h2_min(c0, c1);
    }
    uint4* dst = reinterpret_cast<uint4*>(cout + g0);
    dst[0] = make_uint4(best[0], best[1], best[2], best[3]);
    dst[1] = make_uint4(best[4], best[5], best[6], best[7]);
  }
}

template <bool EXACT>
__device__ __forceinline__ void single_pass1(const uint32_t (&cbv)[64], const uint32_t* wt,
                                             uint16_t* c0, uint16_t* c1, uint8_t* ckp, int L,
                                             int t) {
  const int half = L / 2;
  single_step<true, EXACT>(cbv, wt[half], nullptr, reinterpret_cast<uint32_t*>(c0), t, -1);
  __syncthreads();
  for (int i = 1; i < L; ++i) {
    const uint16_t* cin = (i & 1) ? c0 : c1;
    uint16_t* cout = (i & 1) ? c1 : c0;
    single_step<false, EXACT>(cbv, wt[i < half ? i + half : i - half], cin,
                              reinterpret_cast<uint32_t*>(cout), t, -1);
    const int rel = i - (half - 1);
    const bool ckpt = rel >= 0 && rel % SGeo::R == 0 && i <= L - 2;
    if (ckpt) ck_fence();
    if (t == 0) ck_wait_read();
    __syncthreads();
    if (ckpt && t == 0)
      ck_issue(ckp + (size_t)(rel / SGeo::R) * SGeo::CKB, reinterpret_cast<uint32_t*>(cout),
               SGeo::CKB);
  }
  if (t == 0) ck_wait_read();
}

template <bool EXACT>
__device__ __forceinline__ void single_pass2(const uint32_t (&cbv)[64], const uint32_t* wt,
                                             uint16_t* c0, uint16_t* c1, uint8_t* ckp, int L,
                                             int t, int pre) {
  single_step<true, EXACT>(cbv, wt[0], nullptr, reinterpret_cast<uint32_t*>(c0), t, pre);
  __syncthreads();
  for (int i = 1; i < L; ++i) {
    const uint16_t* cin = (i & 1) ? c0 : c1;
    uint16_t* cout = (i & 1) ? c1 : c0;
    single_step<false, EXACT>(cbv, wt[i], cin, reinterpret_cast<uint32_t*>(cout), t, -1);
    const bool ckpt = (i + 1) % SGeo::R == 0 && i <= L - 2;
    if (ckpt) ck_fence();
    if (t == 0) ck_wait_read();
    __syncthreads();
    if (ckpt && t == 0)
      ck_issue(ckp + (size_t)((i + 1) / SGeo::R - 1) * SGeo::CKB,
               reinterpret_cast<uint32_t*>(cout), SGeo::CKB);
  }
  if (t == 0) ck_wait_read();
}

// minimum cost, lowest edge on ties, non-finite skipped, none finite -> 0
__device__ __forceinline__ int single_argmin(const uint16_t* costs, uint32_t* red, int t) {
  uint32_t key = 0xFFFFFFFFu;
  for (int e = t; e < SGeo::S; e += kPairNT) {
    const uint32_t b = costs[e];
    if ((b & 0x7C00u) != 0x7C00u) key = min(key, (b << 16) | (uint32_t)e);
  }
  key = __reduce_min_sync(0xFFFFFFFFu, key);
  if ((t & 31) == 0) red[t >> 5] = key;
  __syncthreads();
  if (t < 32) {
    uint32_t v = (t < kPairNT / 32) ? red[t] : 0xFFFFFFFFu;
    v = __reduce_min_sync(0xFFFFFFFFu, v);
    if (t == 0) red[0] = v;
  }
  __syncthreads();
  const uint32_t v = red[0];
  __syncthreads();
  return v == 0xFFFFFFFFu ? 0 : (int)(v & 0xFFFFu);
}

constexpr size_t kSingleSmem = 2ull * SGeo::S * sizeof(uint16_t) + 256 * sizeof(uint32_t);

template <int PASS>
__global__ void __launch_bounds__(kPairNT, 1)
acs_single_kernel(const float* __restrict__ in, int n, int L, int cb, uint8_t* __restrict__ ck,
                  size_t ck_tile_bytes, int32_t* __restrict__ best_edge,
                  const int32_t* __restrict__ end_state, float* __restrict__ path_cost) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t* c0 = reinterpret_cast<uint16_t*>(smem);
  uint16_t* c1 = c0 + SGeo::S;
  uint32_t* wt = reinterpret_cast<uint32_t*>(smem + 2ull * SGeo::S * sizeof(uint16_t));
  __shared__ uint32_t red[kPairNT / 32];
  const int t = threadIdx.x;
  uint32_t cbv[64];
  single_init_codebook(cbv, cb, t);
  for (int tile = blockIdx.x; tile < n; tile += gridDim.x) {
    int nan = 0;
    for (int i = t; i < L; i += kPairNT) {
      const __half h = __float2half_rn(in[(size_t)tile * L + i]);
      const uint32_t b = __half_as_ushort(h);
      nan |= __hisnan(h) ? 1 : 0;
      wt[i] = b | (b << 16);
    }
    nan = __syncthreads_or(nan);
    uint8_t* tck = ck + (size_t)tile * ck_tile_bytes;
    const uint16_t* fin = ((L - 1) & 1) ? c1 : c0;
    if constexpr (PASS == 1) {
      if (nan) single_pass1<true>(cbv, wt, c0, c1, tck, L, t);
      else     single_pass1<false>(cbv, wt, c0, c1, tck, L, t);
      const int be = single_argmin(fin, red, t);
      if (t == 0) best_edge[tile] = be;
    } else {
      const int pre = end_state[tile];
      if (nan) single_pass2<true>(cbv, wt, c0, c1, tck, L, t, pre);
      else     single_pass2<false>(cbv, wt, c0, c1, tck, L, t, pre);
      if (t == 0 && path_cost) path_cost[tile] = half_bits_to_float(fin[pre]);
    }
    __syncthreads();
  }
  if (t == 0) ck_wait_all();
}

__global__ void __launch_bounds__(32 * kTbWarps)
single_tb1_kernel(const float* __restrict__ in, const uint8_t* __restrict__ ck,
                  size_t ck_tile_bytes, int n, int L, int cb,
                  const int32_t* __restrict__ best_edge, int32_t* __restrict__ end_state) {
  __shared__ uint16_t w[kTbWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x * kTbWarps + warp;
  if (tile >= n) return;
  tb_load_weights<1>(in, tile, L, w[warp], lane);
  const int e = ck_walk_single_reg<1>(ck + (size_t)tile * ck_tile_bytes, cb, w[warp], L,
                                      best_edge[tile], -1, nullptr, lane);
  if (lane == 0) end_state[tile] = e;
}

__global__ void __launch_bounds__(32 * kTbWarps)
single_tb2_kernel(const float* __restrict__ in, const uint8_t* __restrict__ ck,
                  size_t ck_tile_bytes, int n, int L, int cb,
                  const int32_t* __restrict__ end_state, float* __restrict__ out_w,
                  int16_t* __restrict__ out_idx, int16_t* __restrict__ out_packed) {
  __shared__ uint16_t w[kTbWarps][256];
  __shared__ uint16_t st[kTbWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x * kTbWarps + warp;
  if (tile >= n) return;
  tb_load_weights<1>(in, tile, L, w[warp], lane);
  const int pre = end_state[tile];
  ck_walk_single_reg<2>(ck + (size_t)tile * ck_tile_bytes, cb, w[warp], L, pre, pre, st[warp],
                        lane);
  __syncwarp();
  for (int i = lane; i < L; i += 32) {
    const uint16_t s = st[warp][i];
    out_idx[(size_t)tile * L + i] = (int16_t)s;
    out_w[(size_t)tile * L + i] = half_bits_to_float(cb_state_bits(cb, s));
  }
  if (out_packed && L == 256 && lane < 16)
    pack_span(st[warp], 1, lane, out_packed + (size_t)tile * 16);
}

int single_encode(const float* in, float* out_w, int16_t* out_idx, int16_t* out_packed,
                  float* out_cost, int64_t n, int cb, int L, uint8_t* ws, size_t ws_bytes,
                  cudaStream_t stream) {
  static DeviceBits attr_done;
  int dev = 0;
  EXL3_CUDA(cudaGetDevice(&dev));
  if (!attr_done.has(dev)) {
    EXL3_CUDA(cudaFuncSetAttribute(acs_single_kernel<1>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSingleSmem));
    EXL3_CUDA(cudaFuncSetAttribute(acs_single_kernel<2>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSingleSmem));
    attr_done.set(dev);
  }
  const size_t per_tile = single_tile_ws_bytes(L);
  const size_t ck_tile = single_ck_bytes(L);
  int64_t cap = (int64_t)(ws_bytes / per_tile);
  EXL3_REQUIRE(cap >= 1, "workspace of %zu bytes is smaller than one tile (%zu bytes)", ws_bytes,
               per_tile);
  if (cap > n) cap = n;
  if (cap > (1 << 30)) cap = 1 << 30;
  uint8_t* ck = ws;
  int32_t* best_edge = reinterpret_cast<int32_t*>(ws + (size_t)cap * ck_tile);
  int32_t* end_state = best_edge + cap;
  const int sms = sm_count();
  for (int64_t start = 0; start < n; start += cap) {
    const int m = (int)((n - start) < cap ? (n - start) : cap);
    const int grid = m < sms ? m : sms;
    const int tb_grid = (m + kTbWarps - 1) / kTbWarps;
    const float* cin = in + start * L;
    {
      LaunchTimer lt(stream, 0);
      acs_single_kernel<1><<<grid, kPairNT, kSingleSmem, stream>>>(cin, m, L, cb, ck, ck_tile,
                                                                   best_edge, nullptr, nullptr);
    }
    EXL3_LAUNCHED();
    {
      LaunchTimer lt(stream, 1);
      single_tb1_kernel<<<tb_grid, 32 * kTbWarps, 0, stream>>>(cin, ck, ck_tile, m, L, cb,
                                                               best_edge, end_state);
    }
    EXL3_LAUNCHED();
    {
      LaunchTimer lt(stream, 0);
      acs_single_kernel<2><<<grid, kPairNT, kSingleSmem, stream>>>(
          cin, m, L, cb, ck, ck_tile, nullptr, end_state, out_cost ? out_cost + start : nullptr);
    }
    EXL3_LAUNCHED();
    {
      LaunchTimer lt(stream, 1);
      single_tb2_kernel<<<tb_grid, 32 * kTbWarps, 0, stream>>>(
          cin, ck, ck_tile, m, L, cb, end_state, out_w + start * L, out_idx + start * L,
          out_packed ? out_packed + start * 16 : nullptr);
    }
    EXL3_LAUNCHED();
  }
  return EXL3_OK;
}

int pair_encode(int K, const float* in, float* out_w, int16_t* out_idx, int16_t* out_packed,
                float* out_cost, int64_t n, int cb, int L, uint8_t* ws, size_t ws_bytes,
                cudaStream_t stream) {
  switch (K) {
    case 2: return pair_encode_chunks<2>(in, out_w, out_idx, out_packed, out_cost, n, cb, L, ws, ws_bytes, stream);
    case 3: return pair_encode_chunks<3>(in, out_w, out_idx, out_packed, out_cost, n, cb, L, ws, ws_bytes, stream);
    case 4: return pair_encode_chunks<4>(in, out_w, out_idx, out_packed, out_cost, n, cb, L, ws, ws_bytes, stream);
    case 5: return pair_encode_chunks<5>(in, out_w, out_idx, out_packed, out_cost, n, cb, L, ws, ws_bytes, stream);
    case 6: return pair_encode_chunks<6>(in, out_w, out_idx, out_packed, out_cost, n, cb, L, ws, ws_bytes, stream);
    case 7: return pair_encode_chunks<7>(in, out_w, out_idx, out_packed, out_cost, n, cb, L, ws, ws_bytes, stream);
    case 8: return pair_encode_chunks<8>(in, out_w, out_idx, out_packed, out_cost, n, cb, L, ws, ws_bytes, stream);
    default:
      set_error("pair encoder supports K in 2..8, got %d", K);
      return EXL3_EINVAL;
  }
}

}  // namespace exl3
