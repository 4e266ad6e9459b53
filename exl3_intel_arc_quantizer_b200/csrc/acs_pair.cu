// Tile-pair ACS encoder (K = 2..8): two tiles share one CTA, one per fp16
// half2 lane.
//
// Both tiles walk the same trellis, so a candidate's codebook value is one
// scalar shared by the two lanes; everything per-tile (weight, accumulated
// cost, branch choice) is a lane of one 32-bit register. Consequences:
//   * the cost vector is stored as {cost_A, cost_B} words in natural edge
//     order: a predecessor cost is read as one word that already holds both
//     lanes, and a result is written as one word -- no lane shuffles;
//   * every barrier covers two tiles' work (half the barriers per tile) and
//     each thread carries twice the independent dependency chains;
//   * threads take edges chunk-major (consecutive threads own consecutive
//     chunks) so a warp's shared-memory stores are contiguous.
// The arithmetic, tie-breaking and NaN behaviour are those of encoder.cu
// (reference_encoder.py:130-324); only the data layout differs.
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
  static constexpr int EPW = SPLIT ? 1 : (K == 2 ? 8 : (K <= 4 ? 4 : 2));
  static constexpr int NW = SPLIT ? 1 : (E + EPW - 1) / EPW;
  static constexpr int BPS = SPLIT ? S * 4 : NW * kPairNT * 4;  // bytes / step / pair
  static_assert(E * QT == 128, "codebook register budget: 128 values per thread");
};

int pair_bp_step_bytes(int K) {
  switch (K) {
    case 2: return PGeo<2>::BPS;
    case 3: return PGeo<3>::BPS;
    case 4: return PGeo<4>::BPS;
    case 5: return PGeo<5>::BPS;
    case 6: return PGeo<6>::BPS;
    case 7: return PGeo<7>::BPS;
    case 8: return PGeo<8>::BPS;
    default: return 0;
  }
}

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

// acc + idx * 2^sh through the integer multiply-add (keeps the ALU pipe free).
__device__ __forceinline__ uint32_t mad_shift(uint32_t idx, int sh, uint32_t acc) {
  uint32_t r;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(idx), "r"(1u << sh), "r"(acc));
  return r;
}

// One ACS step over both lanes.
//   FIRST : step 0; pre2 = {pre_A, pre_B} wrap constraint (-1 = none)
//   TRACK : record branch choices (COMPACT words) for the traceback
//   EXACT : compare-and-select for the cost too (NaN-faithful)
template <int K, bool FIRST, bool TRACK, bool EXACT>
__device__ __forceinline__ void pair_step(const uint32_t (&cbv)[64], uint32_t w2,
                                          const uint32_t* __restrict__ cin,
                                          uint32_t* __restrict__ cout,
                                          uint32_t* __restrict__ bp_step, int t, int preA,
                                          int preB) {
  using G = PGeo<K>;
  if constexpr (!G::SPLIT) {
#pragma unroll
    for (int c = 0; c < G::NCH; ++c) {
      const int e0 = (c * kPairNT + t) * G::CE;
      const int g0 = e0 >> K;
      uint32_t best[G::CE], idx[G::CE];
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
              idx[j] = 0;
            } else if constexpr (TRACK || EXACT) {
              const uint32_t msk = h2_lt_mask(cst, best[j]);
              best[j] = EXACT ? bsel(msk, cst, best[j]) : h2_min(best[j], cst);
              if constexpr (TRACK) idx[j] = bsel(msk, kconst(k), idx[j]);
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
      if constexpr (TRACK) {
#pragma unroll
        for (int a = 0; a < (G::CE + G::EPW - 1) / G::EPW; ++a) {
          uint32_t acc = 0;
#pragma unroll
          for (int j = a * G::EPW; j < (a + 1) * G::EPW && j < G::CE; ++j)
            acc = (j == a * G::EPW) ? idx[j] : mad_shift(idx[j], K * (j - a * G::EPW), acc);
          const int w = (c * G::CE) / G::EPW + a;
          bp_step[w * kPairNT + t] = acc;
        }
      }
    }
  } else {
    // K = 8: lanes t and t^1 split the 256 branches of edge t >> 1.
    const int e = t >> 1, r = t & 1;
    const int k0 = r * G::QT;
    uint32_t best = kHInf2, idx = kconst(k0);
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
          const uint32_t msk = h2_lt_mask(cst, best) | (r == 0 ? 0xFFFFFFFFu : 0u);
          best = bsel(msk, cst, best);
          if constexpr (TRACK) idx = bsel(msk, kconst(k), idx);
        } else if constexpr (TRACK || EXACT) {
          const uint32_t msk = h2_lt_mask(cst, best);
          best = EXACT ? bsel(msk, cst, best) : h2_min(best, cst);
          if constexpr (TRACK) idx = bsel(msk, kconst(k), idx);
        } else {
          best = h2_min(best, cst);
        }
      }
    }
    // lower branch range (r = 0) wins ties
    const uint32_t ob = __shfl_xor_sync(0xFFFFFFFFu, best, 1);
    const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, idx, 1);
    const uint32_t lo_c = r ? ob : best, hi_c = r ? best : ob;
    const uint32_t lo_i = r ? oi : idx, hi_i = r ? idx : oi;
    const uint32_t msk = h2_lt_mask(hi_c, lo_c);
    if (r == 0) {
      cout[e] = bsel(msk, hi_c, lo_c);
      if constexpr (TRACK) bp_step[e] = bsel(msk, hi_i, lo_i);
    }
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

template <int K, bool EXACT>
__device__ __forceinline__ void pair_pass1(const uint32_t (&cbv)[64], const uint32_t* wt,
                                           uint32_t* c0, uint32_t* c1, uint8_t* bp, int L,
                                           int t) {
  using G = PGeo<K>;
  const int half = L / 2;
  pair_step<K, true, false, EXACT>(cbv, wt[half], nullptr, c0, nullptr, t, -1, -1);
  __syncthreads();
  for (int i = 1; i < half; ++i) {
    const uint32_t* cin = (i & 1) ? c0 : c1;
    uint32_t* cout = (i & 1) ? c1 : c0;
    pair_step<K, false, false, EXACT>(cbv, wt[i + half], cin, cout, nullptr, t, -1, -1);
    __syncthreads();
  }
  for (int i = half; i < L; ++i) {
    const int ri = i - half;
    const uint32_t* cin = (i & 1) ? c0 : c1;
    uint32_t* cout = (i & 1) ? c1 : c0;
    pair_step<K, false, true, EXACT>(cbv, wt[ri], cin, cout,
                                     reinterpret_cast<uint32_t*>(bp + (size_t)ri * G::BPS), t,
                                     -1, -1);
    __syncthreads();
  }
}

template <int K, bool EXACT>
__device__ __forceinline__ void pair_pass2(const uint32_t (&cbv)[64], const uint32_t* wt,
                                           uint32_t* c0, uint32_t* c1, uint8_t* bp, int L,
                                           int t, int preA, int preB) {
  using G = PGeo<K>;
  pair_step<K, true, true, EXACT>(cbv, wt[0], nullptr, c0, reinterpret_cast<uint32_t*>(bp), t,
                                  preA, preB);
  __syncthreads();
  for (int i = 1; i < L; ++i) {
    const uint32_t* cin = (i & 1) ? c0 : c1;
    uint32_t* cout = (i & 1) ? c1 : c0;
    pair_step<K, false, true, EXACT>(cbv, wt[i], cin, cout,
                                     reinterpret_cast<uint32_t*>(bp + (size_t)i * G::BPS), t,
                                     -1, -1);
    __syncthreads();
  }
}

template <int K, int PASS>
__global__ void __launch_bounds__(kPairNT, 1)
acs_pair_kernel(const float* __restrict__ in, int n, int L, int cb, uint8_t* __restrict__ bp,
                size_t bp_pair_bytes, int32_t* __restrict__ best_edge,
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
    uint8_t* pbp = bp + (size_t)tp * bp_pair_bytes;
    const uint32_t* fin = ((L - 1) & 1) ? c1 : c0;
    const int ta = 2 * tp, tb = 2 * tp + 1;
    if constexpr (PASS == 1) {
      if (nan) pair_pass1<K, true>(cbv, wt, c0, c1, pbp, L, t);
      else     pair_pass1<K, false>(cbv, wt, c0, c1, pbp, L, t);
      int ea, eb;
      pair_argmin<K>(fin, red, t, &ea, &eb);
      if (t == 0) {
        best_edge[ta] = ea;
        if (tb < n) best_edge[tb] = eb;
      }
    } else {
      const int preA = end_state[ta];
      const int preB = (tb < n) ? end_state[tb] : preA;
      if (nan) pair_pass2<K, true>(cbv, wt, c0, c1, pbp, L, t, preA, preB);
      else     pair_pass2<K, false>(cbv, wt, c0, c1, pbp, L, t, preA, preB);
      if (t == 0 && path_cost) {
        path_cost[ta] = half_bits_to_float((uint16_t)(fin[preA] & 0xFFFFu));
        if (tb < n) path_cost[tb] = half_bits_to_float((uint16_t)(fin[preB] >> 16));
      }
    }
    __syncthreads();
  }
}

// Branch recorded for (step, edge e, lane b) in the pair layout.
template <int K>
__device__ __forceinline__ int pair_bp_branch(const uint8_t* step_base, int e, int b) {
  using G = PGeo<K>;
  if constexpr (!G::SPLIT) {
    const int c = e / (kPairNT * G::CE);
    const int t = (e / G::CE) % kPairNT;
    const int le = c * G::CE + e % G::CE;
    const int w = le / G::EPW, pos = le % G::EPW;
    const uint32_t word = reinterpret_cast<const uint32_t*>(step_base)[w * kPairNT + t];
    return (int)((word >> (16 * b + K * pos)) & (G::Q - 1));
  } else {
    const uint32_t word = reinterpret_cast<const uint32_t*>(step_base)[e];
    return (int)((word >> (16 * b)) & (G::Q - 1));
  }
}

template <int K>
__global__ void pair_tb1_kernel(const uint8_t* __restrict__ bp, size_t bp_pair_bytes, int n,
                                int L, const int32_t* __restrict__ best_edge,
                                int32_t* __restrict__ end_state) {
  using G = PGeo<K>;
  const int tile = blockIdx.x * blockDim.x + threadIdx.x;
  if (tile >= n) return;
  const uint8_t* pbp = bp + (size_t)(tile >> 1) * bp_pair_bytes;
  const int b = tile & 1;
  int e = best_edge[tile];
  for (int ri = L / 2 - 1; ri >= 0; --ri) {
    const int k = pair_bp_branch<K>(pbp + (size_t)ri * G::BPS, e, b);
    e = (k << G::GB) | (e >> K);
  }
  end_state[tile] = e;
}

template <int K>
__global__ void pair_tb2_kernel(const uint8_t* __restrict__ bp, size_t bp_pair_bytes, int n,
                                int L, int cb, const int32_t* __restrict__ end_state,
                                float* __restrict__ out_w, int16_t* __restrict__ out_idx,
                                int16_t* __restrict__ out_packed) {
  using G = PGeo<K>;
  __shared__ uint16_t st[kTbWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x * kTbWarps + warp;
  if (tile >= n) return;
  const uint8_t* pbp = bp + (size_t)(tile >> 1) * bp_pair_bytes;
  const int b = tile & 1;
  if (lane == 0) {
    int e = end_state[tile];
    for (int i = L - 1; i >= 0; --i) {
      const int k = pair_bp_branch<K>(pbp + (size_t)i * G::BPS, e, b);
      st[warp][i] = (uint16_t)((k << G::Kr) | e);
      e = (k << G::GB) | (e >> K);
    }
  }
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
  static int attr_done = 0;  // one bit per device
  int dev = 0;
  EXL3_CUDA(cudaGetDevice(&dev));
  if (!(dev < 32 && (attr_done & (1 << dev)))) {
    EXL3_CUDA(cudaFuncSetAttribute(acs_pair_kernel<K, 1>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)PSmem<K>::bytes));
    EXL3_CUDA(cudaFuncSetAttribute(acs_pair_kernel<K, 2>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)PSmem<K>::bytes));
    if (dev < 32) attr_done |= (1 << dev);
  }
  const size_t per_tile = pair_tile_ws_bytes(K, L);
  const size_t bp_pair = pair_bp_bytes(K, L);
  int64_t cap = (int64_t)(ws_bytes / per_tile) & ~(int64_t)1;  // whole pairs
  EXL3_REQUIRE(cap >= 2, "workspace of %zu bytes is smaller than one tile pair (%zu bytes)",
               ws_bytes, 2 * per_tile);
  if (cap > n) cap = (n + 1) & ~(int64_t)1;
  if (cap > (1 << 30)) cap = 1 << 30;
  uint8_t* bp = ws;
  int32_t* best_edge = reinterpret_cast<int32_t*>(ws + (size_t)(cap / 2) * bp_pair);
  int32_t* end_state = best_edge + cap;
  const int sms = sm_count();
  for (int64_t start = 0; start < n; start += cap) {
    const int m = (int)((n - start) < cap ? (n - start) : cap);
    const int pairs = (m + 1) / 2;
    const int grid = pairs < sms ? pairs : sms;
    const float* cin = in + start * L;
    {
      LaunchTimer lt(stream, 0);
      acs_pair_kernel<K, 1><<<grid, kPairNT, PSmem<K>::bytes, stream>>>(
          cin, m, L, cb, bp, bp_pair, best_edge, nullptr, nullptr);
    }
    EXL3_LAUNCHED();
    {
      LaunchTimer lt(stream, 1);
      pair_tb1_kernel<K><<<(m + 127) / 128, 128, 0, stream>>>(bp, bp_pair, m, L, best_edge,
                                                              end_state);
    }
    EXL3_LAUNCHED();
    {
      LaunchTimer lt(stream, 0);
      acs_pair_kernel<K, 2><<<grid, kPairNT, PSmem<K>::bytes, stream>>>(
          cin, m, L, cb, bp, bp_pair, nullptr, end_state, out_cost ? out_cost + start : nullptr);
    }
    EXL3_LAUNCHED();
    {
      LaunchTimer lt(stream, 1);
      pair_tb2_kernel<K><<<(m + kTbWarps - 1) / kTbWarps, 32 * kTbWarps, 0, stream>>>(
          bp, bp_pair, m, L, cb, end_state, out_w + start * L, out_idx + start * L,
          out_packed ? out_packed + start * 16 * K : nullptr);
    }
    EXL3_LAUNCHED();
  }
  return EXL3_OK;
}

size_t pair_bp_bytes(int K, int L) {
  return ((size_t)L * pair_bp_step_bytes(K) + 255) / 256 * 256;
}

size_t pair_tile_ws_bytes(int K, int L) { return pair_bp_bytes(K, L) / 2 + 8; }

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
