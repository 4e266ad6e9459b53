// EXL3 trellis Viterbi tile encoder for B200 (sm_100a).
//
// Algorithm restated from the reference CPU encoder
// (exl3_quant/reference_encoder.py:130-324) and its SYCL kernel
// (csrc/quantize_xpu/quantize_kernels.sycl:82-360):
//   * 16-bit shift-register states, K bits per weight, S = 65536 >> K edges;
//     for edge e and branch k: state = (k << (16-K)) | e,
//     pred = state >> K = (k << (16-2K)) | (e >> K);
//   * metric  d = fp16(v - w);  cost = fp16_fma(d, d, cost_prev[pred]);
//   * winner  = first k (ascending) with strictly smaller cost;
//   * two tail-biting passes: (roll = L/2, unconstrained) -> argmin ->
//     traceback to ring index 0 = end_state; (roll = 0, step 0 masked to
//     pred == end_state) -> traceback emitting states.
//
// This file holds the reference-layout split passes, which keep the
// reference's scratch contract (temp_costs (B, 2, S) fp16, temp_edges
// (B, L, S) int16 predecessors, every step recorded) for callers of
// quantize_tiles_forward_pass / _backward_pass; the codebook and container
// kernels; and the C-ABI entry points. exl3_quantize_tiles dispatches to the
// checkpoint encoders in acs_pair.cu (tile pairs for K >= 2, single tiles
// for K = 1).
//
// Reference-layout ACS: one tile per CTA iteration, 512 threads, persistent
// CTAs; the tile's 65536 codebook values live in registers (64 packed half2
// per thread); each thread owns adjacent edge pairs (one half2 lane each,
// both lanes share every predecessor); the fp16 cost vector ping-pongs in
// shared memory; compare-and-select on every branch (NaN-faithful), writing
// the winning predecessor of every edge and step.
#include "common.cuh"
#include "encoder_shared.cuh"
#include "trellis_span.cuh"

namespace exl3 {

std::mutex g_timing_mu;
bool g_timing_on = false;
std::vector<TimedLaunch> g_timed;

constexpr int kNT = 512;  // threads per ACS CTA

template <int K>
struct Geo {
  static constexpr int S = 1 << (16 - K);          // tracked edges
  static constexpr int Kr = 16 - K;                // state = (k << Kr) | e
  static constexpr int GB = 16 - 2 * K;            // pred = (k << GB) | g
  static constexpr int Q = 1 << K;                 // branches per edge
  static constexpr bool SPLIT = (K >= 7);          // branches split over lanes
  static constexpr int EPT = SPLIT ? 2 : S / kNT;  // edges per thread
  static constexpr int NP = EPT / 2;               // edge pairs per thread
  static constexpr int QT = SPLIT ? 64 : Q;        // branches per thread
  static constexpr int R = Q / QT;                 // lanes per edge pair
  static constexpr int CP = SPLIT ? 1 : (K == 1 ? 4 : (NP < 8 ? NP : 8));  // pairs per chunk
  static constexpr int NCH = NP / CP;                       // chunks per step
  static constexpr int CG = SPLIT ? 1 : (((2 * CP) >> K) > 0 ? ((2 * CP) >> K) : 1);
  static constexpr int NCB = NP * QT;              // codebook half2 registers
  static_assert(NCB == 64, "codebook register budget");
};


// Codebook values of this thread's candidates, packed per edge pair.
template <int K>
__device__ __forceinline__ void init_codebook(uint32_t (&cbv)[64], int cb, int t) {
  using G = Geo<K>;
  if constexpr (!G::SPLIT) {
#pragma unroll
    for (int p = 0; p < G::NP; ++p) {
      const uint32_t e0 = (uint32_t)(t * G::EPT + 2 * p);
#pragma unroll
      for (int k = 0; k < G::Q; ++k) {
        const uint32_t s0 = ((uint32_t)k << G::Kr) | e0;
        cbv[p * G::Q + k] = (uint32_t)cb_state_bits(cb, s0) |
                            ((uint32_t)cb_state_bits(cb, s0 + 1) << 16);
      }
    }
  } else {
    const uint32_t P = (uint32_t)(t / G::R), r = (uint32_t)(t % G::R);
    const uint32_t e0 = 2 * P;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const uint32_t k = 64 * r + j;
      const uint32_t s0 = (k << G::Kr) | e0;
      cbv[j] = (uint32_t)cb_state_bits(cb, s0) |
               ((uint32_t)cb_state_bits(cb, s0 + 1) << 16);
    }
  }
}

// Backpointer storage modes.
enum BpMode { BP_NONE = 0, BP_PRED16 = 2 };

// One ACS step for K <= 6: thread owns NP adjacent edge pairs and all Q
// branches of each.
//   FIRST : step 0 (no accumulated cost; optional wrap mask on pred)
//   BPM   : what to record for the traceback
//   EXACT : compare-and-select on every branch (NaN-faithful)
template <int K, bool FIRST, int BPM, bool EXACT>
__device__ __forceinline__ void step_pairs(const uint32_t (&cbv)[64], uint32_t w2,
                                           const uint16_t* __restrict__ cin,
                                           uint16_t* __restrict__ cout,
                                           void* __restrict__ bp_step, int t,
                                           int pre_state) {
  using G = Geo<K>;
#pragma unroll
  for (int c = 0; c < G::NCH; ++c) {
    const int e_base = t * G::EPT + 2 * c * G::CP;
    const int g_base = e_base >> K;
    constexpr int PCW = (G::CG + 1) / 2;
    uint32_t pc[G::Q][PCW];
    if constexpr (!FIRST) {
#pragma unroll
      for (int k = 0; k < G::Q; ++k) {
        const uint16_t* src = cin + (k << G::GB) + g_base;
        if constexpr (G::CG == 8) {
          const uint4 v = *reinterpret_cast<const uint4*>(src);
          pc[k][0] = v.x; pc[k][1] = v.y; pc[k][2] = v.z; pc[k][3] = v.w;
        } else if constexpr (G::CG == 4) {
          const uint2 v = *reinterpret_cast<const uint2*>(src);
          pc[k][0] = v.x; pc[k][1] = v.y;
        } else if constexpr (G::CG == 2) {
          pc[k][0] = *reinterpret_cast<const uint32_t*>(src);
        } else {
          pc[k][0] = (uint32_t)(*src);
        }
      }
    }
    uint32_t res[G::CP];
#pragma unroll
    for (int p = 0; p < G::CP; ++p) {
      const int gi = (G::CG == 1) ? 0 : ((2 * p) >> K);
      const int pp = c * G::CP + p;  // pair index within the thread
      uint32_t best = 0, idx = 0;
#pragma unroll
      for (int k = 0; k < G::Q; ++k) {
        uint32_t P = 0;
        if constexpr (!FIRST) {
          const uint32_t word = pc[k][gi >> 1];
          P = (gi & 1) ? h2_hi2(word) : h2_lo2(word);
        }
        const uint32_t d = h2_sub(cbv[pp * G::Q + k], w2);
        uint32_t cst = h2_fma(d, d, P);
        if constexpr (FIRST) {
          if (pre_state >= 0) {
            const int g = (e_base + 2 * p) >> K;
            cst = (((k << G::GB) | g) == pre_state) ? cst : kHInf2;
          }
        }
        if (k == 0) {
          best = cst;
        } else if constexpr (BPM != BP_NONE || EXACT) {
          const uint32_t m = h2_lt_mask(cst, best);
          best = EXACT ? bsel(m, cst, best) : h2_min(best, cst);
          if constexpr (BPM != BP_NONE) idx = bsel(m, kconst(k), idx);
        } else {
          best = h2_min(best, cst);
        }
      }
      res[p] = best;
      if constexpr (BPM == BP_PRED16) {
        const uint32_t g = (uint32_t)((e_base + 2 * p) >> K);
        reinterpret_cast<uint32_t*>(bp_step)[(e_base >> 1) + p] =
            (idx << G::GB) | (g | (g << 16));
      }
    }
    // results: CP packed pairs at edges [e_base, e_base + 2*CP)
    uint32_t* dst = reinterpret_cast<uint32_t*>(cout + e_base);
    if constexpr (G::CP >= 4) {
#pragma unroll
      for (int q = 0; q < G::CP / 4; ++q)
        reinterpret_cast<uint4*>(dst)[q] =
            make_uint4(res[4 * q], res[4 * q + 1], res[4 * q + 2], res[4 * q + 3]);
    } else if constexpr (G::CP == 2) {
      *reinterpret_cast<uint2*>(dst) = make_uint2(res[0], res[1]);
    } else {
      dst[0] = res[0];
    }
  }
}

// One ACS step for K >= 7: each edge pair is shared by R lanes, each lane
// scanning 64 consecutive branches; lanes combine with warp shuffles, the
// lower branch range winning ties (equivalent to one ascending scan).
template <int K, bool FIRST, int BPM, bool EXACT>
__device__ __forceinline__ void step_split(const uint32_t (&cbv)[64], uint32_t w2,
                                           const uint16_t* __restrict__ cin,
                                           uint16_t* __restrict__ cout,
                                           void* __restrict__ bp_step, int t,
                                           int pre_state) {
  using G = Geo<K>;
  const int P = t / G::R, r = t % G::R;
  const int g = (2 * P) >> K;
  const int k0 = 64 * r;
  uint32_t best = kHInf2, idx = kconst(k0);
#pragma unroll
  for (int j8 = 0; j8 < 8; ++j8) {
    uint32_t pc[8];
    if constexpr (!FIRST) {
      if constexpr (G::GB == 0) {
        const uint4 v = *reinterpret_cast<const uint4*>(cin + k0 + 8 * j8);
        pc[0] = v.x & 0xFFFFu; pc[1] = v.x >> 16; pc[2] = v.y & 0xFFFFu; pc[3] = v.y >> 16;
        pc[4] = v.z & 0xFFFFu; pc[5] = v.z >> 16; pc[6] = v.w & 0xFFFFu; pc[7] = v.w >> 16;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) pc[j] = cin[((k0 + 8 * j8 + j) << G::GB) | g];
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int jj = 8 * j8 + j;
      const int k = k0 + jj;
      const uint32_t P2 = FIRST ? 0u : h2_lo2(pc[j]);
      const uint32_t d = h2_sub(cbv[jj], w2);
      uint32_t cst = h2_fma(d, d, P2);
      if constexpr (FIRST) {
        if (pre_state >= 0) cst = (((k << G::GB) | g) == pre_state) ? cst : kHInf2;
      }
      if (jj == 0) {
        // lane r = 0 seeds with branch 0 unconditionally (a NaN there sticks);
        // the other lanes start from +inf and only take strictly smaller costs
        const uint32_t m = h2_lt_mask(cst, best) | ((r == 0) ? 0xFFFFFFFFu : 0u);
        best = bsel(m, cst, best);
        if constexpr (BPM != BP_NONE) idx = bsel(m, kconst(k), idx);
      } else if constexpr (BPM != BP_NONE || EXACT) {
        const uint32_t m = h2_lt_mask(cst, best);
        best = EXACT ? bsel(m, cst, best) : h2_min(best, cst);
        if constexpr (BPM != BP_NONE) idx = bsel(m, kconst(k), idx);
      } else {
        best = h2_min(best, cst);
      }
    }
  }
#pragma unroll
  for (int off = 1; off < G::R; off <<= 1) {
    const uint32_t ob = __shfl_xor_sync(0xFFFFFFFFu, best, off);
    const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, idx, off);
    const bool upper = (r & off) != 0;
    const uint32_t lo_c = upper ? ob : best, hi_c = upper ? best : ob;
    const uint32_t lo_i = upper ? oi : idx, hi_i = upper ? idx : oi;
    const uint32_t m = h2_lt_mask(hi_c, lo_c);
    best = bsel(m, hi_c, lo_c);
    idx = bsel(m, hi_i, lo_i);
  }
  if (r == 0) {
    reinterpret_cast<uint32_t*>(cout)[P] = best;
    if constexpr (BPM == BP_PRED16) {
      reinterpret_cast<uint32_t*>(bp_step)[P] =
          (idx << G::GB) | ((uint32_t)g | ((uint32_t)g << 16));
    }
  }
}

template <int K, bool FIRST, int BPM, bool EXACT>
__device__ __forceinline__ void acs_step(const uint32_t (&cbv)[64], uint32_t w2,
                                         const uint16_t* cin, uint16_t* cout,
                                         void* bp_step, int t, int pre_state) {
  if constexpr (Geo<K>::SPLIT)
    step_split<K, FIRST, BPM, EXACT>(cbv, w2, cin, cout, bp_step, t, pre_state);
  else
    step_pairs<K, FIRST, BPM, EXACT>(cbv, w2, cin, cout, bp_step, t, pre_state);
}

// Shared-memory layout of an ACS CTA.
template <int K>
struct Smem {
  static constexpr size_t costs = 2ull * Geo<K>::S * sizeof(uint16_t);
  static constexpr size_t tile = 256 * sizeof(uint32_t);
  static constexpr size_t bytes = costs + tile;
};

// Load one tile: fp32 -> fp16 (round to nearest even), stored as {w, w}.
// Returns nonzero (CTA-uniform) when any element is NaN.
__device__ __forceinline__ int load_tile(const float* __restrict__ src, int L,
                                         uint32_t* wt, int t) {
  int nan = 0;
  for (int i = t; i < L; i += kNT) {
    const __half h = __float2half_rn(src[i]);
    const uint32_t b = __half_as_ushort(h);
    nan |= __hisnan(h) ? 1 : 0;
    wt[i] = b | (b << 16);
  }
  return __syncthreads_or(nan);
}

// ---------------------------------------------------------------------------
// Reference-layout split passes (int16 predecessors, every step recorded).
// ---------------------------------------------------------------------------
template <int K>
__global__ void __launch_bounds__(kNT, 1)
acs_ref_kernel(const float* __restrict__ in, int n, int L, int cb, int roll,
               const int32_t* __restrict__ pre_states, int16_t* __restrict__ temp_edges,
               uint16_t* __restrict__ temp_costs, int cost_slot) {
  using G = Geo<K>;
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t* cbuf0 = reinterpret_cast<uint16_t*>(smem);
  uint16_t* cbuf1 = cbuf0 + G::S;
  uint32_t* wt = reinterpret_cast<uint32_t*>(smem + Smem<K>::costs);
  const int t = threadIdx.x;
  uint32_t cbv[64];
  init_codebook<K>(cbv, cb, t);
  for (int tile = blockIdx.x; tile < n; tile += gridDim.x) {
    load_tile(in + (size_t)tile * L, L, wt, t);
    int16_t* te = temp_edges + (size_t)tile * L * G::S;
    const int pre = pre_states[tile];
    const int r0 = roll % L;
    acs_step<K, true, BP_PRED16, true>(cbv, wt[r0], nullptr, cbuf0, te + (size_t)r0 * G::S,
                                       t, pre);
    __syncthreads();
    for (int i = 1; i < L; ++i) {
      int ri = i + roll;
      if (ri >= L) ri -= L;
      const uint16_t* cin = (i & 1) ? cbuf0 : cbuf1;
      uint16_t* cout = (i & 1) ? cbuf1 : cbuf0;
      acs_step<K, false, BP_PRED16, true>(cbv, wt[ri], cin, cout, te + (size_t)ri * G::S,
                                          t, -1);
      __syncthreads();
    }
    const uint16_t* final_buf = ((L - 1) & 1) ? cbuf1 : cbuf0;
    uint16_t* dst = temp_costs + ((size_t)tile * 2 + cost_slot) * G::S;
    for (int e = t; e < G::S; e += kNT) dst[e] = final_buf[e];
    __syncthreads();
  }
}

__global__ void ref_backward_kernel(const uint16_t* __restrict__ temp_costs,
                                    const int16_t* __restrict__ temp_edges,
                                    float* __restrict__ out_w, int16_t* __restrict__ out_idx,
                                    int32_t* __restrict__ end_states, int n, int K, int cb,
                                    int L, int roll, int cost_slot, int write_output) {
  const int tile = blockIdx.x * blockDim.x + threadIdx.x;
  if (tile >= n) return;
  const int S = 65536 >> K;
  const int16_t* te = temp_edges + (size_t)tile * L * S;
  if (!write_output) {
    const uint16_t* c = temp_costs + ((size_t)tile * 2 + cost_slot) * S;
    uint32_t key = 0xFFFFFFFFu;
    for (int e = 0; e < S; ++e) {
      const uint32_t b = c[e];
      if ((b & 0x7C00u) != 0x7C00u) key = min(key, (b << 16) | (uint32_t)e);
    }
    int edge = key == 0xFFFFFFFFu ? 0 : (int)(key & 0xFFFFu);
    for (int i = L - 1; i >= 0; --i) {
      int ri = i + roll;
      if (ri >= L) ri -= L;
      edge = (uint16_t)te[(size_t)ri * S + edge];
      if (ri == 0) break;
    }
    end_states[tile] = edge;
  } else {
    int edge = end_states[tile];
    for (int i = L - 1; i >= 0; --i) {
      int ri = i + roll;
      if (ri >= L) ri -= L;
      const int prev = (uint16_t)te[(size_t)ri * S + edge];
      const uint16_t s = (uint16_t)((prev << K) | edge);
      edge = prev;
      out_idx[(size_t)tile * L + ri] = (int16_t)s;
      out_w[(size_t)tile * L + ri] = half_bits_to_float(cb_state_bits(cb, s));
    }
  }
}

__global__ void decode_codebook_kernel(int cb, uint16_t* __restrict__ out) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s < 65536) out[s] = cb_state_bits(cb, (uint32_t)s);
}

// One thread per span: its 16 states come in as two 16-byte loads (a warp
// reads two tiles' states, 1 KiB, contiguously), its K packed words go to a
// warp-private shared buffer in storage (SWAP16) order, and the warp writes
// its two tiles' containers with coalesced 32-bit stores.
constexpr int kPackThreads = 256;

template <int K>
__global__ void __launch_bounds__(kPackThreads)
pack_kernel(const int16_t* __restrict__ states, uint32_t* __restrict__ packed, int64_t n) {
  __shared__ uint16_t words[kPackThreads / 32][2 * 16 * K];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int64_t tile0 = ((int64_t)blockIdx.x * (kPackThreads / 32) + warp) * 2;
  const int nt = (int)(n - tile0 < 2 ? n - tile0 : 2);
  if (nt <= 0) return;
  const int tt = lane >> 4, sp = lane & 15;
  if (tt < nt) {
    const uint4* src = reinterpret_cast<const uint4*>(states + (tile0 + tt) * 256 + 16 * sp);
    const uint4 a = src[0], b = src[1];
    const uint32_t st[16] = {a.x & 0xFFFFu, a.x >> 16, a.y & 0xFFFFu, a.y >> 16,
                             a.z & 0xFFFFu, a.z >> 16, a.w & 0xFFFFu, a.w >> 16,
                             b.x & 0xFFFFu, b.x >> 16, b.y & 0xFFFFu, b.y >> 16,
                             b.z & 0xFFFFu, b.z >> 16, b.w & 0xFFFFu, b.w >> 16};
    uint32_t w[K];
    span_words<K>(st, w);
#pragma unroll
    for (int j = 0; j < K; ++j) words[warp][tt * 16 * K + ((sp * K + j) ^ 1)] = (uint16_t)w[j];
  }
  __syncwarp();
  const uint32_t* wsm = reinterpret_cast<const uint32_t*>(words[warp]);
  for (int i = lane; i < nt * 8 * K; i += 32) packed[tile0 * 8 * K + i] = wsm[i];
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

inline size_t tile_ws_bytes(int K, int L) {
  return K >= 2 ? pair_tile_ws_bytes(K, L) : single_tile_ws_bytes(L);
}

int validate(int K, int cb, int L) {
  EXL3_REQUIRE(K >= 1 && K <= 8, "K must be in 1..8, got %d", K);
  EXL3_REQUIRE(cb >= 0 && cb <= 2, "cb must be 0, 1 or 2, got %d", cb);
  EXL3_REQUIRE(L == 256 || L == 160, "tile length L must be 256 or 160, got %d", L);
  EXL3_REQUIRE(L != 160 || cb == 2, "tile length L=160 is only supported with mul1 (cb=2)");
  return EXL3_OK;
}

template <int K>
int set_smem_attrs() {
  static DeviceBits done;
  int dev = 0;
  EXL3_CUDA(cudaGetDevice(&dev));
  if (done.has(dev)) return EXL3_OK;
  const int bytes = (int)Smem<K>::bytes;
  EXL3_CUDA(cudaFuncSetAttribute(acs_ref_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.set(dev);
  return EXL3_OK;
}

template <int K>
int forward_ref_layout(const float* in, uint16_t* temp_costs, int16_t* temp_edges,
                       const int32_t* pre_states, int64_t n, int cb, int L, int roll,
                       int cost_slot, cudaStream_t stream) {
  int rc = set_smem_attrs<K>();
  if (rc) return rc;
  const int sms = sm_count();
  const int grid = n < sms ? (int)n : sms;
  acs_ref_kernel<K><<<grid, kNT, Smem<K>::bytes, stream>>>(
      in, (int)n, L, cb, roll, pre_states, temp_edges, temp_costs, cost_slot);
  EXL3_LAUNCHED();
  return EXL3_OK;
}

}  // namespace
}  // namespace exl3

using namespace exl3;

#define EXL3_DISPATCH_K(K, FN, ...)                     \
  switch (K) {                                          \
    case 1: return FN<1>(__VA_ARGS__);                  \
    case 2: return FN<2>(__VA_ARGS__);                  \
    case 3: return FN<3>(__VA_ARGS__);                  \
    case 4: return FN<4>(__VA_ARGS__);                  \
    case 5: return FN<5>(__VA_ARGS__);                  \
    case 6: return FN<6>(__VA_ARGS__);                  \
    case 7: return FN<7>(__VA_ARGS__);                  \
    case 8: return FN<8>(__VA_ARGS__);                  \
    default: set_error("K must be in 1..8, got %d", K); \
      return EXL3_EINVAL;                               \
  }

extern "C" int exl3_decode_codebook(int cb, uint16_t* out_lut, exl3_stream_t stream) {
  EXL3_REQUIRE(cb >= 0 && cb <= 2, "cb must be 0, 1 or 2, got %d", cb);
  EXL3_REQUIRE(out_lut != nullptr, "out_lut is NULL");
  decode_codebook_kernel<<<256, 256, 0, (cudaStream_t)stream>>>(cb, out_lut);
  EXL3_LAUNCHED();
  return EXL3_OK;
}

extern "C" size_t exl3_quantize_tiles_ws_bytes(int64_t n, int K, int L) {
  if (K < 1 || K > 8 || n < 0 || (L != 256 && L != 160)) return 0;
  // K >= 2 encodes tiles in pairs: an odd count is rounded up to whole pairs
  if (K >= 2) n = (n + 1) & ~(int64_t)1;
  return (size_t)n * tile_ws_bytes(K, L);
}

extern "C" int exl3_quantize_tiles(const float* in, float* out_w, int16_t* out_idx,
                                   int16_t* out_packed, float* out_cost, int64_t n, int K,
                                   int cb, int L, void* ws, size_t ws_bytes,
                                   exl3_stream_t stream) {
  int rc = validate(K, cb, L);
  if (rc) return rc;
  EXL3_REQUIRE(n > 0, "num_tiles must be positive, got %lld", (long long)n);
  EXL3_REQUIRE(n <= (int64_t)1 << 31, "num_tiles %lld too large", (long long)n);
  EXL3_REQUIRE(in && out_w && out_idx, "input/output pointers must be non-NULL");
  EXL3_REQUIRE(ws != nullptr, "workspace is NULL");
  EXL3_REQUIRE(out_packed == nullptr || L == 256, "packed output requires L=256");
  if (K >= 2)
    return pair_encode(K, in, out_w, out_idx, out_packed, out_cost, n, cb, L,
                       static_cast<uint8_t*>(ws), ws_bytes, (cudaStream_t)stream);
  return single_encode(in, out_w, out_idx, out_packed, out_cost, n, cb, L,
                       static_cast<uint8_t*>(ws), ws_bytes, (cudaStream_t)stream);
}

extern "C" int exl3_forward_pass_ref_layout(const float* in, uint16_t* temp_costs,
                                            int16_t* temp_edges, const int32_t* pre_states,
                                            int64_t n, int K, int cb, int L, int roll,
                                            int cost_slot, exl3_stream_t stream) {
  int rc = validate(K, cb, L);
  if (rc) return rc;
  EXL3_REQUIRE(n > 0, "num_tiles must be positive");
  EXL3_REQUIRE(cost_slot == 0 || cost_slot == 1, "cost_slot must be 0 or 1");
  EXL3_REQUIRE(roll >= 0 && roll < L, "roll must be in [0, L)");
  EXL3_REQUIRE(in && temp_costs && temp_edges && pre_states, "NULL pointer argument");
  EXL3_DISPATCH_K(K, forward_ref_layout, in, temp_costs, temp_edges, pre_states, n, cb, L,
                  roll, cost_slot, (cudaStream_t)stream);
}

extern "C" int exl3_backward_pass_ref_layout(const uint16_t* temp_costs,
                                             const int16_t* temp_edges, float* out_w,
                                             int16_t* out_idx, int32_t* end_states,
                                             int64_t n, int K, int cb, int L, int roll,
                                             int cost_slot, int write_output,
                                             exl3_stream_t stream) {
  int rc = validate(K, cb, L);
  if (rc) return rc;
  EXL3_REQUIRE(n > 0, "num_tiles must be positive");
  EXL3_REQUIRE(cost_slot == 0 || cost_slot == 1, "cost_slot must be 0 or 1");
  EXL3_REQUIRE(roll >= 0 && roll < L, "roll must be in [0, L)");
  EXL3_REQUIRE(temp_costs && temp_edges && end_states, "NULL pointer argument");
  EXL3_REQUIRE(!write_output || (out_w && out_idx), "outputs required when write_output");
  ref_backward_kernel<<<(int)((n + 127) / 128), 128, 0, (cudaStream_t)stream>>>(
      temp_costs, temp_edges, out_w, out_idx, end_states, (int)n, K, cb, L, roll, cost_slot,
      write_output);
  EXL3_LAUNCHED();
  return EXL3_OK;
}

extern "C" int exl3_pack_trellis(const int16_t* states, int16_t* packed, int64_t n, int K,
                                 exl3_stream_t stream) {
  EXL3_REQUIRE(K >= 1 && K <= 8, "K must be in 1..8, got %d", K);
  EXL3_REQUIRE(n > 0 && states && packed, "bad arguments");
  EXL3_REQUIRE(reinterpret_cast<uintptr_t>(states) % 16 == 0, "states must be 16-byte aligned");
  EXL3_REQUIRE(reinterpret_cast<uintptr_t>(packed) % 4 == 0, "packed must be 4-byte aligned");
  const int64_t tiles_per_cta = 2 * (kPackThreads / 32);
  const int64_t blocks = (n + tiles_per_cta - 1) / tiles_per_cta;
  EXL3_REQUIRE(blocks < (1ll << 31), "too many tiles");
  uint32_t* pw = reinterpret_cast<uint32_t*>(packed);
  cudaStream_t s = (cudaStream_t)stream;
  EXL3_SWITCH_K(K, (pack_kernel<KK><<<(unsigned)blocks, kPackThreads, 0, s>>>(states, pw, n)));
  EXL3_LAUNCHED();
  return EXL3_OK;
}

extern "C" int exl3_timing_begin(void) {
  std::lock_guard<std::mutex> g(g_timing_mu);
  for (auto& t : g_timed) {
    cudaEventDestroy(t.start);
    cudaEventDestroy(t.stop);
  }
  g_timed.clear();
  g_timing_on = true;
  return EXL3_OK;
}

extern "C" int exl3_timing_end(double* acs_ms, double* traceback_ms, int64_t* acs_launches,
                               int64_t* total_launches) {
  std::vector<TimedLaunch> v;
  {
    std::lock_guard<std::mutex> g(g_timing_mu);
    g_timing_on = false;
    v.swap(g_timed);
  }
  double a = 0.0, b = 0.0;
  int64_t na = 0;
  int rc = EXL3_OK;
  for (auto& t : v) {
    float ms = 0.f;
    if (cudaEventSynchronize(t.stop) != cudaSuccess ||
        cudaEventElapsedTime(&ms, t.start, t.stop) != cudaSuccess) {
      set_error("timing event failed");
      rc = EXL3_ECUDA;
    }
    if (t.kind == 0) {
      a += ms;
      ++na;
    } else {
      b += ms;
    }
    cudaEventDestroy(t.start);
    cudaEventDestroy(t.stop);
  }
  if (acs_ms) *acs_ms = a;
  if (traceback_ms) *traceback_ms = b;
  if (acs_launches) *acs_launches = na;
  if (total_launches) *total_launches = (int64_t)v.size();
  return rc;
}
