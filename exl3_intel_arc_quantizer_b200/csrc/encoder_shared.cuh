// Pieces shared by the single-tile (encoder.cu) and tile-pair (acs_pair.cu)
// encoders: packing epilogue, launch timing, sizes.
#pragma once

#include <mutex>
#include <vector>

#include "common.cuh"

namespace exl3 {

constexpr int kPairNT = 512;  // threads per tile-pair ACS CTA

// Steps between cost checkpoints of the tile-pair encoders (acs_pair.cu,
// acs_cluster.cu): every 2nd step at K = 2 (the traceback recomputes one
// level of 16 ancestors per two-step segment), every step above (measured:
// a stride of 2 at K = 3 and 4 cut the LDLQ tracebacks by 8% but the bulk
// encoder's throughput by 2-4%).
__host__ __device__ constexpr int ck_stride(int K) { return K == 2 ? 2 : 1; }
constexpr int kTbWarps = 4;   // tiles (warps) per traceback CTA

__device__ __forceinline__ uint32_t kconst(int k) {
  return (uint32_t)k | ((uint32_t)k << 16);
}

// EXL3 container for one 16-element span: low K bits of each state,
// MSB-first, 16 bits per word; written after the SWAP16 half-word exchange
// (trellis_format.py:120-174).
__device__ __forceinline__ void pack_span(const uint16_t* st16, int K, int span,
                                          int16_t* out_tile) {
  uint32_t acc = 0;
  int nb = 0, j = K * span;
  const uint32_t mask = (1u << K) - 1u;
  for (int i = 0; i < 16; ++i) {
    acc = (acc << K) | ((uint32_t)st16[16 * span + i] & mask);
    nb += K;
    if (nb >= 16) {
      out_tile[j ^ 1] = (int16_t)((acc >> (nb - 16)) & 0xFFFFu);
      nb -= 16;
      acc &= (1u << nb) - 1u;
      ++j;
    }
  }
}

// Optional launch timing (diagnostics): when enabled, every encoder launch is
// bracketed by events on its own stream; exl3_timing_end resolves them.
struct TimedLaunch {
  int kind;  // 0 = ACS pass, 1 = traceback
  cudaEvent_t start, stop;
};
extern std::mutex g_timing_mu;
extern bool g_timing_on;
extern std::vector<TimedLaunch> g_timed;

struct LaunchTimer {
  cudaStream_t s;
  int kind;
  cudaEvent_t a = nullptr, b = nullptr;
  LaunchTimer(cudaStream_t stream, int k) : s(stream), kind(k) {
    std::lock_guard<std::mutex> g(g_timing_mu);
    if (!g_timing_on) return;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a, s);
  }
  ~LaunchTimer() {
    if (!a) return;
    cudaEventRecord(b, s);
    std::lock_guard<std::mutex> g(g_timing_mu);
    g_timed.push_back({kind, a, b});
  }
};

// tile-pair encoder (acs_pair.cu)
size_t pair_ck_bytes(int K, int L);       // cost checkpoints of one tile pair
size_t pair_tile_ws_bytes(int K, int L);  // workspace per tile (half a pair + scalars)
// single-tile K = 1 encoder (acs_pair.cu)
size_t single_tile_ws_bytes(int L);
int single_encode(const float* in, float* out_w, int16_t* out_idx, int16_t* out_packed,
                  float* out_cost, int64_t n, int cb, int L, uint8_t* ws, size_t ws_bytes,
                  cudaStream_t stream);
// cluster-split ACS passes for few tile pairs (acs_cluster.cu): the cluster
// size to use for `pairs` pairs at K (1 = the one-CTA-per-pair kernel), and
// one pass (1 or 2) with the tile-pair kernel's arguments and checkpoints
// Cluster split of a call of `pairs` tile pairs: C CTAs per group of P pairs
// (C = 1: no split); cluster_size_for returns its C.
void cluster_choice(int K, int pairs, int* C, int* P);
int cluster_size_for(int K, int pairs);
int cluster_acs_pass(int K, int C, int P, int pass, cudaStream_t stream, const float* in, int n,
                     int L, int cb, uint8_t* ck, size_t ck_pair, int32_t* best_edge,
                     const int32_t* end_state, float* path_cost);
int pair_encode(int K, const float* in, float* out_w, int16_t* out_idx, int16_t* out_packed,
                float* out_cost, int64_t n, int cb, int L, uint8_t* ws, size_t ws_bytes,
                cudaStream_t stream);

}  // namespace exl3
