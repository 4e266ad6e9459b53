// One 16-element span of an EXL3 trellis tile, held by one thread: its 16
// states from the packed words, or its K packed words from the states
// (trellis_format.py:120-174). A tile's 256*K-bit stream is its 16*K packed
// 16-bit words in order, each read MSB-first; element t's state is the
// 16-bit window of the circular stream that ends at bit (t+1)*K. Span s
// (elements 16s..16s+15) therefore reads packed words sK-1 .. sK+K-1 and
// writes words sK .. sK+K-1. With K a template parameter every shift and
// word index below is a compile-time constant.
#pragma once

#include "common.cuh"

namespace exl3 {

// states st[0..15] of span s; word(j) returns packed (not swapped) word j of
// the tile, 0 <= j < 16K
template <int K, class WordFn>
__device__ __forceinline__ void span_states(WordFn word, int s, uint32_t (&st)[16]) {
  uint32_t w[K + 1];
#pragma unroll
  for (int m = 0; m <= K; ++m) {
    int j = s * K - 1 + m;
    if (j < 0) j += 16 * K;
    w[m] = word(j);
  }
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    const int o = (u + 1) * K;  // the window is bits [o, o + 16) of w[0] w[1] ... w[K]
    const int m = o >> 4, sh = o & 15;
    if (sh == 0)
      st[u] = w[m];
    else
      st[u] = (((w[m] << 16) | w[m + 1]) >> (16 - sh)) & 0xFFFFu;
  }
}

// packed words out[0..K-1] (words sK .. sK+K-1 of the tile) from the span's
// states: the low K bits of each, MSB-first
template <int K>
__device__ __forceinline__ void span_words(const uint32_t (&st)[16], uint32_t (&out)[K]) {
  uint32_t acc = 0;
  int nb = 0, j = 0;
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    acc = (acc << K) | (st[u] & ((1u << K) - 1u));
    nb += K;
    if (nb >= 16) {
      out[j++] = (acc >> (nb - 16)) & 0xFFFFu;
      nb -= 16;
      acc &= (1u << nb) - 1u;
    }
  }
}

#define EXL3_SWITCH_K(K, CALL)                \
  switch (K) {                                \
    case 1: { constexpr int KK = 1; CALL; break; } \
    case 2: { constexpr int KK = 2; CALL; break; } \
    case 3: { constexpr int KK = 3; CALL; break; } \
    case 4: { constexpr int KK = 4; CALL; break; } \
    case 5: { constexpr int KK = 5; CALL; break; } \
    case 6: { constexpr int KK = 6; CALL; break; } \
    case 7: { constexpr int KK = 7; CALL; break; } \
    default: { constexpr int KK = 8; CALL; break; } \
  }

}  // namespace exl3
