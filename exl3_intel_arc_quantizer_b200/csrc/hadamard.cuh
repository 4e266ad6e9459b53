// 128-point fast Walsh-Hadamard transform held by one warp: lane l holds
// elements l, l+32, l+64, l+96 in v[0..3]. Sylvester order (the partner of
// element i at stride h is i ^ h; the lower index keeps the sum), strides
// 1..16 across lanes by shuffles, 32 and 64 inside the thread. Every helper
// here (and the weight decode's pair-line transform) takes the same
// butterflies in the same order, strides 1, 2, ..., 64, the lower element
// keeping lower + upper, each rounded once, then one scale by 1/sqrt(128),
// so the rotation rounds identically whichever kernel and data layout runs
// it (reference exl3_quant/hadamard.py:94-140 multiplies by H128/sqrt(128)
// as a GEMM).
#pragma once

namespace exl3 {

constexpr float kHad128Scale = 0.08838834764831845f;  // 1/sqrt(128)

// Butterfly across lanes: the lower element keeps mine + other, the upper
// one other - mine, as one fma with a +-1 factor (an exact product, so the
// single rounding is that of the addition or subtraction).
__device__ __forceinline__ float had_bfly(float mine, float other, float sign) {
  return fmaf(sign, mine, other);
}

__device__ __forceinline__ void fwht128_warp(float (&v)[4], int lane) {
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
    const float sign = (lane & h) ? -1.0f : 1.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = had_bfly(v[q], __shfl_xor_sync(0xFFFFFFFFu, v[q], h), sign);
  }
  const float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
  v[0] = a0 + a2;
  v[1] = a1 + a3;
  v[2] = a0 - a2;
  v[3] = a1 - a3;
}

// H128 (x / su) on the columns of one 128-row block, four threads per
// column: thread (c, q) holds rows 4i + q (i < 32) of column c in registers;
// the butterflies of strides 1 and 2 are shuffles with the partner lanes, the
// five wider ones run in registers (the order and roundings of
// fwht128_warp). A warp's loads and stores cover 8 columns of four rows: four
// full 32-byte sectors. DIV: divide by su[row] first (the regularization's
// left step; su best in shared memory); else the plain rotation. Every lane of the
// warp must call it (the shuffles are warp-wide); a lane whose column is past
// the matrix passes valid = false and neither loads nor stores.
template <bool DIV>
__device__ __forceinline__ void had_left_quad_cols(float* __restrict__ col, int64_t n,
                                                   const float* __restrict__ su, int q,
                                                   bool valid) {
  float v[32];
  const int64_t step = 4 * n;
  const float* src = col + (int64_t)q * n;
  // every load is issued before the first division (a division's slow path
  // would otherwise hold back the loads behind it)
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = valid ? *src : 0.f;
    src += step;
  }
  if (DIV) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __fdiv_rn(v[i], su[4 * i + q]);
  }
  const float s1 = (q & 1) ? -1.0f : 1.0f, s2 = (q & 2) ? -1.0f : 1.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = had_bfly(v[i], __shfl_xor_sync(0xFFFFFFFFu, v[i], 1), s1);
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = had_bfly(v[i], __shfl_xor_sync(0xFFFFFFFFu, v[i], 2), s2);
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (i & h) continue;
      const float lo = v[i], hi = v[i + h];
      v[i] = lo + hi;
      v[i + h] = lo - hi;
    }
  }
  if (!valid) return;
  float* dst = col + (int64_t)q * n;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    *dst = __fmul_rn(v[i], kHad128Scale);
    dst += step;
  }
}

// The same transform on two adjacent columns at once: thread (p, q) holds
// rows 4i + q of columns 2p and 2p + 1 as one float2 per row, so each load,
// store and shuffle moves both columns and every butterfly and the scale are
// one packed f32x2 operation (each lane rounds as the scalar operation does:
// fma with a +-1 factor for the shuffle strides, add and fma(hi, -1, lo) for
// the register strides, the order of had_left_quad_cols). A warp covers 16
// columns of four rows per access (64-byte row segments). `col` points at
// column 2p of the block's first row and must be 8-byte aligned with n even.
template <bool DIV>
__device__ __forceinline__ void had_left_pair_cols(float* __restrict__ col, int64_t n,
                                                   const float* __restrict__ su, int q,
                                                   bool valid) {
  float2 v[32];
  const int64_t step = 4 * n;
  const float* src = col + (int64_t)q * n;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = valid ? *reinterpret_cast<const float2*>(src) : make_float2(0.f, 0.f);
    src += step;
  }
  if (DIV) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float s = su[4 * i + q];
      v[i] = make_float2(__fdiv_rn(v[i].x, s), __fdiv_rn(v[i].y, s));
    }
  }
#pragma unroll
  for (int b = 1; b <= 2; b <<= 1) {
    const float sg = (q & b) ? -1.0f : 1.0f;
    const float2 sg2 = make_float2(sg, sg);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const unsigned long long mine = *reinterpret_cast<const unsigned long long*>(&v[i]);
      const unsigned long long theirs = __shfl_xor_sync(0xFFFFFFFFu, mine, b);
      v[i] = __ffma2_rn(sg2, v[i], *reinterpret_cast<const float2*>(&theirs));
    }
  }
  const float2 neg = make_float2(-1.0f, -1.0f);
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (i & h) continue;
      const float2 lo = v[i], hi = v[i + h];
      v[i] = __fadd2_rn(lo, hi);
      v[i + h] = __ffma2_rn(hi, neg, lo);
    }
  }
  if (!valid) return;
  float* dst = col + (int64_t)q * n;
  // an opaque copy of the pointer: the store addresses are stepped afresh
  // instead of 32 load addresses being held through the butterflies
  asm volatile("" : "+l"(dst));
  const float2 sc = make_float2(kHad128Scale, kHad128Scale);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    *reinterpret_cast<float2*>(dst) = __fmul2_rn(v[i], sc);
    dst += step;
  }
}

}  // namespace exl3
