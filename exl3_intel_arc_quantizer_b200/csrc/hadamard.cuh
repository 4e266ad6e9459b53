// 128-point fast Walsh-Hadamard transform held by one warp: lane l holds
// elements l, l+32, l+64, l+96 in v[0..3]. Sylvester order (the partner of
// element i at stride h is i ^ h; the lower index keeps the sum), strides
// 1..16 across lanes by shuffles, 32 and 64 inside the thread. Every kernel
// that applies the 128-block rotation uses this one function so that the
// rotation rounds identically wherever it runs (reference
// exl3_quant/hadamard.py:94-140 multiplies by H128/sqrt(128) as a GEMM).
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

}  // namespace exl3
