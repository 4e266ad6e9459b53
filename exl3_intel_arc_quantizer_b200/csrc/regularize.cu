// Weight regularization and the block-LDL fold on the device.
//
// Regularization (reference exl3_quant/regularize.py:83-211, the order of
// upstream quantize.py:1130-1236) of a (k, n) fp32 weight W, in seven
// launches and no host round trip:
//   reg_skew_kernel      skew = (sum of the k/50 largest sqrt(H_ii)) / (sum of
//                        all), by a radix select over the float bits (one CTA)
//   reg_colsq_kernel     sum of W^2 over each 32-row slice of each column
//   reg_colrms_kernel    column RMS (slice sums added in a fixed order)
//   reg_colfinal_kernel  their mean, the output-scale decision, sv and the
//                        column divisors (one CTA)
//   reg_right_kernel     W / sv, then the 128-column Hadamard of each row (the
//                        shared FWHT), plus each row's sum of squares over
//                        each 32-column slice
//   reg_rowfinal_kernel  row RMS (slice sums added in a fixed order) and su
//   reg_left_kernel      work / su, then the 128-row Hadamard (two adjacent
//                        columns per thread; four threads per column when
//                        work is not 8-byte aligned; no shared memory)
// The reference's sums (torch reductions) have their own order; here every
// sum has one fixed order (32-element slices, then eight interleaved chains
// of slices added in order), so results are deterministic and agree with the
// reference to fp32 rounding.
//
// Block-LDL fold (reference exl3_quant/ldlq.py:96-117): with C the Cholesky
// factor of H and D_b its 16x16 diagonal blocks, L[:, b] = C[:, b] D_b^-1
// and the diagonal blocks become identities. ldl_inv_kernel inverts every
// (lower-triangular) D_b once by forward substitution; ldl_fold_kernel, one
// CTA per 64 x 64 tile of L, multiplies its rows by the four inverses of its
// block columns (inverse columns held in registers); tiles above the
// diagonal are zeros.
#include "common.cuh"
#include "hadamard.cuh"

namespace exl3 {
namespace {

constexpr float kRegEps = 1e-10f;
constexpr float kRegZeroFloor = 0.1f;
constexpr float kCodebookScale = -1.24371088f;   // su divisor (reference CODEBOOK_SCALE, negated)
constexpr double kSkewCutoff = 0.15;             // reference OUT_SCALE_SKEW_CUTOFF
constexpr int kSkewFraction = 50;                // reference SKEW_FRACTION

// info words written by the kernels (device memory the caller reads once)
struct RegInfo {
  int32_t apply_out;  // 1: output scales applied
  int32_t zeros;      // 1: the column RMS mean was <= 1e-30
  float skew;         // NaN when not computed
  float mean;         // column RMS mean
};

__device__ __forceinline__ float block_sum_f(float v, float* red) {
  // sum over the CTA (<= 1024 threads): warp shuffles, then warp 0
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  if (w == 0) {
    s = (l < (int)(blockDim.x >> 5)) ? red[l] : 0.f;
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    if (l == 0) red[0] = s;
  }
  __syncthreads();
  s = red[0];
  __syncthreads();
  return s;
}

// skew factor of sqrt(diag(H)): one CTA of 1024 threads. For d <= kSkewCacheKeys
// the keys sqrt(H_ii) are read from H once (all loads of a thread in flight
// together) into dynamic shared memory, and the four digit passes and the sums
// read them there; larger d re-reads H_ii in every pass. Either way every
// thread visits the same keys in the same order, so the sums are the same.
constexpr int64_t kSkewCacheKeys = 32768;  // 128 KiB of shared memory
__global__ void __launch_bounds__(1024) reg_skew_kernel(const float* __restrict__ hdiag,
                                                        int64_t stride, int64_t d,
                                                        RegInfo* __restrict__ info) {
  extern __shared__ float keys_s[];  // d keys when cached
  __shared__ unsigned int hist[256];
  __shared__ float red[32];
  __shared__ uint32_t sel[2];  // digit prefix, remaining count
  const int t = threadIdx.x;
  const int64_t want = d / kSkewFraction;
  const bool cached = d <= kSkewCacheKeys;
  if (cached) {
#pragma unroll 8
    for (int64_t i = t; i < d; i += blockDim.x) keys_s[i] = sqrtf(hdiag[i * stride]);
    __syncthreads();
  }
  auto key_at = [&](int64_t i) { return cached ? keys_s[i] : sqrtf(hdiag[i * stride]); };
  uint32_t prefix = 0u, mask = 0u;
  int64_t remaining = want;
  for (int shift = 24; shift >= 0 && want > 0; shift -= 8) {
    for (int i = t; i < 256; i += blockDim.x) hist[i] = 0u;
    __syncthreads();
    for (int64_t i = t; i < d; i += blockDim.x) {
      const uint32_t key = __float_as_uint(key_at(i));
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (t < 32) {
      // the digit holding the remaining-th largest key: lane l owns digits
      // 255 - 8l .. 248 - 8l; an exclusive scan over lanes gives the count
      // above each lane's digits, the first lane that reaches `remaining`
      // walks its eight (digit 0 takes whatever is left)
      uint32_t cnt[8], own = 0u;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        cnt[u] = hist[255 - 8 * t - u];
        own += cnt[u];
      }
      uint32_t incl = own;
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (t >= o) incl += y;
      }
      const uint32_t above = incl - own;
      const unsigned hit = __ballot_sync(0xFFFFFFFFu, (int64_t)incl >= remaining);
      const int owner = hit ? __ffs(hit) - 1 : 31;
      if (t == owner) {
        int64_t rem = remaining - (int64_t)above;
        int digit = 255 - 8 * t;
        for (int u = 0; u < 7 && (int64_t)cnt[u] < rem; ++u) {
          rem -= cnt[u];
          --digit;
        }
        sel[0] = (uint32_t)digit;
        sel[1] = (uint32_t)rem;
      }
    }
    __syncthreads();
    prefix |= sel[0] << shift;
    mask |= 255u << shift;
    remaining = sel[1];
    __syncthreads();
  }
  // top = sum of keys above the want-th largest + remaining copies of it
  float top = 0.f, all = 0.f;
  for (int64_t i = t; i < d; i += blockDim.x) {
    const float v = key_at(i);
    all += v;
    if (want > 0 && __float_as_uint(v) > prefix) top += v;
  }
  top = block_sum_f(top, red);
  all = block_sum_f(all, red);
  if (t == 0) {
    if (want > 0) top += (float)remaining * __uint_as_float(prefix);
    info->skew = top / all;
  }
}

// partial[b][c] = sum of W[r][c]^2 over the 32-row slice b
__global__ void reg_colsq_kernel(const float* __restrict__ W, int64_t k, int64_t n,
                                 float* __restrict__ partial) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t b = blockIdx.y;
  if (c >= n) return;
  const int64_t r1 = (b + 1) * 32 < k ? (b + 1) * 32 : k;
  float s = 0.f;
  for (int64_t r = b * 32; r < r1; ++r) {
    const float w = W[r * n + c];
    s = __fadd_rn(s, __fmul_rn(w, w));
  }
  partial[b * n + c] = s;
}

// Sum over s < ns of part[s * stride + x] for the 32 consecutive x of a CTA
// of 32 x 8 threads: thread (x, g) adds the slices s = g, g + 8, ... in order
// (eight loads in flight per step), then the eight chains are added in order
// g = 0..7. Returns the sum in threads with g == 0.
__device__ __forceinline__ float slice_sum_32x8(const float* __restrict__ part, int64_t ns,
                                                int64_t stride, int64_t x, bool valid) {
  __shared__ float chains[8][33];
  const int tx = threadIdx.x & 31, g = threadIdx.x >> 5;
  float acc = 0.f;
  if (valid) {
    int64_t sl = g;
    for (; sl + 56 < ns; sl += 64) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = part[(sl + 8 * u) * stride + x];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, v[u]);
    }
    for (; sl < ns; sl += 8) acc = __fadd_rn(acc, part[sl * stride + x]);
  }
  chains[g][tx] = acc;
  __syncthreads();
  float total = 0.f;
  if (g == 0) {
#pragma unroll
    for (int u = 0; u < 8; ++u) total = __fadd_rn(total, chains[u][tx]);
  }
  return total;
}

// Column RMS from the 32-row slice sums (CTA of 32 columns x 8 chains)
__global__ void __launch_bounds__(256) reg_colrms_kernel(const float* __restrict__ partial,
                                                         int64_t nb, int64_t k, int64_t n,
                                                         float* __restrict__ out_scales) {
  const int64_t c = (int64_t)blockIdx.x * 32 + (threadIdx.x & 31);
  const float acc = slice_sum_32x8(partial, nb, n, c, c < n);
  if (threadIdx.x < 32 && c < n) out_scales[c] = sqrtf(__fdiv_rn(acc, (float)k));
}

// The column RMS mean, the output-scale decision (regularize.py:145-182),
// out_scales, the column divisors of W and sv. One CTA of 1024 threads.
__global__ void __launch_bounds__(1024) reg_colfinal_kernel(
    int64_t n, const float* __restrict__ sv_in, int force, int q_fallback, int has_skew,
    RegInfo* __restrict__ info, float* __restrict__ out_scales, float* __restrict__ divisor,
    float* __restrict__ sv_out) {
  __shared__ float red[32];
  __shared__ int s_apply, s_zeros;
  __shared__ float s_mean;
  const int t = threadIdx.x;
  float local = 0.f;
  for (int64_t c = t; c < n; c += blockDim.x) local += out_scales[c];
  const float sum = block_sum_f(local, red);
  if (t == 0) {
    const float mean = __fdiv_rn(sum, (float)n);
    int apply;
    if (!q_fallback && has_skew)
      apply = force < 0 ? ((double)info->skew < kSkewCutoff ? 1 : 0) : (force ? 1 : 0);
    else
      apply = force < 0 ? 1 : (force ? 1 : 0);
    if (q_fallback) apply = force > 0 ? 1 : 0;
    const int zeros = ((double)mean > 1e-30) ? 0 : 1;
    if (zeros && force >= 0) apply = 1;
    info->apply_out = apply;
    info->zeros = zeros;
    info->mean = mean;
    s_apply = apply;
    s_zeros = zeros;
    s_mean = mean;
  }
  __syncthreads();
  const int apply = s_apply, zeros = s_zeros;
  const float mean = s_mean;
  for (int64_t c = t; c < n; c += blockDim.x) {
    float os = out_scales[c];
    if (!zeros) os = __fdiv_rn(os, mean);
    const bool zero_out = fabsf(os) < 1e-30f;
    if (apply && zero_out) os = kRegZeroFloor;
    const float sv = sv_in[c];
    const float dv = apply ? __fadd_rn(__fmul_rn(sv, os), kRegEps) : sv;
    divisor[c] = dv;
    sv_out[c] = zero_out ? 0.f : dv;
    out_scales[c] = os;
  }
}

// work = (W / divisor) H128 per 128-column block of each row (one warp per
// (row, block)); rpart[s * k + row] = sum of work^2 over 32-column slice s
__global__ void reg_right_kernel(const float* __restrict__ W, const float* __restrict__ divisor,
                                 float* __restrict__ work, float* __restrict__ rpart, int64_t k,
                                 int64_t n) {
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t nb = n >> 7;
  if (warp >= k * nb) return;
  const int64_t row = warp / nb, blk = warp % nb;
  const float* src = W + row * n + blk * 128;
  const float* dv = divisor + blk * 128;
  float v[4], d[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    v[q] = src[lane + 32 * q];
    d[q] = dv[lane + 32 * q];
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) v[q] = __fdiv_rn(v[q], d[q]);
  fwht128_warp(v, lane);
  float* dst = work + row * n + blk * 128;
  float sq[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    v[q] = __fmul_rn(v[q], kHad128Scale);
    dst[lane + 32 * q] = v[q];
    sq[q] = __fmul_rn(v[q], v[q]);
  }
  // the four slice sums by one transposed reduction: at offset 16 a lane
  // keeps two slices (lanes < 16 slices 0, 1, the others 2, 3) and adds its
  // partner's values of them, at offset 8 one slice, then offsets 4, 2, 1.
  // Every slice is summed over the same pairwise tree (lane pairs 16 apart,
  // then 8, 4, 2, 1) as a full warp reduction per slice, so the sums are
  // bit-identical to that, with 6 shuffles instead of 20.
  const bool h16 = lane & 16, h8 = lane & 8;
  float a0 = h16 ? sq[2] : sq[0], a1 = h16 ? sq[3] : sq[1];
  const float g0 = __shfl_xor_sync(0xFFFFFFFFu, h16 ? sq[0] : sq[2], 16);
  const float g1 = __shfl_xor_sync(0xFFFFFFFFu, h16 ? sq[1] : sq[3], 16);
  a0 = __fadd_rn(a0, g0);
  a1 = __fadd_rn(a1, g1);
  float t = h8 ? a1 : a0;
  t = __fadd_rn(t, __shfl_xor_sync(0xFFFFFFFFu, h8 ? a0 : a1, 8));
  for (int o = 4; o; o >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xFFFFFFFFu, t, o));
  // lane 0 holds slice 0, lane 8 slice 1, lane 16 slice 2, lane 24 slice 3
  if ((lane & 7) == 0) rpart[(blk * 4 + (lane >> 3)) * k + row] = t;
}

// Row RMS from the 32-column slice sums (CTA of 32 rows x 8 chains) and su
// (regularize.py:187-190): su = su_in * rms / -1.24371088 + 1e-10
__global__ void __launch_bounds__(256) reg_rowfinal_kernel(
    const float* __restrict__ rpart, int64_t ns, int64_t k, int64_t n,
    const float* __restrict__ su_in, float* __restrict__ in_scales, float* __restrict__ su_out) {
  const int64_t row = (int64_t)blockIdx.x * 32 + (threadIdx.x & 31);
  const float acc = slice_sum_32x8(rpart, ns, k, row, row < k);
  if (threadIdx.x >= 32 || row >= k) return;
  float rms = sqrtf(__fdiv_rn(acc, (float)n));
  if (fabsf(rms) < 1e-30f) rms = kRegZeroFloor;
  in_scales[row] = rms;
  su_out[row] = __fadd_rn(__fdiv_rn(__fmul_rn(su_in[row], rms), kCodebookScale), kRegEps);
}

// work = H128 (work / su) on 128-row blocks: a CTA of 256 threads takes 64
// columns of one row block, four threads per column (had_left_quad_cols).
// Used when work is not 8-byte aligned; otherwise reg_left_pair_kernel runs.
__global__ void __launch_bounds__(256, 2) reg_left_kernel(float* __restrict__ work,
                                                          const float* __restrict__ su,
                                                          int64_t k, int64_t n) {
  __shared__ float su_s[128];
  const int t = threadIdx.x;
  if (t < 128) su_s[t] = su[(int64_t)blockIdx.y * 128 + t];
  __syncthreads();
  const int64_t c = (int64_t)blockIdx.x * 64 + (t >> 2);
  const bool valid = c < n;
  had_left_quad_cols<true>(work + (int64_t)blockIdx.y * 128 * n + (valid ? c : 0), n, su_s,
                           t & 3, valid);
}

// the same with two adjacent columns per thread (had_left_pair_cols; work
// 8-byte aligned): a CTA takes 128 columns of one row block
__global__ void __launch_bounds__(256, 2) reg_left_pair_kernel(float* __restrict__ work,
                                                               const float* __restrict__ su,
                                                               int64_t k, int64_t n) {
  __shared__ float su_s[128];
  const int t = threadIdx.x;
  if (t < 128) su_s[t] = su[(int64_t)blockIdx.y * 128 + t];
  __syncthreads();
  const int64_t c = (int64_t)blockIdx.x * 128 + 2 * (t >> 2);
  const bool valid = c < n;
  had_left_pair_cols<true>(work + (int64_t)blockIdx.y * 128 * n + (valid ? c : 0), n, su_s,
                           t & 3, valid);
}

// D_b^-1 of every 16x16 diagonal block of C (lower triangular) by forward
// substitution: one CTA per four blocks, D staged in shared memory, thread
// (g, j) computes column j of block g's inverse.
__global__ void __launch_bounds__(64) ldl_inv_kernel(const float* __restrict__ chol,
                                                     float* __restrict__ inverses, int64_t m,
                                                     int64_t n) {
  __shared__ float D[4][16][17];
  const int t = threadIdx.x, g = t >> 4, j = t & 15;
  const int64_t b = (int64_t)blockIdx.x * 4 + g;
  if (b < m) {
    const float* src = chol + (b * 16) * n + b * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) D[g][i][j] = src[(int64_t)i * n + j];
  }
  __syncthreads();
  if (b >= m) return;
  float x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = 0.f;
  x[j] = __fdiv_rn(1.f, D[g][j][j]);
  for (int i = j + 1; i < 16; ++i) {
    float acc = 0.f;
    for (int p = j; p < i; ++p) acc = fmaf(D[g][i][p], x[p], acc);
    x[i] = -__fdiv_rn(acc, D[g][i][i]);
  }
  float* out = inverses + b * 256;
#pragma unroll
  for (int i = 0; i < 16; ++i) out[i * 16 + j] = x[i];
}

// L = C D^-1 per 16-column block, identity diagonal blocks, zeros above:
// one CTA per 64 x 64 tile (4 block columns); n % 16 == 0. Thread (g, j, q)
// holds column j of D_g^-1 in registers and computes column 16 g + j of the
// 16 rows of row block q: per row one chain of 16 fmaf (i = 0..15) over the
// row's C entries, read from shared memory four at a time and shared by the
// 16 threads of the block column. A warp stores 32 consecutive columns of one
// row per instruction.
__global__ void __launch_bounds__(256) ldl_fold_kernel(const float* __restrict__ chol,
                                                       float* __restrict__ L,
                                                       const float* __restrict__ inverses,
                                                       int64_t n) {
  __shared__ __align__(16) float T[64][68];  // the tile of C
  const int64_t r0 = (int64_t)blockIdx.y * 64, c0 = (int64_t)blockIdx.x * 64;
  const int t = threadIdx.x;
  const int rows = (int)((n - r0) < 64 ? (n - r0) : 64);
  const int cols = (int)((n - c0) < 64 ? (n - c0) : 64);
  if (c0 > r0) {  // strictly above the block diagonal
    for (int i = t; i < 64 * 16; i += 256) {
      const int r = i >> 4, c = (i & 15) * 4;
      if (r < rows && c < cols)
        *reinterpret_cast<float4*>(L + (r0 + r) * n + c0 + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return;
  }
  for (int i = t; i < 64 * 16; i += 256) {
    const int r = i >> 4, c = (i & 15) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < rows && c < cols) v = *reinterpret_cast<const float4*>(chol + (r0 + r) * n + c0 + c);
    *reinterpret_cast<float4*>(&T[r][c]) = v;
  }
  __syncthreads();
  const int lane = t & 31, w = t >> 5;
  const int j = lane & 15, g = 2 * (w & 1) + (lane >> 4), q = w >> 1;
  if (16 * g >= cols || 16 * q >= rows) return;
  const int64_t gblk = (c0 >> 4) + g, rblk = (r0 >> 4) + q;
  float* dst = L + (r0 + 16 * q) * n + c0 + 16 * g + j;
  if (rblk < gblk) {
#pragma unroll
    for (int rr = 0; rr < 16; ++rr) dst[rr * n] = 0.f;
    return;
  }
  if (rblk == gblk) {
#pragma unroll
    for (int rr = 0; rr < 16; ++rr) dst[rr * n] = (rr == j) ? 1.f : 0.f;
    return;
  }
  float x[16];
  const float* xs = inverses + gblk * 256 + j;
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = xs[16 * i];
#pragma unroll 4
  for (int rr = 0; rr < 16; ++rr) {
    const float4* tr = reinterpret_cast<const float4*>(&T[16 * q + rr][16 * g]);
    float acc = 0.f;
#pragma unroll
    for (int i4 = 0; i4 < 4; ++i4) {
      const float4 a = tr[i4];
      acc = fmaf(a.x, x[4 * i4], acc);
      acc = fmaf(a.y, x[4 * i4 + 1], acc);
      acc = fmaf(a.z, x[4 * i4 + 2], acc);
      acc = fmaf(a.w, x[4 * i4 + 3], acc);
    }
    dst[rr * n] = acc;
  }
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

void reg_layout(int64_t k, int64_t n, size_t* cpart, size_t* div, size_t* rpart, size_t* total) {
  size_t off = 0;
  *cpart = off;
  off = align256(off + (size_t)((k + 31) / 32) * n * 4);
  *div = off;
  off = align256(off + (size_t)n * 4);
  *rpart = off;
  off = align256(off + (size_t)(n / 32) * k * 4);
  *total = off;
}

}  // namespace
}  // namespace exl3

using namespace exl3;

extern "C" size_t exl3_regularize_ws_bytes(int64_t k, int64_t n) {
  if (k <= 0 || n <= 0 || k % 128 || n % 128) return 0;
  size_t a, b, c, total;
  reg_layout(k, n, &a, &b, &c, &total);
  return total;
}

extern "C" int exl3_regularize(const float* W, const float* su_in, const float* sv_in,
                               const float* h_diag, int64_t h_diag_stride,
                               int force_out_scales, int q_fallback, float* work,
                               float* su_out, float* sv_out, float* out_scales,
                               float* in_scales, void* info, int64_t k, int64_t n, void* ws,
                               size_t ws_bytes, exl3_stream_t stream) {
  EXL3_REQUIRE(W && su_in && sv_in && work && su_out && sv_out && out_scales && in_scales && info,
               "NULL pointer argument");
  EXL3_REQUIRE(k > 0 && n > 0 && k % 128 == 0 && n % 128 == 0,
               "both dimensions must be positive multiples of 128, got (%lld, %lld)",
               (long long)k, (long long)n);
  EXL3_REQUIRE(k / 128 < 65536 && (k + 31) / 32 < 65536, "too many rows");
  EXL3_REQUIRE(force_out_scales >= -1 && force_out_scales <= 1,
               "force_out_scales must be -1 (auto), 0 or 1, got %d", force_out_scales);
  EXL3_REQUIRE(!h_diag || h_diag_stride >= 1, "h_diag_stride must be positive");
  EXL3_REQUIRE(work != W, "work must not alias W");
  size_t cpart, div, rpart, total;
  reg_layout(k, n, &cpart, &div, &rpart, &total);
  EXL3_REQUIRE(ws && ws_bytes >= total, "workspace of %zu bytes is smaller than the %zu needed",
               ws_bytes, total);
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* base = static_cast<uint8_t*>(ws);
  float* cp = reinterpret_cast<float*>(base + cpart);
  float* dv = reinterpret_cast<float*>(base + div);
  float* rp = reinterpret_cast<float*>(base + rpart);
  RegInfo* inf = static_cast<RegInfo*>(info);
  EXL3_CUDA(cudaMemsetAsync(inf, 0xFF, sizeof(RegInfo), s));  // skew NaN until computed
  const int has_skew = (h_diag != nullptr && !q_fallback) ? 1 : 0;
  if (has_skew) {
    static DeviceBits attr_done;
    int dev = 0;
    EXL3_CUDA(cudaGetDevice(&dev));
    if (!attr_done.has(dev)) {
      EXL3_CUDA(cudaFuncSetAttribute(reg_skew_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)(kSkewCacheKeys * sizeof(float))));
      attr_done.set(dev);
    }
    const size_t cache = k <= kSkewCacheKeys ? (size_t)k * sizeof(float) : 0;
    reg_skew_kernel<<<1, 1024, cache, s>>>(h_diag, h_diag_stride, k, inf);
    EXL3_LAUNCHED();
  }
  const int64_t nb = (k + 31) / 32;
  reg_colsq_kernel<<<dim3((unsigned)((n + 255) / 256), (unsigned)nb), 256, 0, s>>>(W, k, n, cp);
  EXL3_LAUNCHED();
  reg_colrms_kernel<<<(unsigned)((n + 31) / 32), 256, 0, s>>>(cp, nb, k, n, out_scales);
  EXL3_LAUNCHED();
  reg_colfinal_kernel<<<1, 1024, 0, s>>>(n, sv_in, force_out_scales, q_fallback, has_skew, inf,
                                        out_scales, dv, sv_out);
  EXL3_LAUNCHED();
  const int64_t warps = k * (n / 128);
  reg_right_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(W, dv, work, rp, k, n);
  EXL3_LAUNCHED();
  reg_rowfinal_kernel<<<(unsigned)((k + 31) / 32), 256, 0, s>>>(rp, n / 32, k, n, su_in,
                                                                 in_scales, su_out);
  EXL3_LAUNCHED();
  if (reinterpret_cast<uintptr_t>(work) % 8 == 0) {  // n is a multiple of 128
    reg_left_pair_kernel<<<dim3((unsigned)(n / 128), (unsigned)(k / 128)), 256, 0, s>>>(
        work, su_out, k, n);
  } else {
    reg_left_kernel<<<dim3((unsigned)((n + 63) / 64), (unsigned)(k / 128)), 256, 0, s>>>(
        work, su_out, k, n);
  }
  EXL3_LAUNCHED();
  return EXL3_OK;
}

extern "C" int exl3_block_ldl_fold(const float* chol, float* L, float* inverses, int64_t n,
                                   exl3_stream_t stream) {
  EXL3_REQUIRE(chol && L && inverses, "NULL pointer argument");
  EXL3_REQUIRE(chol != L, "L must not alias the Cholesky factor");
  EXL3_REQUIRE(n > 0 && n % 16 == 0, "n (%lld) must be a positive multiple of 16", (long long)n);
  EXL3_REQUIRE(reinterpret_cast<uintptr_t>(chol) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(L) % 16 == 0,
               "chol and L must be 16-byte aligned");
  const int64_t tiles = (n + 63) / 64;
  EXL3_REQUIRE(tiles < 65536, "matrix too large");
  const int64_t m = n / 16;
  ldl_inv_kernel<<<(unsigned)((m + 3) / 4), 64, 0, (cudaStream_t)stream>>>(chol, inverses, m, n);
  EXL3_LAUNCHED();
  ldl_fold_kernel<<<dim3((unsigned)tiles, (unsigned)tiles), 256, 0, (cudaStream_t)stream>>>(
      chol, L, inverses, n);
  EXL3_LAUNCHED();
  return EXL3_OK;
}
