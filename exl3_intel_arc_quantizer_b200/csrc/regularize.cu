// Weight regularization and the block-LDL fold on the device.
//
// Regularization (reference exl3_quant/regularize.py:83-211, the order of
// upstream quantize.py:1130-1236) of a (k, n) fp32 weight W, in seven
// launches and no host round trip:
//   reg_skew_kernel      skew = (sum of the k/50 largest sqrt(H_ii)) / (sum of
//                        all), by a radix select over the float bits (one CTA)
//   reg_colsq_kernel     sum of W^2 over each 32-row slice of each column
//   reg_colrms_kernel    column RMS (slices added in order)
//   reg_colfinal_kernel  their mean, the output-scale decision, sv and the
//                        column divisors (one CTA)
//   reg_right_kernel     W / sv, then the 128-column Hadamard of each row (the
//                        shared FWHT), plus each row's sum of squares over
//                        each 32-column slice
//   reg_rowfinal_kernel  row RMS (slices added in order) and su
//   reg_left_kernel      work / su, then the 128-row Hadamard (four threads
//                        per column, no shared memory)
// The reference's sums (torch reductions) have their own order; here every
// slice sum is one fixed order and the slices are added in the reference's
// slice order, so results agree to fp32 rounding.
//
// Block-LDL fold (reference exl3_quant/ldlq.py:96-117): with C the Cholesky
// factor of H and D_b its 16x16 diagonal blocks, L[:, b] = C[:, b] D_b^-1
// and the diagonal blocks become identities. ldl_inv_kernel inverts every
// (lower-triangular) D_b once by forward substitution; ldl_fold_kernel, one
// CTA per 64 x 64 tile of L, multiplies its rows by the four inverses of its
// block columns; tiles above the diagonal are zeros.
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

// skew factor of sqrt(diag(H)): one CTA of 1024 threads
__global__ void __launch_bounds__(1024) reg_skew_kernel(const float* __restrict__ hdiag,
                                                        int64_t stride, int64_t d,
                                                        RegInfo* __restrict__ info) {
  __shared__ unsigned int hist[256];
  __shared__ float red[32];
  __shared__ uint32_t sel[2];  // digit prefix, remaining count
  const int t = threadIdx.x;
  const int64_t want = d / kSkewFraction;
  uint32_t prefix = 0u, mask = 0u;
  int64_t remaining = want;
  for (int shift = 24; shift >= 0 && want > 0; shift -= 8) {
    for (int i = t; i < 256; i += blockDim.x) hist[i] = 0u;
    __syncthreads();
    for (int64_t i = t; i < d; i += blockDim.x) {
      const uint32_t key = __float_as_uint(sqrtf(hdiag[i * stride]));
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (t == 0) {
      int64_t rem = remaining;
      int digit = 255;
      for (; digit > 0; --digit) {
        if ((int64_t)hist[digit] >= rem) break;
        rem -= hist[digit];
      }
      sel[0] = (uint32_t)digit;
      sel[1] = (uint32_t)rem;
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
    const float v = sqrtf(hdiag[i * stride]);
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

// Column RMS: the 32-row slice sums of a column added in slice order
__global__ void reg_colrms_kernel(const float* __restrict__ partial, int64_t nb, int64_t k,
                                  int64_t n, float* __restrict__ out_scales) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  float acc = partial[c];
  for (int64_t b = 1; b < nb; ++b) acc = __fadd_rn(acc, partial[b * n + c]);
  out_scales[c] = sqrtf(__fdiv_rn(acc, (float)k));
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
  float v[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) v[q] = __fdiv_rn(src[lane + 32 * q], dv[lane + 32 * q]);
  fwht128_warp(v, lane);
  float* dst = work + row * n + blk * 128;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    v[q] = __fmul_rn(v[q], kHad128Scale);
    dst[lane + 32 * q] = v[q];
    float s = __fmul_rn(v[q], v[q]);
    for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, o));
    if (lane == 0) rpart[(blk * 4 + q) * k + row] = s;
  }
}

// Row RMS (the 32-column slices added in order) and su
// (regularize.py:187-190): su = su_in * rms / -1.24371088 + 1e-10
__global__ void reg_rowfinal_kernel(const float* __restrict__ rpart, int64_t ns, int64_t k,
                                    int64_t n, const float* __restrict__ su_in,
                                    float* __restrict__ in_scales, float* __restrict__ su_out) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= k) return;
  float acc = rpart[row];
  for (int64_t s = 1; s < ns; ++s) acc = __fadd_rn(acc, rpart[s * k + row]);
  float rms = sqrtf(__fdiv_rn(acc, (float)n));
  if (fabsf(rms) < 1e-30f) rms = kRegZeroFloor;
  in_scales[row] = rms;
  su_out[row] = __fadd_rn(__fdiv_rn(__fmul_rn(su_in[row], rms), kCodebookScale), kRegEps);
}

// work = H128 (work / su) on 128-row blocks: a CTA of 256 threads takes 64
// columns of one row block, four threads per column (had_left_quad_cols)
__global__ void __launch_bounds__(256, 2) reg_left_kernel(float* __restrict__ work,
                                                          const float* __restrict__ su,
                                                          int64_t k, int64_t n) {
  const int t = threadIdx.x;
  const int64_t c = (int64_t)blockIdx.x * 64 + (t >> 2);
  const bool valid = c < n;
  had_left_quad_cols<true>(work + (int64_t)blockIdx.y * 128 * n + (valid ? c : 0), n,
                           su + (int64_t)blockIdx.y * 128, t & 3, valid);
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
// one CTA per 64 x 64 tile (4 block columns); n % 16 == 0.
__global__ void __launch_bounds__(256) ldl_fold_kernel(const float* __restrict__ chol,
                                                       float* __restrict__ L,
                                                       const float* __restrict__ inverses,
                                                       int64_t n) {
  __shared__ float X[4][16][17];  // D_g^-1 of the tile's block columns g = 0..3
  __shared__ float T[64][65];     // the tile of C
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
    T[r][c] = v.x;
    T[r][c + 1] = v.y;
    T[r][c + 2] = v.z;
    T[r][c + 3] = v.w;
  }
  for (int i = t; i < 4 * 256; i += 256) {
    const int g = i >> 8, e = i & 255;
    if (16 * g < cols) X[g][e >> 4][e & 15] = inverses[((c0 >> 4) + g) * 256 + e];
  }
  __syncthreads();
  const int r = t >> 2, g = t & 3;  // row r, block column g: 16 outputs
  if (r >= rows || 16 * g >= cols) return;
  float o[16];
  const int64_t grow = r0 + r, gblk = (c0 >> 4) + g;
  if ((grow >> 4) < gblk) {
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = 0.f;
  } else if ((grow >> 4) == gblk) {
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = (j == (int)(grow & 15)) ? 1.f : 0.f;
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) acc = fmaf(T[r][16 * g + i], X[g][i][j], acc);
      o[j] = acc;
    }
  }
  float4* dst = reinterpret_cast<float4*>(L + grow * n + c0 + 16 * g);
#pragma unroll
  for (int q = 0; q < 4; ++q) dst[q] = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
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
    reg_skew_kernel<<<1, 1024, 0, s>>>(h_diag, h_diag_stride, k, inf);
    EXL3_LAUNCHED();
  }
  const int64_t nb = (k + 31) / 32;
  reg_colsq_kernel<<<dim3((unsigned)((n + 255) / 256), (unsigned)nb), 256, 0, s>>>(W, k, n, cp);
  EXL3_LAUNCHED();
  reg_colrms_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(cp, nb, k, n, out_scales);
  EXL3_LAUNCHED();
  reg_colfinal_kernel<<<1, 1024, 0, s>>>(n, sv_in, force_out_scales, q_fallback, has_skew, inf,
                                        out_scales, dv, sv_out);
  EXL3_LAUNCHED();
  const int64_t warps = k * (n / 128);
  reg_right_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(W, dv, work, rp, k, n);
  EXL3_LAUNCHED();
  reg_rowfinal_kernel<<<(unsigned)((k + 255) / 256), 256, 0, s>>>(rp, n / 32, k, n, su_in,
                                                                   in_scales, su_out);
  EXL3_LAUNCHED();
  reg_left_kernel<<<dim3((unsigned)((n + 63) / 64), (unsigned)(k / 128)), 256, 0, s>>>(
      work, su_out, k, n);
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
