// Floating-point stages around the encoder on B200: the blockwise 128-point
// Sylvester Hadamard rotation and the Hessian finalize.
//
// Hadamard (reference exl3_quant/hadamard.py:94-119, blockwise_preapply_had_l_/r_):
// the reference multiplies each 128-block by the orthonormal Sylvester matrix
// H128 / sqrt(128) as an fp32 GEMM. Here it is a fast Walsh-Hadamard
// transform: seven exact +/- butterfly stages in fp32 registers followed by
// one scale, reading and writing each element once (HBM-bound; 2 x 4 B per
// element per side).
//
// Hessian finalize (reference exl3_quant/calibration.py:359-407): H /= count,
// diag += max(1e-8, lambda * mean(diag)), diag entries with |d| < floor set to
// floor.
#include "common.cuh"
#include "hadamard.cuh"

namespace exl3 {

namespace {

// x @ H on 128-column blocks: two (row, block) tasks per warp, both tasks'
// loads issued first; lane l holds elements l, l+32, l+64, l+96 of a block.
constexpr int kRightTasks = 2;
__global__ void had_right_kernel(float* __restrict__ x, int64_t k, int64_t n, float scale) {
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t nb = n >> 7, total = k * nb;
  if (warp * kRightTasks >= total) return;
  float v[kRightTasks][4];
  float* p[kRightTasks];
  bool ok[kRightTasks];
#pragma unroll
  for (int j = 0; j < kRightTasks; ++j) {
    const int64_t task = warp * kRightTasks + j;
    ok[j] = task < total;  // the same for every lane of the warp
    p[j] = x + (ok[j] ? (task / nb) * n + (task % nb) * 128 : 0);
#pragma unroll
    for (int q = 0; q < 4; ++q) v[j][q] = ok[j] ? p[j][lane + 32 * q] : 0.f;
  }
#pragma unroll
  for (int j = 0; j < kRightTasks; ++j) fwht128_warp(v[j], lane);
#pragma unroll
  for (int j = 0; j < kRightTasks; ++j) {
    if (!ok[j]) continue;
#pragma unroll
    for (int q = 0; q < 4; ++q) p[j][lane + 32 * q] = v[j][q] * scale;
  }
}

// H @ x on 128-row blocks: a CTA of 256 threads takes 64 columns of one row
// block, four threads per column (had_left_quad_cols). Used when n is odd or
// x is not 8-byte aligned; otherwise had_left_pair_kernel runs.
__global__ void __launch_bounds__(256, 2) had_left_kernel(float* __restrict__ x, int64_t k,
                                                          int64_t n) {
  const int t = threadIdx.x;
  const int64_t c = (int64_t)blockIdx.x * 64 + (t >> 2);
  const bool valid = c < n;
  had_left_quad_cols<false>(x + (int64_t)blockIdx.y * 128 * n + (valid ? c : 0), n, nullptr,
                            t & 3, valid);
}

// The same with two adjacent columns per thread (had_left_pair_cols; n even,
// x 8-byte aligned): a CTA of 256 threads takes 128 columns of one row block.
__global__ void __launch_bounds__(256, 2) had_left_pair_kernel(float* __restrict__ x, int64_t k,
                                                               int64_t n) {
  const int t = threadIdx.x;
  const int64_t c = (int64_t)blockIdx.x * 128 + 2 * (t >> 2);
  const bool valid = c < n;
  had_left_pair_cols<false>(x + (int64_t)blockIdx.y * 128 * n + (valid ? c : 0), n, nullptr,
                            t & 3, valid);
}

// diag mean of H / count (one CTA)
__global__ void hess_diag_mean_kernel(const float* __restrict__ H, int64_t d, double inv_count,
                                      double* __restrict__ out) {
  __shared__ double red[32];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < d; i += blockDim.x) s += (double)H[i * d + i] * inv_count;
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.0;
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    if (threadIdx.x == 0) *out = v / (double)d;
  }
}

// H = H / count; diag += damp; |diag| < floor -> floor. Elementwise over H.
__global__ void hess_finalize_kernel(float* __restrict__ H, int64_t d, float count,
                                     const double* __restrict__ mean_diag, float lambda,
                                     float floor_val, float* __restrict__ damp_out) {
  const float damp = fmaxf(1e-8f, (float)((double)lambda * *mean_diag));
  const int64_t total = d * d;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v = H[i] / count;
    if (i / d == i % d) {
      v += damp;
      if (fabsf(v) < floor_val) v = floor_val;
    }
    H[i] = v;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && damp_out) *damp_out = damp;
}

}  // namespace
}  // namespace exl3

using namespace exl3;

extern "C" int exl3_had128_right(float* x, int64_t k, int64_t n, exl3_stream_t stream) {
  EXL3_REQUIRE(x != nullptr, "x is NULL");
  EXL3_REQUIRE(k > 0 && n > 0 && n % 128 == 0, "columns (%lld) must be a positive multiple of 128",
               (long long)n);
  const int64_t warps = (k * (n / 128) + kRightTasks - 1) / kRightTasks;
  const int threads = 256;
  const int64_t blocks = (warps + 7) / 8;
  EXL3_REQUIRE(blocks < (1ll << 31), "matrix too large");
  had_right_kernel<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(
      x, k, n, 0.08838834764831845f);
  EXL3_LAUNCHED();
  return EXL3_OK;
}

extern "C" int exl3_had128_left(float* x, int64_t k, int64_t n, exl3_stream_t stream) {
  EXL3_REQUIRE(x != nullptr, "x is NULL");
  EXL3_REQUIRE(n > 0 && k > 0 && k % 128 == 0, "rows (%lld) must be a positive multiple of 128",
               (long long)k);
  EXL3_REQUIRE(k / 128 < 65536, "too many row blocks");
  if (n % 2 == 0 && reinterpret_cast<uintptr_t>(x) % 8 == 0) {
    const dim3 grid((unsigned)((n + 127) / 128), (unsigned)(k / 128));
    had_left_pair_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, k, n);
  } else {
    const dim3 grid((unsigned)((n + 63) / 64), (unsigned)(k / 128));
    had_left_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, k, n);
  }
  EXL3_LAUNCHED();
  return EXL3_OK;
}

extern "C" int exl3_hessian_finalize(float* H, int64_t d, int64_t count, float damping_lambda,
                                     float zero_floor, float* damp_out, void* scratch8,
                                     exl3_stream_t stream) {
  EXL3_REQUIRE(H && scratch8, "NULL pointer argument");
  EXL3_REQUIRE(d > 0, "d must be positive");
  if (count < 1) count = 1;
  double* mean = static_cast<double*>(scratch8);
  hess_diag_mean_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(H, d, 1.0 / (double)count, mean);
  EXL3_LAUNCHED();
  const int64_t total = d * d;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  hess_finalize_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      H, d, (float)count, mean, damping_lambda, zero_floor, damp_out);
  EXL3_LAUNCHED();
  return EXL3_OK;
}
