// Library-wide C ABI plumbing: error strings, version, device queries.
#include "common.cuh"

namespace exl3 {

namespace {
thread_local char g_last_error[1024] = "";
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int sm_count() {
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms <= 0)
    sms = 148;
  if (dev >= 0 && dev < 64) cached[dev].store(sms, std::memory_order_relaxed);
  return sms;
}

}  // namespace exl3

extern "C" const char* exl3_last_error(void) { return exl3::g_last_error; }

extern "C" const char* exl3_version(void) { return "exl3k 0.1.0 (sm_100a)"; }

// ---------------------------------------------------------------------------
// fp16x2 FMA issue-rate probe: the denominator of the encoder's roofline
// (packed fp16 ALU, not the tensor pipe). Eight independent fma.rn.f16x2
// chains per thread, full occupancy; timed with events on `stream`.
// ---------------------------------------------------------------------------
namespace exl3 {
__global__ void __launch_bounds__(512) hfma2_probe_kernel(uint32_t* sink, int iters) {
  uint32_t a[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = 0x3C003C00u ^ (threadIdx.x + j);
  const uint32_t b = 0x3BFF3BFFu, c = 0x14001400u;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = h2_fma(a[j], b, c);
    }
  }
  uint32_t x = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) x ^= a[j];
  if (x == 0x12345678u) sink[blockIdx.x] = x;
}
}  // namespace exl3

extern "C" int exl3_probe_fp16x2_rate(double* fp16_ops_per_s, exl3_stream_t stream) {
  using namespace exl3;
  EXL3_REQUIRE(fp16_ops_per_s != nullptr, "output pointer is NULL");
  const int blocks = sm_count() * 4, threads = 512, iters = 16384;
  uint32_t* sink = nullptr;
  cudaEvent_t e0, e1;
  EXL3_CUDA(cudaMallocAsync(&sink, sizeof(uint32_t) * blocks, (cudaStream_t)stream));
  EXL3_CUDA(cudaEventCreate(&e0));
  EXL3_CUDA(cudaEventCreate(&e1));
  hfma2_probe_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>(sink, iters / 8);  // warm-up
  EXL3_CUDA(cudaEventRecord(e0, (cudaStream_t)stream));
  hfma2_probe_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>(sink, iters);
  EXL3_CUDA(cudaEventRecord(e1, (cudaStream_t)stream));
  EXL3_CUDA(cudaEventSynchronize(e1));
  float ms = 0.f;
  EXL3_CUDA(cudaEventElapsedTime(&ms, e0, e1));
  EXL3_CUDA(cudaEventDestroy(e0));
  EXL3_CUDA(cudaEventDestroy(e1));
  EXL3_CUDA(cudaFreeAsync(sink, (cudaStream_t)stream));
  // each fma.rn.f16x2 is two fp16 fused multiply-adds
  const double ops = (double)blocks * threads * iters * 4.0 * 8.0 * 2.0;
  *fp16_ops_per_s = ops / (ms * 1e-3);
  return EXL3_OK;
}

// ---------------------------------------------------------------------------
// fp16 FMA rounding probe (probe_kernels.sycl:45-70): one thread per element
// pair, so mode 0 feeds the two elements through one packed instruction as
// the ACS kernels do.
// ---------------------------------------------------------------------------
namespace exl3 {
__global__ void hfma_probe_kernel(const uint16_t* __restrict__ dh,
                                  const uint16_t* __restrict__ cost, uint16_t* __restrict__ out,
                                  int64_t n, int mode) {
  const int64_t i0 = 2 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
  if (i0 >= n) return;
  const bool two = i0 + 1 < n;
  const uint16_t a0 = dh[i0], c0 = cost[i0];
  const uint16_t a1 = two ? dh[i0 + 1] : (uint16_t)0, c1 = two ? cost[i0 + 1] : (uint16_t)0;
  uint16_t r0, r1;
  if (mode == 0) {
    const uint32_t a = (uint32_t)a0 | ((uint32_t)a1 << 16);
    const uint32_t d = h2_fma(a, a, (uint32_t)c0 | ((uint32_t)c1 << 16));
    r0 = (uint16_t)(d & 0xFFFFu);
    r1 = (uint16_t)(d >> 16);
  } else {
    r0 = h_fma(a0, a0, c0);
    r1 = h_fma(a1, a1, c1);
  }
  out[i0] = r0;
  if (two) out[i0 + 1] = r1;
}
}  // namespace exl3

extern "C" int exl3_probe_hfma(const uint16_t* dh, const uint16_t* cost, uint16_t* out, int64_t n,
                               int mode, exl3_stream_t stream) {
  using namespace exl3;
  EXL3_REQUIRE(mode == 0 || mode == 1, "mode must be 0 (packed fma.rn.f16x2) or 1 (scalar "
               "fma.rn.f16), got %d", mode);
  EXL3_REQUIRE(n >= 0, "n must be >= 0, got %lld", (long long)n);
  if (n == 0) return EXL3_OK;
  EXL3_REQUIRE(dh && cost && out, "dh, cost and out must not be NULL");
  const int threads = 256;
  const int64_t pairs = (n + 1) / 2;
  const int64_t blocks = (pairs + threads - 1) / threads;
  EXL3_REQUIRE(blocks <= 0x7FFFFFFF, "n = %lld is too large", (long long)n);
  hfma_probe_kernel<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(dh, cost, out, n,
                                                                            mode);
  EXL3_LAUNCHED();
  return EXL3_OK;
}
