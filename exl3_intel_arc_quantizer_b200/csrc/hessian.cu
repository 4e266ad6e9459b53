// Hessian accumulation H += X^T X on the sm_100a tensor cores.
//
// Reference: exl3_quant/calibration.py:337-352 (HessianCollector._accumulate),
// an fp32 GEMM of the layer's fp16 activations. fp16/bf16 products are exact
// in fp32, so tcgen05 kind::f16 MMAs with fp32 accumulation compute the same
// sums up to summation order.
//
// Design:
//   * one CTA per 128x128 tile of the upper triangle of H (i0 <= j0); the
//     lower triangle is written by mirroring, halving the MMA work;
//   * A = X[:, i0:i0+128]^T and B = X[:, j0:j0+128]^T are both MN-major
//     (X is row-major (tokens, d)), staged into shared memory in the
//     canonical no-swizzle MN-major layout (8 K-rows x 16 B core matrices)
//     by 16-byte cp.async copies, 4 stages of 64 tokens, 2 chunks prefetched;
//   * one thread issues tcgen05.mma (M=128, N=128, K=16) into a 128-column
//     TMEM accumulator; tcgen05.commit arrives on the stage's mbarrier when
//     the MMAs reading that stage are done, which releases it for reuse;
//   * epilogue: tcgen05.ld 32x32b, fused H += acc (and the mirrored block).
// Every mbarrier wait is bounded; on timeout the CTA records an error flag,
// still frees its TMEM and returns.
#include <cuda_bf16.h>

#include "common.cuh"

namespace exl3 {
namespace {

constexpr int kHT = 128;           // tile (M = N)
constexpr int kHK = 64;            // tokens per stage
constexpr int kHStages = 4;        // smem stages
constexpr int kHPD = 2;            // prefetch distance (chunks in flight ahead of the MMA)
constexpr int kHThreads = 128;     // 4 warps: loaders, MMA issuer (thread 0), epilogue
constexpr int kStageBytes = kHT * kHK * 2;   // 16 KiB per operand per stage
constexpr uint32_t kWaitLimit = 1u << 24;    // bounded mbarrier polls (~1 s)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// canonical MN-major, no swizzle: core matrix (8 MN elems x 8 K rows) = 128 B;
// LBO = stride between K-groups, SBO = stride between MN-groups (bytes).
constexpr uint32_t kLBO = 128;                  // K-groups adjacent
constexpr uint32_t kSBO = (kHK / 8) * 128;      // 1024 B per MN-group (8 K-groups)

__device__ __forceinline__ uint64_t make_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((kLBO >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((kSBO >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;                        // descriptor version (sm_100)
  // base offset 0, lbo mode 0, layout type 0 = SWIZZLE_NONE
  return d;
}

// kind::f16 instruction descriptor: D f32, A/B f16 or bf16, both MN-major,
// M = 128, N = 128.
__host__ __device__ constexpr uint32_t make_idesc(int ab_bf16) {
  return (1u << 4)                      // c_format f32
       | ((uint32_t)ab_bf16 << 7)       // a_format
       | ((uint32_t)ab_bf16 << 10)      // b_format
       | (1u << 15)                     // a major = MN
       | (1u << 16)                     // b major = MN
       | ((uint32_t)(kHT >> 3) << 17)   // N >> 3
       | ((uint32_t)(kHT >> 4) << 24);  // M >> 4
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// true when the phase completed, false after kWaitLimit polls
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // 0 source bytes -> 16 zero bytes
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}

// Stage the (tokens t0..t0+64) x (columns c0..c0+128) slab of X into the
// canonical MN-major layout. 1024 chunks of 16 B; lanes cover 8 K-rows x
// 4 MN-groups so each warp's writes hit every bank once per 128 B.
template <typename T>
__device__ __forceinline__ void load_slab(const T* __restrict__ X, int64_t T_tokens, int64_t d,
                                          int64_t t0, int64_t c0, uint32_t sbase, int tid) {
  const int lane = tid & 31, warp = tid >> 5;
  const int r = lane & 7, gsub = lane >> 3;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    // 4 warps x 8 iterations x (8 rows x 4 groups) = 64 rows x 16 groups
    const int idx = it * 4 + warp;          // 0..31
    const int kgrp = idx & 7;               // which 8-token group
    const int ggrp = idx >> 3;              // which 4 MN-groups (0..3)
    const int k = kgrp * 8 + r;             // token within stage
    const int g = ggrp * 4 + gsub;          // MN-group (8 columns)
    const int64_t t = t0 + k;
    const int64_t c = c0 + g * 8;
    const bool valid = (t < T_tokens) && (c < d);
    const T* src = valid ? (X + t * d + c) : X;
    const uint32_t dst = sbase + (uint32_t)g * kSBO + (uint32_t)kgrp * kLBO + (uint32_t)r * 16;
    cp_async16(dst, src, valid);
  }
}

template <typename T, int BF16>
__global__ void __launch_bounds__(kHThreads, 1)
hessian_tc_kernel(const T* __restrict__ X, int64_t T_tokens, int64_t d, float* __restrict__ H,
                  int ntiles_1d, int* __restrict__ err_flag) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint64_t mma_bar[kHStages];
  __shared__ uint32_t tmem_base_slot;
  __shared__ int abort_flag;
  const int tid = threadIdx.x;

  // upper-triangle tile from the linear block index
  int bi = 0, rem = blockIdx.x;
  while (rem >= ntiles_1d - bi) {
    rem -= ntiles_1d - bi;
    ++bi;
  }
  const int bj = bi + rem;
  const int64_t i0 = (int64_t)bi * kHT, j0 = (int64_t)bj * kHT;

  uint8_t* sA = smem;
  uint8_t* sB = smem + kHStages * kStageBytes;

  if (tid == 0) {
    for (int s = 0; s < kHStages; ++s) mbar_init(&mma_bar[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_flag = 0;
  }
  if (tid < 32) {  // warp 0 allocates 128 TMEM columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&tmem_base_slot)), "r"(kHT));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base_slot;

  const int nchunks = (int)((T_tokens + kHK - 1) / kHK);
  const uint32_t idesc = make_idesc(BF16);

  // prologue: the first kHPD chunks
  for (int s = 0; s < kHPD; ++s) {
    if (s < nchunks) {
      const int64_t t0 = (int64_t)s * kHK;
      load_slab<T>(X, T_tokens, d, t0, i0, smem_u32(sA + s * kStageBytes), tid);
      load_slab<T>(X, T_tokens, d, t0, j0, smem_u32(sB + s * kStageBytes), tid);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }

  // Stage s is reused every kHStages chunks; before refilling it for chunk
  // cn the MMAs of chunk cn - kHStages (= c - 2) must be done. Every commit is
  // waited exactly once, in order, so the per-stage parity stays in step.
  uint32_t phase_bits = 0;
  for (int c = 0; c < nchunks; ++c) {
    const int s = c % kHStages;
    const int cn = c + kHPD;
    if (cn < nchunks) {
      const int sn = cn % kHStages;
      if (cn >= kHStages) {
        if (!mbar_wait_bounded(&mma_bar[sn], (phase_bits >> sn) & 1u)) atomicExch(&abort_flag, 1);
        phase_bits ^= (1u << sn);
      }
      const int64_t t0 = (int64_t)cn * kHK;
      load_slab<T>(X, T_tokens, d, t0, i0, smem_u32(sA + sn * kStageBytes), tid);
      load_slab<T>(X, T_tokens, d, t0, j0, smem_u32(sB + sn * kStageBytes), tid);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group %0;" ::"n"(kHPD) : "memory");
    // generic-proxy smem writes -> visible to the tensor core (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (abort_flag) break;
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a0 = smem_u32(sA + s * kStageBytes), b0 = smem_u32(sB + s * kStageBytes);
#pragma unroll
      for (int ks = 0; ks < kHK / 16; ++ks) {
        // K slice of 16 tokens = K-groups 2ks, 2ks+1
        const uint64_t da = make_desc(a0 + ks * 2 * kLBO);
        const uint64_t db = make_desc(b0 + ks * 2 * kLBO);
        const uint32_t accum = (c > 0 || ks > 0) ? 1u : 0u;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(tmem), "l"(da), "l"(db), "r"(idesc), "r"(accum));
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                   ::"r"(smem_u32(&mma_bar[s])) : "memory");
    }
    __syncwarp();
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  // drain: commits of chunks c >= nchunks - kHStages were not waited above
  bool ok = !abort_flag;
  if (ok) {
    const int first = nchunks > kHStages ? nchunks - kHStages : 0;
    for (int c = first; c < nchunks; ++c) {
      const int s = c % kHStages;
      if (!mbar_wait_bounded(&mma_bar[s], (phase_bits >> s) & 1u)) ok = false;
      phase_bits ^= (1u << s);
    }
  }
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  __syncthreads();
  ok = ok && !abort_flag;

  if (ok && nchunks > 0) {
    const int warp = tid >> 5, lane = tid & 31;
    const int64_t row = i0 + warp * 32 + lane;   // TMEM lane = tile row
#pragma unroll 1
    for (int cb = 0; cb < kHT; cb += 32) {
      uint32_t v[32];
      const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)cb;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
          "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
          "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
            "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]),
            "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]),
            "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
            "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
            "=r"(v[30]), "=r"(v[31])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (row < d) {
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          const int64_t col = j0 + cb + q;
          if (col < d) {
            const float a = __uint_as_float(v[q]);
            H[row * d + col] += a;
            if (bi != bj) H[col * d + row] += a;
          }
        }
      }
    }
  }
  if (!ok && tid == 0) atomicExch(err_flag, 1);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (tid < 32)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kHT));
}

constexpr size_t kHSmem = 2ull * kHStages * kStageBytes;  // 128 KiB

}  // namespace
}  // namespace exl3

using namespace exl3;

extern "C" int exl3_hessian_accumulate(float* H, const void* X, int dtype, int64_t T, int64_t d,
                                       int* err_flag, exl3_stream_t stream) {
  EXL3_REQUIRE(H && X && err_flag, "NULL pointer argument");
  EXL3_REQUIRE(dtype == 0 || dtype == 1, "dtype must be 0 (fp16) or 1 (bf16), got %d", dtype);
  EXL3_REQUIRE(d > 0 && d % 8 == 0, "d (%lld) must be a positive multiple of 8", (long long)d);
  EXL3_REQUIRE(T >= 0, "token count must be non-negative");
  EXL3_REQUIRE(reinterpret_cast<uintptr_t>(X) % 16 == 0, "X must be 16-byte aligned");
  if (T == 0) return EXL3_OK;
  const int nt = (int)((d + kHT - 1) / kHT);
  const int64_t ntiles = (int64_t)nt * (nt + 1) / 2;
  EXL3_REQUIRE(ntiles < (1ll << 31), "d too large");
  static uint32_t attr_done[2] = {0u, 0u};  // per dtype, one bit per device
  int dev = 0;
  EXL3_CUDA(cudaGetDevice(&dev));
  const uint32_t bit = dev < 32 ? (1u << dev) : 0u;
  if (dtype == 0) {
    if (!(attr_done[0] & bit)) {
      EXL3_CUDA(cudaFuncSetAttribute(hessian_tc_kernel<__half, 0>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kHSmem));
      attr_done[0] |= bit;
    }
    hessian_tc_kernel<__half, 0><<<(unsigned)ntiles, kHThreads, kHSmem, (cudaStream_t)stream>>>(
        static_cast<const __half*>(X), T, d, H, nt, err_flag);
  } else {
    if (!(attr_done[1] & bit)) {
      EXL3_CUDA(cudaFuncSetAttribute(hessian_tc_kernel<__nv_bfloat16, 1>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kHSmem));
      attr_done[1] |= bit;
    }
    hessian_tc_kernel<__nv_bfloat16, 1><<<(unsigned)ntiles, kHThreads, kHSmem,
                                          (cudaStream_t)stream>>>(
        static_cast<const __nv_bfloat16*>(X), T, d, H, nt, err_flag);
  }
  EXL3_LAUNCHED();
  return EXL3_OK;
}
