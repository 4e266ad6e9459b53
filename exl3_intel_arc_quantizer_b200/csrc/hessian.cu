// Hessian accumulation H += X^T X on the sm_100a tensor cores.
//
// Reference: exl3_quant/calibration.py:337-352 (HessianCollector._accumulate),
// an fp32 GEMM of the layer's fp16 activations. fp16/bf16 products are exact
// in fp32, so tcgen05 kind::f16 MMAs with fp32 accumulation compute the same
// sums up to summation order.
//
// Design (one CTA per 128 x 256 tile of H that reaches the upper triangle,
// or per 256 x 256 tile for wide H, see HGeo; 10 warps with fixed roles):
//   * warp 0 (one lane) streams X through TMA: per 64-token chunk, the
//     128-column A slab X[t:t+64, i0:i0+128] and the 256-column B slab
//     X[t:t+64, j0:j0+256] as 64 x 64 boxes with 128-byte swizzle, straight
//     into the canonical MN-major SW128 operand layout; 4 stages of 48 KiB;
//   * warp 1 allocates 512 TMEM columns (two 128 x 256 fp32 accumulators)
//     and one lane issues tcgen05.mma (M=128, N=256, K=16) per 16 tokens;
//     tcgen05.commit frees each stage and, every 8192 tokens (a segment),
//     hands the finished accumulator to the epilogue and switches to the
//     other one;
//   * warps 2-9 (two per TMEM lane quarter, each half of the columns) drain
//     a finished accumulator (tcgen05.ld), stage each 32x32
//     block in shared memory and add its elements (r, c), c >= r, into H
//     with 16-byte red.global.add.v4.f32 (L2 evict-last, so H's lines stay
//     cached between segments), while the MMAs of the next segment run;
//   * hessian_mirror_kernel then copies the upper triangle to the lower one.
// Long calls run as one launch per 65,536-token slab (kSlabTokens).
// Draining every segment bounds the length of each tensor-core accumulation
// chain (its additions are not round-to-nearest, so long chains drift). H is
// symmetric after every call; on entry only its upper triangle is read (the
// lower one is rewritten from it), so H must be symmetric on entry, as any
// sum of earlier calls is. Each element of the upper triangle is updated by
// one thread in a fixed order, so results are deterministic.
// Every wait is bounded by the global timer; a role that gives up records
// the error flag and the others stop at their next wait; the CTA then waits
// (bounded) for its own TMA copies and MMAs before it frees TMEM and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace exl3 {
namespace {

constexpr int kBM = 128;                 // tile rows (i)
constexpr int kBN = 256;                 // tile columns (j)
constexpr int kBK = 64;                  // tokens per stage
constexpr int kStages = 4;
constexpr int kSegChunks = 128;          // 8192 tokens per accumulator segment
constexpr int kEpiWarps = 8;            // two per TMEM lane quarter
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr int kABytes = kBM * kBK * 2;   // 16 KiB
constexpr int kBBytes = kBN * kBK * 2;   // 32 KiB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kBoxBytes = 64 * kBK * 2;  // one 64-column x 64-token box, 8 KiB
constexpr int kStgPitch = 33;
constexpr int kStgBytes = kEpiWarps * 32 * kStgPitch * 4;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s per wait

// MB = 128-row A slabs per tile. MB = 1: 128 x 256 tiles, four stages of
// 48 KiB and two accumulator sets in TMEM (a segment drains while the next
// one accumulates). MB = 2: 256 x 256 tiles whose two halves share the B
// slab (64 KiB per stage for twice the MMAs: a third less L2 traffic per
// flop), three stages, one accumulator set (the MMAs wait for each drain).
template <int MB>
struct HGeo {
  static constexpr int kStagesM = MB == 1 ? 4 : 3;
  static constexpr int kABytesM = MB * kABytes;
  static constexpr int kStageBytesM = kABytesM + kBBytes;
  static constexpr int kNBuf = MB == 1 ? 2 : 1;
  static constexpr size_t kSmem = 1024 + (size_t)kStagesM * kStageBytesM + kStgBytes + 12 * 8 + 16;
  static_assert(kStagesM <= kStages, "barrier slots");
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// MN-major, 128-byte swizzle: 64-element MN blocks LBO apart, 8-row K groups
// SBO apart (canonical Swizzle<3,4,3> o ((8,8,m),(8,k)):((1,8,LBO),(64,SBO))
// in elements).
constexpr uint32_t kLBO = kBoxBytes;  // next 64 columns = next TMA box
constexpr uint32_t kSBO = 1024;       // 8 tokens x 128 B

__device__ __forceinline__ uint64_t make_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((kLBO >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((kSBO >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;  // layout SWIZZLE_128B
  return d;
}

// kind::f16: D f32, A/B f16 or bf16, both MN-major, M = 128, N = 256
__host__ __device__ constexpr uint32_t make_idesc(int ab_bf16) {
  return (1u << 4) | ((uint32_t)ab_bf16 << 7) | ((uint32_t)ab_bf16 << 10) | (1u << 15) |
         (1u << 16) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// true when the phase completed; false on timeout (which raises the abort
// flag) or when another role has aborted
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          bool sleep) {
  const uint64_t t0 = gtimer();
  for (uint32_t it = 0;; ++it) {
    if (mbar_test(bar, parity)) return true;
    if ((it & 63u) == 63u) {
      if (*abort_flag) return false;
      if (gtimer() - t0 > kWaitNs) {
        *abort_flag = 1;
        return false;
      }
    }
    if (sleep) __nanosleep(64);
  }
}

// the same wait for the shutdown path: ignores the abort flag
__device__ __forceinline__ bool mbar_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = gtimer();
  while (!mbar_test(bar, parity)) {
    if (gtimer() - t0 > kWaitNs) return false;
    __nanosleep(64);
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// L2 policy for H: its lines stay in L2 ahead of the streamed X slabs, so the
// tile's next segment adds into cached lines instead of re-reading HBM
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void red_add4(float* p, float a, float b, float c, float e,
                                         uint64_t pol) {
  asm volatile("red.global.add.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p),
               "f"(a), "f"(b), "f"(c), "f"(e), "l"(pol)
               : "memory");
}

// MB = 1: i-block bi (128 rows) pairs with the j-blocks bj >= bi/2 (256
// columns): the ones that reach column >= row somewhere. MB = 2 (SQ): 256 x
// 256 blocks with bj >= bi. Launch order walks groups of 8 consecutive
// i-blocks column by column (bi fastest), so the CTAs resident at one time
// share few A and B slabs of X in L2.
#ifndef EXL3_HESS_RASTER
#define EXL3_HESS_RASTER 8
#endif
constexpr int kRasterGroup = EXL3_HESS_RASTER;
// Tile shape by waves (one CTA per SM either way): a 256 x 256 tile costs
// about 1.8 times a 128 x 256 one (twice the MMAs, a third less L2 traffic
// per MMA; measured 1.75-1.83 on B200 with 262,144 tokens), so the shape
// with fewer waves x cost wins: 256 x 256 at d = 4096, 12288, 14336 and
// 128 x 256 at d = 2048 and 5120.
constexpr double kSquareTileCost = 1.8;

template <bool SQ>
int64_t tile_count(int64_t d) {
  const int64_t nbi = (d + kBM * (SQ ? 2 : 1) - 1) / (kBM * (SQ ? 2 : 1));
  const int64_t nbj = (d + kBN - 1) / kBN;
  int64_t n = 0;
  for (int64_t bi = 0; bi < nbi; ++bi) n += nbj - (SQ ? bi : (bi >> 1));
  return n;
}

int choose_mb(int64_t d, int sms) {
  const int64_t w1 = (tile_count<false>(d) + sms - 1) / sms;
  const int64_t w2 = (tile_count<true>(d) + sms - 1) / sms;
  return (double)w2 * kSquareTileCost < (double)w1 ? 2 : 1;
}

template <bool SQ>
__device__ __forceinline__ void tile_of(int idx, int nbi, int nbj, int& bi, int& bj) {
  int g0 = 0;
  for (;;) {
    const int g1 = min(g0 + kRasterGroup, nbi);
    int cnt = 0;
    for (int b = g0; b < g1; ++b) cnt += nbj - (SQ ? b : (b >> 1));
    if (idx < cnt) break;
    idx -= cnt;
    g0 = g1;
  }
  const int glast = min(g0 + kRasterGroup, nbi) - 1;
  for (int j = SQ ? g0 : (g0 >> 1);; ++j) {
    // SQ: bj >= bi; else bj >= bi/2  <=>  bi <= 2*bj + 1
    const int hi = min(glast, SQ ? j : 2 * j + 1);
    const int cnt = hi - g0 + 1;
    if (idx < cnt) {
      bi = g0 + idx;
      bj = j;
      return;
    }
    idx -= cnt;
  }
}

template <int BF16, int MB>
__global__ void __launch_bounds__(kThreads, 1)
hessian_tma_kernel(const __grid_constant__ CUtensorMap xmap, int64_t t_base, int64_t T_tokens,
                   int64_t d,
                   float* __restrict__ H, int nbi, int nbj, int* __restrict__ err_flag) {
  using G = HGeo<MB>;
  extern __shared__ uint8_t dsm_raw[];
  // 1024-byte alignment for the swizzled operand tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* stage_base = smem;
  float* stg = reinterpret_cast<float*>(smem + G::kStagesM * G::kStageBytesM);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::kStagesM * G::kStageBytesM + kStgBytes);
  // bars: full[4], empty[4], accf[2], acce[2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int bi, bj;
  tile_of<MB == 2>(blockIdx.x, nbi, nbj, bi, bj);
  const int i0 = bi * kBM * MB, j0 = bj * kBN;
  const int nchunks = (int)((T_tokens + kBK - 1) / kBK);
  const int nseg = (nchunks + kSegChunks - 1) / kSegChunks;

  auto full = [&](int s) { return smem_u32(&bars[s]); };
  auto empty = [&](int s) { return smem_u32(&bars[kStages + s]); };
  auto accf = [&](int b) { return smem_u32(&bars[2 * kStages + b]); };
  auto acce = [&](int b) { return smem_u32(&bars[2 * kStages + 2 + b]); };

  if (tid == 0) {
    for (int s = 0; s < G::kStagesM; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf(b), 1);
      mbar_init(acce(b), kEpiWarps);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(2 * kBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
      int issued = 0;
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % G::kStagesM, r = c / G::kStagesM;
        if (r > 0 && !mbar_wait(empty(s), (r - 1) & 1, abort_flag, false)) break;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(full(s)),
                     "r"(G::kStageBytesM)
                     : "memory");
        const uint32_t a = smem_u32(stage_base + s * G::kStageBytesM);
        const uint32_t b = a + G::kABytesM;
        const int t0 = (int)(t_base + (int64_t)c * kBK);
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          tma_load_2d(a + m * kABytes, &xmap, i0 + 128 * m, t0, full(s));
          tma_load_2d(a + m * kABytes + kBoxBytes, &xmap, i0 + 128 * m + 64, t0, full(s));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) tma_load_2d(b + q * kBoxBytes, &xmap, j0 + 64 * q, t0, full(s));
        issued = c + 1;
      }
      // stopped early: every copy in flight must land before the CTA exits
      if (issued < nchunks) {
        const int first = issued > G::kStagesM ? issued - G::kStagesM : 0;
        for (int c = first; c < issued; ++c)
          mbar_drain(full(c % G::kStagesM), (c / G::kStagesM) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = make_idesc(BF16);
      int last_commit = -1;
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % G::kStagesM, r = c / G::kStagesM;
        const int seg = c / kSegChunks, buf = seg % G::kNBuf;
        const bool seg_first = (c % kSegChunks) == 0;
        const bool seg_last = (c % kSegChunks) == kSegChunks - 1 || c == nchunks - 1;
        if (seg_first && seg >= G::kNBuf) {
          if (!mbar_wait(acce(buf), ((seg / G::kNBuf) - 1) & 1, abort_flag, false)) break;
        }
        if (!mbar_wait(full(s), r & 1, abort_flag, false)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a0 = smem_u32(stage_base + s * G::kStageBytesM);
        const uint32_t b0 = a0 + G::kABytesM;
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ++ks) {
          const uint64_t db = make_desc_sw128(b0 + ks * 2 * kSBO);
          const uint32_t accum = (seg_first && ks == 0) ? 0u : 1u;
#pragma unroll
          for (int m = 0; m < MB; ++m) {
            const uint64_t da = make_desc_sw128(a0 + m * kABytes + ks * 2 * kSBO);
            const uint32_t dacc = tmem + (uint32_t)((buf * MB + m) * kBN);
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "setp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                ::"r"(dacc), "l"(da), "l"(db), "r"(idesc), "r"(accum));
          }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(empty(s)) : "memory");
        if (seg_last)
          asm volatile(
              "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
              ::"r"(accf(buf)) : "memory");
        last_commit = c;
      }
      // stopped early: the MMAs in flight must finish before TMEM is freed
      if (last_commit >= 0 && last_commit < nchunks - 1)
        mbar_drain(empty(last_commit % G::kStagesM), (last_commit / G::kStagesM) & 1);
    }
  } else {
    // ---------------- epilogue: warps 2..9 ----------------
    const int quarter = warp & 3;  // this warp may read TMEM lanes 32*quarter .. +31
    const int half = (warp - 2) >> 2;  // and drains this half of the accumulator columns
    const uint64_t hpol = l2_evict_last_policy();
    float* my_stg = stg + (warp - 2) * 32 * kStgPitch;
    for (int seg = 0; seg < nseg; ++seg) {
      const int buf = seg % G::kNBuf;
      const bool ok = mbar_wait(accf(buf), (seg / G::kNBuf) & 1, abort_flag, true);
      if (!__all_sync(0xFFFFFFFFu, ok)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll 1
      for (int mc = half * (MB * kBN / 2); mc < (half + 1) * (MB * kBN / 2); mc += 32) {
        const int m = mc / kBN, cb = mc % kBN;
        const int row_base = i0 + 128 * m + 32 * quarter;
        uint32_t v[32];
        const uint32_t taddr = tmem + ((uint32_t)(32 * quarter) << 16) +
                               (uint32_t)((buf * MB + m) * kBN + cb);
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
#pragma unroll
        for (int q = 0; q < 32; ++q) my_stg[lane * kStgPitch + q] = __uint_as_float(v[q]);
        __syncwarp();
        const int col0 = j0 + cb;
        const int sub = lane >> 3, quad = (lane & 7) * 4;
        // (r, c), c >= r: 8 lanes per row, 4 columns per lane (the lower
        // triangle is written once per call by hessian_mirror_kernel)
#pragma unroll 2
        for (int it = 0; it < 8; ++it) {
          const int rr = it * 4 + sub;
          const int r = row_base + rr, c = col0 + quad;
          if (r < d && c < d && c + 3 >= r) {
            const float* s = my_stg + rr * kStgPitch + quad;
            red_add4(H + (int64_t)r * d + c, (c >= r) ? s[0] : 0.f, (c + 1 >= r) ? s[1] : 0.f,
                     (c + 2 >= r) ? s[2] : 0.f, s[3], hpol);
          }
        }
        __syncwarp();
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0)
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(acce(buf)) : "memory");
    }
  }

  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (tid == 0 && *abort_flag) atomicExch(err_flag, 1);
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kBN));
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// H[c][r] = H[r][c] for c > r: the lower triangle from the upper one, one
// CTA of 32 x 8 threads per 32 x 32 block of the upper triangle (blocks
// below the diagonal exit at once), transposed through shared memory
__global__ void __launch_bounds__(256) hessian_mirror_kernel(float* __restrict__ H, int64_t d) {
  const int64_t bi = blockIdx.y, bj = blockIdx.x;
  if (bj < bi) return;
  __shared__ float t[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t r0 = bi * 32, c0 = bj * 32;
  for (int k = ty; k < 32; k += 8) {
    const int64_t r = r0 + k, c = c0 + tx;
    if (r < d && c < d) t[k][tx] = H[r * d + c];
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int64_t r = c0 + k, c = r0 + tx;  // lower (r, c) takes upper (c, r)
    if (r < d && c < d && r > c) H[r * d + c] = t[tx][k];
  }
}

// Tile shape: 0 = by waves (choose_mb), 1 = 128 x 256,
// 2 = 256 x 256. Set only by exl3_hessian_set_tile (tests and probes).
std::atomic<int> g_tile_mode{0};

// Tokens per launch: a wave of CTAs shares each X slab in L2 only while its
// CTAs stay near the same token chunk, and over a long call they drift apart
// (d = 12288: 262,144 tokens in one launch ran at 1,140 TFLOP/s, 65,536 at
// 1,430). A multiple of the 8192-token segment, so the segments, and with
// them the sums, are those of one launch.
#ifndef EXL3_HESS_SLAB
#define EXL3_HESS_SLAB 65536
#endif
constexpr int64_t kSlabTokens = EXL3_HESS_SLAB;
static_assert(kSlabTokens % (kSegChunks * kBK) == 0, "slabs hold whole segments");

template <int BF16, int MB>
int launch_hessian(const CUtensorMap& map, int64_t T, int64_t d, float* H, int nbi, int nbj,
                   int64_t ntiles, int* err_flag, int dev, exl3_stream_t stream) {
  static DeviceBits attr_done;
  constexpr size_t smem = HGeo<MB>::kSmem;
  if (!attr_done.has(dev)) {
    EXL3_CUDA(cudaFuncSetAttribute(hessian_tma_kernel<BF16, MB>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_done.set(dev);
  }
  for (int64_t tb = 0; tb < T; tb += kSlabTokens) {
    const int64_t len = T - tb < kSlabTokens ? T - tb : kSlabTokens;
    hessian_tma_kernel<BF16, MB><<<(unsigned)ntiles, kThreads, smem, (cudaStream_t)stream>>>(
        map, tb, len, d, H, nbi, nbj, err_flag);
    EXL3_LAUNCHED();
  }
  return EXL3_OK;
}

}  // namespace
}  // namespace exl3

using namespace exl3;

extern "C" int exl3_hessian_set_tile(int mode) {
  EXL3_REQUIRE(mode >= 0 && mode <= 2, "tile mode must be 0 (by d), 1 (128x256) or 2 (256x256)");
  g_tile_mode.store(mode);
  return EXL3_OK;
}

extern "C" int exl3_hessian_accumulate(float* H, const void* X, int dtype, int64_t T, int64_t d,
                                       int* err_flag, exl3_stream_t stream) {
  EXL3_REQUIRE(H && X && err_flag, "NULL pointer argument");
  EXL3_REQUIRE(dtype == 0 || dtype == 1, "dtype must be 0 (fp16) or 1 (bf16), got %d", dtype);
  EXL3_REQUIRE(d > 0 && d % 8 == 0, "d (%lld) must be a positive multiple of 8", (long long)d);
  EXL3_REQUIRE(d < (1ll << 20), "d too large");
  EXL3_REQUIRE(T >= 0 && T < (1ll << 31) - 64, "token count must be in [0, 2^31 - 64)");
  EXL3_REQUIRE(reinterpret_cast<uintptr_t>(X) % 16 == 0, "X must be 16-byte aligned");
  EXL3_REQUIRE(reinterpret_cast<uintptr_t>(H) % 16 == 0, "H must be 16-byte aligned");
  if (T == 0) return EXL3_OK;
  const int mode = g_tile_mode.load();
  const int mb = mode == 1 ? 1 : mode == 2 ? 2 : choose_mb(d, sm_count());
  const int nbi = (int)((d + kBM * mb - 1) / (kBM * mb));
  const int nbj = (int)((d + kBN - 1) / kBN);
  const int64_t ntiles = mb == 2 ? tile_count<true>(d) : tile_count<false>(d);

  auto enc = encode_fn();
  EXL3_REQUIRE(enc != nullptr, "cuTensorMapEncodeTiled is unavailable from the driver");
  alignas(64) CUtensorMap map;
  const cuuint64_t gdim[2] = {(cuuint64_t)d, (cuuint64_t)T};
  const cuuint64_t gstride[1] = {(cuuint64_t)d * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kBK};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult cr =
      enc(&map, dtype ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
          const_cast<void*>(X), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  EXL3_REQUIRE(cr == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)cr);

  int dev = 0;
  EXL3_CUDA(cudaGetDevice(&dev));
  const int variant = 2 * dtype + (mb - 1);
  int rc = EXL3_OK;
  switch (variant) {
    case 0: rc = launch_hessian<0, 1>(map, T, d, H, nbi, nbj, ntiles, err_flag, dev, stream); break;
    case 1: rc = launch_hessian<0, 2>(map, T, d, H, nbi, nbj, ntiles, err_flag, dev, stream); break;
    case 2: rc = launch_hessian<1, 1>(map, T, d, H, nbi, nbj, ntiles, err_flag, dev, stream); break;
    default: rc = launch_hessian<1, 2>(map, T, d, H, nbi, nbj, ntiles, err_flag, dev, stream); break;
  }
  if (rc != EXL3_OK) return rc;
  EXL3_LAUNCHED();
  const unsigned nb32 = (unsigned)((d + 31) / 32);
  hessian_mirror_kernel<<<dim3(nb32, nb32), 256, 0, (cudaStream_t)stream>>>(H, d);
  EXL3_LAUNCHED();
  return EXL3_OK;
}
