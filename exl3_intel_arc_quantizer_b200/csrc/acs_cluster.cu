// Cluster-split ACS passes for calls with few tile pairs (K = 2..6).
//
// An LDLQ step of a column-sharded module hands the encoder a few dozen
// tiles: with one tile pair per CTA most SMs idle and the call takes the
// latency of one pair's 2 x 256 dependent steps. Here the cost vector of a
// pair is split over a thread-block cluster of C CTAs (C = 2, 4, 8), each
// owning S/C consecutive edges, so C SMs share every step.
//
// Exchange. Edge x's cost feeds the Q edges whose predecessor group
// (e >> K) equals x mod 2^GB; with consecutive edge ranges per CTA, that
// consumer is CTA (x >> log2(GL)) & (C-1), GL = 2^GB / C. Every CTA keeps an
// input buffer of the Q x GL predecessor words it reads (k-major: word
// (k << GB) | g at k*GL + g - r*GL). After computing a chunk of edges a
// thread writes it straight into the consumer's buffer with st.async, whose
// byte count completes the consumer's mbarrier (own-CTA words go through
// plain shared stores and are left out of the expected byte count; the CTA
// barrier of every step orders them). Four buffers rotate: a producer writing
// message m into a consumer's buffer m % 4 has already received message m-1
// from every CTA that feeds it, and those producers received message m-2
// from theirs; because any CTA reaches every other in two hops of this graph
// (C <= Q^2), all CTAs have passed the step barrier after reading message m-4,
// so the buffer is free without any backwards signal.
//
// Arithmetic, checkpoint steps and checkpoint layout are the tile-pair
// kernel's (acs_pair.cu): each CTA copies its slice of a checkpointed cost
// vector into the same HBM slot at offset r * S/C words, so the traceback
// kernels are shared. Tie-breaking and NaN rules are unchanged (min over
// ascending k in registers; compare-and-select for pairs with NaN inputs).
//
// Every mbarrier wait is bounded (2 s by default, globaltimer); a CTA that
// times out raises a CTA-wide abort flag, stops waiting and sending, runs to
// the end and counts the fault in a device counter (exl3_encoder_fault_count),
// which the layer drivers compare before and after a call. A test hook
// (exl3_encoder_test_cluster_wait) shortens the limit and makes every CTA
// stop sending from one step on, so the waits after it run out while no
// message is in flight.
#include "common.cuh"
#include "encoder_shared.cuh"

namespace exl3 {

__device__ unsigned int g_encoder_faults = 0;

namespace {

constexpr uint64_t kClusterWaitNs = 2000000000ull;

template <int K, int C>
struct CGeo {
  static constexpr int S = 1 << (16 - K);
  static constexpr int Kr = 16 - K;
  static constexpr int GB = 16 - 2 * K;
  static constexpr int Q = 1 << K;
  static constexpr int LOGC = C == 2 ? 1 : (C == 4 ? 2 : 3);
  static constexpr int SL = S / C;                   // edges per CTA
  static constexpr int GL = (1 << GB) / C;           // predecessor groups per CTA
  static constexpr int LOGGL = GB - LOGC;
  static constexpr int NT = SL < 512 ? SL : 512;     // threads per CTA
  static constexpr int E = SL / NT;                  // edges per thread
  static constexpr int CE = E < 8 ? E : 8;           // edges per chunk
  static constexpr int NCH = E / CE;                 // chunks per thread
  static constexpr int NGC = ((CE >> K) > 0) ? (CE >> K) : 1;
  static constexpr int KB = Q < 8 ? Q : 8;
  static constexpr int R = ck_stride(K);              // checkpoint stride (as acs_pair.cu)
  static constexpr int CKB = S * 4;
  static constexpr int NCB = E * Q / 2;              // codebook registers
  static_assert(C == 2 || C == 4 || C == 8, "cluster of 2, 4 or 8 CTAs");
  static_assert(K >= 2 && K <= 6, "cluster split needs 2^GB >= C");
  static_assert(GL >= CE && GL >= 1, "a chunk must land in one consumer");
  static_assert(NCB >= 1 && NCB <= 64, "codebook register budget");
  static_assert(C <= Q * Q, "two-hop reachability of the exchange graph");
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t gclock() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_init1(uint32_t bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for a message; false on timeout (raises *abort) or abort.
__device__ __forceinline__ bool msg_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                         uint64_t wait_ns) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = gclock();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try(bar, parity)) return true;
    if ((it & 15u) == 0u) {
      if (*abort) return false;
      if (gclock() - t0 > wait_ns) {
        *abort = 1;
        return false;
      }
    }
  }
}

// remote stores of CE words that complete the consumer's mbarrier
template <int CE>
__device__ __forceinline__ void st_remote(uint32_t raddr, uint32_t rbar, const uint32_t* v) {
  if constexpr (CE == 1) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];"
                 ::"r"(raddr), "r"(v[0]), "r"(rbar) : "memory");
  } else if constexpr (CE == 2) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b32 [%0], {%1, %2}, [%3];"
        ::"r"(raddr), "r"(v[0]), "r"(v[1]), "r"(rbar) : "memory");
  } else {
#pragma unroll
    for (int q = 0; q < CE / 4; ++q)
      asm volatile(
          "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], "
          "{%1, %2, %3, %4}, [%5];"
          ::"r"(raddr + 16 * q), "r"(v[4 * q]), "r"(v[4 * q + 1]), "r"(v[4 * q + 2]),
          "r"(v[4 * q + 3]), "r"(rbar) : "memory");
  }
}

template <int CE>
__device__ __forceinline__ void st_words(uint32_t* dst, const uint32_t* v) {
  if constexpr (CE % 4 == 0) {
#pragma unroll
    for (int q = 0; q < CE / 4; ++q)
      reinterpret_cast<uint4*>(dst)[q] = make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else if constexpr (CE == 2) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(v[0], v[1]);
  } else {
    dst[0] = v[0];
  }
}

// first local edge of the thread's chunk c
template <int K, int C>
__device__ __forceinline__ int chunk_edge(int c, int t) {
  using G = CGeo<K, C>;
  return (c * G::NT + t) * G::CE;
}

// consumer CTA and its input-buffer position of global edge x
template <int K, int C>
__device__ __forceinline__ int consumer_of(int x) {
  using G = CGeo<K, C>;
  return (x >> G::LOGGL) & (C - 1);
}
template <int K, int C>
__device__ __forceinline__ int consumer_pos(int x) {
  using G = CGeo<K, C>;
  return (x >> G::GB) * G::GL + (x & (G::GL - 1));
}

template <int K, int C>
__device__ __forceinline__ void cl_init_codebook(uint32_t (&cbv)[CGeo<K, C>::NCB], int cb, int t,
                                                 int r) {
  using G = CGeo<K, C>;
#pragma unroll
  for (int c = 0; c < G::NCH; ++c) {
#pragma unroll
    for (int j = 0; j < G::CE; ++j) {
      const uint32_t e = (uint32_t)(r * G::SL + chunk_edge<K, C>(c, t) + j);
#pragma unroll
      for (int k = 0; k < G::Q; k += 2) {
        const uint32_t s0 = ((uint32_t)k << G::Kr) | e, s1 = ((uint32_t)(k + 1) << G::Kr) | e;
        cbv[((c * G::CE + j) * G::Q + k) >> 1] =
            (uint32_t)cb_state_bits(cb, s0) | ((uint32_t)cb_state_bits(cb, s1) << 16);
      }
    }
  }
}

struct Links {
  uint32_t data[4];  // consumer buffer address of each chunk (buffer 0); 0 = own CTA
  uint32_t bar[4];   // consumer mbarrier 0 of each chunk
  int pos[4];        // own-CTA buffer position of each chunk
};

// One step over the thread's chunks: candidates, minimum, then the chunk's
// words go to its consumer (message `mb`: its mbarrier; `slot`: the buffer
// slot of this pair's words in that message) and, when `own_w`, to the
// CTA's own slice `ob` (checkpoints, final costs).
template <int K, int C, bool FIRST, bool EXACT>
__device__ __forceinline__ void cl_step(const uint32_t (&cbv)[CGeo<K, C>::NCB], uint32_t w2,
                                        const uint32_t* __restrict__ cin, uint32_t* inb,
                                        uint32_t* __restrict__ ob, const Links& lk, int mb,
                                        int slot, bool send, bool own_w, int t, int r, int preA,
                                        int preB) {
  using G = CGeo<K, C>;
#pragma unroll
  for (int c = 0; c < G::NCH; ++c) {
    const int le0 = chunk_edge<K, C>(c, t);
    const int gl0 = le0 >> K;
    const int e0 = r * G::SL + le0;
    uint32_t best[G::CE];
#pragma unroll
    for (int kb = 0; kb < G::Q; kb += G::KB) {
      uint32_t P[G::KB][G::NGC];
      if constexpr (!FIRST) {
#pragma unroll
        for (int q = 0; q < G::KB; ++q) {
          const uint32_t* src = cin + (kb + q) * G::GL + gl0;
          if constexpr (G::NGC == 2) {
            const uint2 v = *reinterpret_cast<const uint2*>(src);
            P[q][0] = v.x;
            P[q][1] = v.y;
          } else {
            P[q][0] = *src;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < G::CE; ++j) {
        const int gi = (G::NGC > 1) ? (j >> K) : 0;
#pragma unroll
        for (int q = 0; q < G::KB; ++q) {
          const int k = kb + q;
          const int m = (c * G::CE + j) * G::Q + k;
          const uint32_t d = (m & 1) ? h2_sub_bcast<true>(cbv[m >> 1], w2)
                                     : h2_sub_bcast<false>(cbv[m >> 1], w2);
          uint32_t cst = h2_fma(d, d, FIRST ? 0u : P[q][gi]);
          if constexpr (FIRST) {
            if (preA >= 0 || preB >= 0) {
              const int pred = (k << G::GB) | ((e0 + j) >> K);
              const uint32_t allow = ((pred == preA || preA < 0) ? 0x0000FFFFu : 0u) |
                                     ((pred == preB || preB < 0) ? 0xFFFF0000u : 0u);
              cst = bsel(allow, cst, kHInf2);
            }
          }
          if (k == 0) {
            best[j] = cst;
          } else if constexpr (EXACT) {
            best[j] = bsel(h2_lt_mask(cst, best[j]), cst, best[j]);
          } else {
            best[j] = h2_min(best[j], cst);
          }
        }
      }
    }
    if (send) {
      if (lk.data[c] != 0u)
        st_remote<G::CE>(lk.data[c] + (uint32_t)(slot * G::SL * 4), lk.bar[c] + 8u * mb, best);
      else
        st_words<G::CE>(inb + slot * G::SL + lk.pos[c], best);
    }
    if (own_w) st_words<G::CE>(ob + le0, best);
  }
}

__device__ __forceinline__ void ckc_fence() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void ckc_issue(uint8_t* gdst, const uint32_t* ssrc, uint32_t bytes) {
  asm volatile(
      "cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n\t"
      "cp.async.bulk.commit_group;" ::"l"(gdst), "r"(smem_addr(ssrc)), "r"(bytes)
      : "memory");
}
__device__ __forceinline__ void ckc_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void ckc_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Shared memory of a cluster CTA serving P tile pairs at once: four rotating
// input buffers and two own slices of P x S/C words each, and the P pairs'
// weights. Launched with at least 116 KiB so two CTAs never share an SM: the
// split only pays when every CTA of a cluster has an SM of its own.
template <int K, int C, int P>
struct CSmem {
  static constexpr size_t bytes = (size_t)6 * P * CGeo<K, C>::SL * 4 + (size_t)P * 256 * 4;
  static constexpr size_t launch = bytes > 118784 ? bytes : 118784;
  static_assert(bytes <= 227 * 1024, "shared memory of a cluster CTA");
};

// One pass over P tile pairs at once: L steps, messages msg .. msg+L-2, each
// message carrying every pair's words (one mbarrier phase per step for all
// of them). Pair p's words live in slot (m * P + p) of the message buffers.
template <int K, int C, int P, int PASS, bool EXACT>
__device__ __forceinline__ void cl_pass(const uint32_t (&cbv)[CGeo<K, C>::NCB],
                                        const uint32_t* wt, uint32_t* inb, uint32_t* own,
                                        uint32_t bar0, const Links& lk, uint8_t* const (&ckp)[P],
                                        int L, int t, int r, const int (&preA)[P],
                                        const int (&preB)[P], uint32_t msg, uint32_t expect,
                                        volatile int* abort, uint64_t wait_ns, int stop_at) {
  using G = CGeo<K, C>;
  const int half = L / 2;
  for (int i = 0; i < L; ++i) {
    const bool aborted = *abort != 0;
    if (i > 0 && !aborted) {
      const uint32_t m = msg + (uint32_t)(i - 1);
      const uint32_t bar = bar0 + 8u * (m & 3u);
      if (msg_wait(bar, (m >> 2) & 1u, abort, wait_ns) && t == 0)
        mbar_expect(bar, expect);  // message m+4
    }
    // stop_at >= 0 (test hook only): every CTA stops sending at that step,
    // so all earlier messages were consumed and none is in flight
    const bool send = i < L - 1 && *abort == 0 && (stop_at < 0 || i < stop_at);
    int slot = -1;
    if (PASS == 1) {
      const int rel = i - (half - 1);
      if (rel >= 0 && rel % G::R == 0 && i <= L - 2) slot = rel / G::R;
    } else {
      if ((i + 1) % G::R == 0 && i <= L - 2) slot = (i + 1) / G::R - 1;
    }
    const bool own_w = slot >= 0 || i == L - 1;
    const int mb = (int)((msg + (uint32_t)i) & 3u);
    const int wi = PASS == 1 ? (i < half ? i + half : i - half) : i;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const uint32_t w2 = wt[p * 256 + wi];
      uint32_t* ob = own + ((i & 1) * P + p) * G::SL;
      if (i == 0) {
        cl_step<K, C, true, EXACT>(cbv, w2, nullptr, inb, ob, lk, mb, mb * P + p, send, own_w, t,
                                   r, PASS == 2 ? preA[p] : -1, PASS == 2 ? preB[p] : -1);
      } else {
        const uint32_t* cin = inb + (((msg + (uint32_t)(i - 1)) & 3u) * P + p) * G::SL;
        cl_step<K, C, false, EXACT>(cbv, w2, cin, inb, ob, lk, mb, mb * P + p, send, own_w, t,
                                    r, -1, -1);
      }
    }
    if (slot >= 0) ckc_fence();
    if (t == 0) ckc_wait_read();  // the copy of step i-1 read the slice step i+1 rewrites
    __syncthreads();
    if (slot >= 0 && t == 0) {
#pragma unroll
      for (int p = 0; p < P; ++p)
        if (ckp[p])
          ckc_issue(ckp[p] + (size_t)slot * G::CKB + (size_t)r * G::SL * 4,
                    own + ((i & 1) * P + p) * G::SL, G::SL * 4);
    }
  }
  if (t == 0) ckc_wait_read();
}

template <int K, int C, int P, int PASS>
__global__ void __launch_bounds__(CGeo<K, C>::NT, 1)
acs_cluster_kernel(const float* __restrict__ in, int n, int L, int cb, uint8_t* __restrict__ ck,
                   size_t ck_pair_bytes, int32_t* __restrict__ best_edge,
                   const int32_t* __restrict__ end_state, float* __restrict__ path_cost,
                   uint64_t wait_ns, int stop_at) {
  using G = CGeo<K, C>;
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* inb = reinterpret_cast<uint32_t*>(smem);  // 4 x P message slots of S/C words
  uint32_t* own = inb + 4 * P * G::SL;                 // 2 x P slices of own results
  uint32_t* wt = own + 2 * P * G::SL;                  // {w_A, w_B} per step, per pair
  __shared__ __align__(8) uint64_t bars[4];
  __shared__ uint32_t red[P][64];
  __shared__ uint32_t ckeys[P][2 * C];  // rank 0: per-CTA argmin keys
  __shared__ int abort_s;
  __shared__ int self_words;
  const int t = threadIdx.x;
  const int r = (int)cluster_rank();
  const uint32_t bar0 = smem_addr(&bars[0]);

  // where each chunk's words go (the same for every pair: pair p adds p * S/C)
  Links lk;
  int mine = 0;
#pragma unroll
  for (int c = 0; c < G::NCH; ++c) {
    const int x = r * G::SL + chunk_edge<K, C>(c, t);
    const int rc = consumer_of<K, C>(x);
    lk.pos[c] = consumer_pos<K, C>(x);
    if (rc == r) {
      lk.data[c] = 0u;
      lk.bar[c] = 0u;
      mine += G::CE;
    } else {
      lk.data[c] = map_rank(smem_addr(inb + lk.pos[c]), (uint32_t)rc);
      lk.bar[c] = map_rank(bar0, (uint32_t)rc);
    }
  }
  if (t == 0) {
    abort_s = 0;
    self_words = 0;
  }
  __syncthreads();
  if (mine) atomicAdd(&self_words, mine);
  __syncthreads();
  const uint32_t expect = (uint32_t)(G::SL - self_words) * 4u * (uint32_t)P;
  if (t == 0) {
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      mbar_init1(bar0 + 8u * b);
      mbar_expect(bar0 + 8u * b, expect);  // messages 0..3
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  cluster_sync_all();  // every CTA's barriers exist before the first remote store

  uint32_t cbv[G::NCB];
  cl_init_codebook<K, C>(cbv, cb, t, r);
  const int npairs = (n + 1) / 2;
  const int ngroups = (npairs + P - 1) / P;
  uint32_t msg = 0;
  for (int tg = (int)cluster_id(); tg < ngroups; tg += (int)cluster_count()) {
    // pairs of the group; a missing last one repeats the group's first pair
    // (its words travel like the others', its outputs are not written)
    int ta[P], tb[P];
    bool valid[P], has_b[P];
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int tp = tg * P + p;
      valid[p] = tp < npairs;
      const int tq = valid[p] ? tp : tg * P;
      ta[p] = 2 * tq;
      tb[p] = (2 * tq + 1 < n) ? 2 * tq + 1 : 2 * tq;
      has_b[p] = valid[p] && 2 * tq + 1 < n;
    }
    int nan = 0;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      for (int i = t; i < L; i += G::NT) {
        const __half a = __float2half_rn(in[(size_t)ta[p] * L + i]);
        const __half b = __float2half_rn(in[(size_t)tb[p] * L + i]);
        nan |= (__hisnan(a) || __hisnan(b)) ? 1 : 0;
        wt[p * 256 + i] = (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
      }
    }
    nan = __syncthreads_or(nan);
    uint8_t* pck[P];
#pragma unroll
    for (int p = 0; p < P; ++p)
      pck[p] = valid[p] ? ck + (size_t)(tg * P + p) * ck_pair_bytes : nullptr;
    const uint32_t* fin = own + ((L - 1) & 1) * P * G::SL;
    if constexpr (PASS == 1) {
      int neg[P];
#pragma unroll
      for (int p = 0; p < P; ++p) neg[p] = -1;
      if (nan)
        cl_pass<K, C, P, 1, true>(cbv, wt, inb, own, bar0, lk, pck, L, t, r, neg, neg, msg, expect,
                                  &abort_s, wait_ns, stop_at);
      else
        cl_pass<K, C, P, 1, false>(cbv, wt, inb, own, bar0, lk, pck, L, t, r, neg, neg, msg,
                                   expect, &abort_s, wait_ns, stop_at);
      // argmin over the cluster: lowest key = (cost bits + edge), finite only
#pragma unroll
      for (int p = 0; p < P; ++p) {
        uint32_t ka = 0xFFFFFFFFu, kb = 0xFFFFFFFFu;
        for (int le = t; le < G::SL; le += G::NT) {
          const uint32_t w = fin[p * G::SL + le];
          const uint32_t e = (uint32_t)(r * G::SL + le);
          const uint32_t a = w & 0xFFFFu, b = w >> 16;
          if ((a & 0x7C00u) != 0x7C00u) ka = min(ka, (a << 16) | e);
          if ((b & 0x7C00u) != 0x7C00u) kb = min(kb, (b << 16) | e);
        }
        ka = __reduce_min_sync(0xFFFFFFFFu, ka);
        kb = __reduce_min_sync(0xFFFFFFFFu, kb);
        if ((t & 31) == 0) {
          red[p][t >> 5] = ka;
          red[p][32 + (t >> 5)] = kb;
        }
      }
      __syncthreads();
      if (t < 32) {
#pragma unroll
        for (int p = 0; p < P; ++p) {
          uint32_t va = (t < G::NT / 32) ? red[p][t] : 0xFFFFFFFFu;
          uint32_t vb = (t < G::NT / 32) ? red[p][32 + t] : 0xFFFFFFFFu;
          va = __reduce_min_sync(0xFFFFFFFFu, va);
          vb = __reduce_min_sync(0xFFFFFFFFu, vb);
          if (t == 0) {
            const uint32_t dst = map_rank(smem_addr(&ckeys[p][0]), 0u);
            asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(dst + 4u * r), "r"(va)
                         : "memory");
            asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(dst + 4u * (C + r)), "r"(vb)
                         : "memory");
          }
        }
      }
      cluster_sync_all();
      if (r == 0 && t == 0) {
#pragma unroll
        for (int p = 0; p < P; ++p) {
          if (!valid[p]) continue;
          uint32_t va = 0xFFFFFFFFu, vb = 0xFFFFFFFFu;
#pragma unroll
          for (int q = 0; q < C; ++q) {
            va = min(va, ckeys[p][q]);
            vb = min(vb, ckeys[p][C + q]);
          }
          best_edge[ta[p]] = va == 0xFFFFFFFFu ? 0 : (int)(va & 0xFFFFu);
          if (has_b[p]) best_edge[tb[p]] = vb == 0xFFFFFFFFu ? 0 : (int)(vb & 0xFFFFu);
        }
      }
    } else {
      int preA[P], preB[P];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        preA[p] = end_state[ta[p]];
        preB[p] = (2 * (ta[p] >> 1) + 1 < n) ? end_state[tb[p]] : preA[p];
      }
      if (nan)
        cl_pass<K, C, P, 2, true>(cbv, wt, inb, own, bar0, lk, pck, L, t, r, preA, preB, msg,
                                  expect, &abort_s, wait_ns, stop_at);
      else
        cl_pass<K, C, P, 2, false>(cbv, wt, inb, own, bar0, lk, pck, L, t, r, preA, preB, msg,
                                   expect, &abort_s, wait_ns, stop_at);
      if (t == 0 && path_cost) {
#pragma unroll
        for (int p = 0; p < P; ++p) {
          if (!valid[p]) continue;
          const uint32_t* f = fin + p * G::SL;
          if (preA[p] / G::SL == r)
            path_cost[ta[p]] = half_bits_to_float((uint16_t)(f[preA[p] - r * G::SL] & 0xFFFFu));
          if (has_b[p] && preB[p] / G::SL == r)
            path_cost[tb[p]] = half_bits_to_float((uint16_t)(f[preB[p] - r * G::SL] >> 16));
        }
      }
    }
    msg += (uint32_t)(L - 1);
    __syncthreads();
  }
  if (t == 0) {
    ckc_wait_all();
    if (abort_s) atomicAdd(&g_encoder_faults, 1u);
  }
  cluster_sync_all();  // no CTA leaves while a peer may still address its shared memory
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
int g_cluster_policy = 0;  // 0 automatic, 1 never, 2/4/8 forced
std::atomic<unsigned long long> g_cluster_wait_ns{kClusterWaitNs};
std::atomic<int> g_cluster_stop_at{-1};  // test hook: step at which sends stop

std::atomic<int> g_cluster_pairs{0};  // 0 automatic, 1 / 2 forced

template <int K, int C, int P>
struct ClusterKernels {
  using Sm = CSmem<K, C, P>;
  static int setup(int dev) {
    static DeviceBits done;
    if (done.has(dev)) return EXL3_OK;
    EXL3_CUDA(cudaFuncSetAttribute(acs_cluster_kernel<K, C, P, 1>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Sm::launch));
    EXL3_CUDA(cudaFuncSetAttribute(acs_cluster_kernel<K, C, P, 2>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Sm::launch));
    done.set(dev);
    return EXL3_OK;
  }
  // clusters of this kernel that fit on the device at once (cached per device)
  static int max_active(int dev) {
    static std::atomic<int> cache[64];  // 0 unknown, -1 none fit, else the count
    if (dev >= 0 && dev < 64) {
      const int c = cache[dev].load(std::memory_order_relaxed);
      if (c != 0) return c > 0 ? c : 0;
    }
    if (setup(dev) != EXL3_OK) return 0;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(C * 16, 1, 1);
    cfg.blockDim = dim3(CGeo<K, C>::NT, 1, 1);
    cfg.dynamicSmemBytes = Sm::launch;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (void*)acs_cluster_kernel<K, C, P, 1>, &cfg) !=
        cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    if (dev >= 0 && dev < 64) cache[dev].store(n > 0 ? n : -1, std::memory_order_relaxed);
    return n;
  }
  static int launch(int pass, int clusters, cudaStream_t stream, const float* in, int n, int L,
                    int cb, uint8_t* ck, size_t ck_pair, int32_t* best_edge,
                    const int32_t* end_state, float* path_cost) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(clusters * C), 1, 1);
    cfg.blockDim = dim3(CGeo<K, C>::NT, 1, 1);
    cfg.dynamicSmemBytes = Sm::launch;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const uint64_t wait_ns = (uint64_t)g_cluster_wait_ns.load();
    const int stop_at = g_cluster_stop_at.load();
    if (pass == 1)
      EXL3_CUDA(cudaLaunchKernelEx(&cfg, acs_cluster_kernel<K, C, P, 1>, in, n, L, cb, ck,
                                   ck_pair, best_edge, end_state, path_cost, wait_ns, stop_at));
    else
      EXL3_CUDA(cudaLaunchKernelEx(&cfg, acs_cluster_kernel<K, C, P, 2>, in, n, L, cb, ck,
                                   ck_pair, best_edge, end_state, path_cost, wait_ns, stop_at));
    return EXL3_OK;
  }
};

// The (C, P) combinations built: one pair per cluster of 2, 4 or 8 CTAs, and
// 2 pairs per cluster of 8 CTAs (one exchange round per step for both).
template <int K, class F>
int with_kernels(int C, int P, F&& f) {
  if constexpr (K >= 2 && K <= 6) {
    if (C == 2 && P == 1) return f(ClusterKernels<K, 2, 1>{});
    if (C == 4 && P == 1) return f(ClusterKernels<K, 4, 1>{});
    if (C == 8 && P == 1) return f(ClusterKernels<K, 8, 1>{});
    if (C == 8 && P == 2) return f(ClusterKernels<K, 8, 2>{});
  }
  return -1;
}

template <int K>
int max_active_for(int C, int P, int dev) {
  const int v = with_kernels<K>(C, P, [&](auto tag) { return decltype(tag)::max_active(dev); });
  return v > 0 ? v : 0;
}

// Automatic choice for a call of `pairs` tile pairs (C = 1: no split): every
// group of P pairs must fit on the device at once, and C * groups SMs must
// not exceed the device's. Preference, measured per call (ms, 16 / 32 / 48 /
// 64 / 96 tiles): one pair per cluster of 8 (K=2: 0.42 / - / - ; K=4: 0.51)
// first. K = 2 then takes 2 pairs per cluster of 8 (0.58 / 0.64 at 32 / 48
// tiles, against 0.73 / 0.79 at 4 CTAs per pair, whose CTAs exchange 16 KiB
// each per step), then 4 CTAs per pair (0.84 at 64); a cluster of 2 at K = 2
// exchanges 32 KiB per CTA and step and is not used. K >= 3 takes 4 CTAs per
// pair (K=4: 0.56 / 0.57 / 0.60 at 32 / 48 / 64, against 0.62 / 0.63 for 2
// pairs per cluster of 8), then 2 (0.78 / 0.80 at 96 / 128). Beyond those the
// pair kernel (one pair per CTA) wins (K=2: 0.87 at 96 and 128).
template <int K>
void choose(int pairs, int sms, int dev, int* C_out, int* P_out) {
  *C_out = 1;
  *P_out = 1;
  if (K < 2 || K > 6 || g_cluster_policy == 1) return;
  const int forced_p = g_cluster_pairs.load();
  auto fits = [&](int C, int P) {
    const int groups = (pairs + P - 1) / P;
    return (int64_t)groups * C <= sms && max_active_for<K>(C, P, dev) >= groups;
  };
  static constexpr int kOrderK2[3][2] = {{8, 1}, {8, 2}, {4, 1}};
  static constexpr int kOrderK3[4][2] = {{8, 1}, {4, 1}, {2, 1}, {8, 2}};
  const int(*order)[2] = K == 2 ? kOrderK2 : kOrderK3;
  const int norder = K == 2 ? 3 : 4;
  for (int q = 0; q < norder; ++q) {
    const int C = order[q][0], P = order[q][1];
    if (g_cluster_policy >= 2 && C != g_cluster_policy) continue;
    if (forced_p > 0 && P != forced_p) continue;
    if (K >= 3 && P == 2 && forced_p != 2) continue;   // only when forced
    if (fits(C, P)) {
      *C_out = C;
      *P_out = P;
      return;
    }
  }
  if (g_cluster_policy >= 2) {  // forced size: its smallest P that the device holds at all
    for (int P : {1, 2}) {
      if (forced_p > 0 && P != forced_p) continue;
      if (max_active_for<K>(g_cluster_policy, P, dev) > 0) {
        *C_out = g_cluster_policy;
        *P_out = P;
        return;
      }
    }
  }
}

}  // namespace

void cluster_choice(int K, int pairs, int* C, int* P) {
  *C = 1;
  *P = 1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  const int sms = sm_count();
  switch (K) {
    case 2: choose<2>(pairs, sms, dev, C, P); break;
    case 3: choose<3>(pairs, sms, dev, C, P); break;
    case 4: choose<4>(pairs, sms, dev, C, P); break;
    case 5: choose<5>(pairs, sms, dev, C, P); break;
    case 6: choose<6>(pairs, sms, dev, C, P); break;
    default: break;
  }
}

int cluster_size_for(int K, int pairs) {
  int C, P;
  cluster_choice(K, pairs, &C, &P);
  return C;
}

template <int K>
static int launch_k(int C, int P, int pass, int pairs, cudaStream_t stream, const float* in,
                    int n, int L, int cb, uint8_t* ck, size_t ck_pair, int32_t* best_edge,
                    const int32_t* end_state, float* path_cost) {
  int dev = 0;
  EXL3_CUDA(cudaGetDevice(&dev));
  const int rc = with_kernels<K>(C, P, [&](auto tag) -> int {
    using KK = decltype(tag);
    int r = KK::setup(dev);
    if (r) return r;
    const int cap = KK::max_active(dev);
    EXL3_REQUIRE(cap > 0, "no cluster of %d CTAs fits on this device", C);
    const int groups = (pairs + P - 1) / P;
    const int clusters = groups < cap ? groups : cap;
    return KK::launch(pass, clusters, stream, in, n, L, cb, ck, ck_pair, best_edge, end_state,
                      path_cost);
  });
  if (rc == -1) {
    set_error("no cluster ACS for K=%d, C=%d, %d pairs per cluster", K, C, P);
    return EXL3_EINVAL;
  }
  return rc;
}

int cluster_acs_pass(int K, int C, int P, int pass, cudaStream_t stream, const float* in, int n,
                     int L, int cb, uint8_t* ck, size_t ck_pair, int32_t* best_edge,
                     const int32_t* end_state, float* path_cost) {
  const int pairs = (n + 1) / 2;
  switch (K) {
    case 2: return launch_k<2>(C, P, pass, pairs, stream, in, n, L, cb, ck, ck_pair, best_edge, end_state, path_cost);
    case 3: return launch_k<3>(C, P, pass, pairs, stream, in, n, L, cb, ck, ck_pair, best_edge, end_state, path_cost);
    case 4: return launch_k<4>(C, P, pass, pairs, stream, in, n, L, cb, ck, ck_pair, best_edge, end_state, path_cost);
    case 5: return launch_k<5>(C, P, pass, pairs, stream, in, n, L, cb, ck, ck_pair, best_edge, end_state, path_cost);
    case 6: return launch_k<6>(C, P, pass, pairs, stream, in, n, L, cb, ck, ck_pair, best_edge, end_state, path_cost);
    default:
      set_error("no cluster ACS for K=%d", K);
      return EXL3_EINVAL;
  }
}

}  // namespace exl3

using namespace exl3;

extern "C" int exl3_encoder_set_cluster(int cluster_ctas) {
  EXL3_REQUIRE(cluster_ctas == 0 || cluster_ctas == 1 || cluster_ctas == 2 || cluster_ctas == 4 ||
                   cluster_ctas == 8,
               "cluster size must be 0 (automatic), 1 (off), 2, 4 or 8, got %d", cluster_ctas);
  g_cluster_policy = cluster_ctas;
  return EXL3_OK;
}

extern "C" int exl3_encoder_set_cluster_pairs(int pairs_per_cluster) {
  EXL3_REQUIRE(pairs_per_cluster == 0 || pairs_per_cluster == 1 || pairs_per_cluster == 2,
               "pairs per cluster must be 0 (automatic), 1 or 2, got %d", pairs_per_cluster);
  g_cluster_pairs.store(pairs_per_cluster);
  return EXL3_OK;
}

extern "C" int exl3_encoder_test_cluster_wait(long long wait_limit_ns, int stop_sends_at_step) {
  EXL3_REQUIRE(wait_limit_ns <= 0 || (wait_limit_ns >= 100000 && wait_limit_ns <= 10000000000ll),
               "wait limit must be <= 0 (default 2 s) or in [1e5, 1e10] ns, got %lld",
               wait_limit_ns);
  EXL3_REQUIRE(stop_sends_at_step == -1 || (stop_sends_at_step >= 1 && stop_sends_at_step <= 254),
               "stop step must be -1 (off) or in [1, 254], got %d", stop_sends_at_step);
  g_cluster_wait_ns.store(wait_limit_ns <= 0 ? kClusterWaitNs : (unsigned long long)wait_limit_ns);
  g_cluster_stop_at.store(stop_sends_at_step);
  return EXL3_OK;
}

extern "C" int exl3_encoder_cluster_capacity(int K, int cluster_ctas, int* clusters) {
  EXL3_REQUIRE(clusters != nullptr, "clusters is NULL");
  EXL3_REQUIRE(K >= 1 && K <= 8, "K must be in 1..8, got %d", K);
  EXL3_REQUIRE(cluster_ctas == 2 || cluster_ctas == 4 || cluster_ctas == 8,
               "cluster size must be 2, 4 or 8, got %d", cluster_ctas);
  int dev = 0;
  EXL3_CUDA(cudaGetDevice(&dev));
  int n = 0;
  switch (K) {
    case 2: n = max_active_for<2>(cluster_ctas, 1, dev); break;
    case 3: n = max_active_for<3>(cluster_ctas, 1, dev); break;
    case 4: n = max_active_for<4>(cluster_ctas, 1, dev); break;
    case 5: n = max_active_for<5>(cluster_ctas, 1, dev); break;
    case 6: n = max_active_for<6>(cluster_ctas, 1, dev); break;
    default: n = 0;
  }
  *clusters = n > 0 ? n : 0;
  return EXL3_OK;
}

extern "C" int exl3_encoder_fault_count(unsigned int* out) {
  EXL3_REQUIRE(out != nullptr, "out is NULL");
  EXL3_CUDA(cudaDeviceSynchronize());
  EXL3_CUDA(cudaMemcpyFromSymbol(out, g_encoder_faults, sizeof(unsigned int)));
  return EXL3_OK;
}
