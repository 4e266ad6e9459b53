// LDLQ block-feedback loop on the device, for one or several weight
// matrices at once.
//
// Reference: exl3_quant/ldlq.py:163-309. Per matrix W (k x n, the
// regularized weight) and its block-LDL factor L (k x k): spans of `buf`
// rows bottom-up, 16-row blocks bottom-up inside a span:
//   rows   = W[blk] + prod_cache[blk] + L[below, blk]^T (W - W_q)[below]
//   W_q[blk], encoded[blk] = encode(tiles of rows, tensor-core order)
// and after a span: prod_cache += L[span]^T (W - W_q)[span].
//
// Here every step is three launches for all matrices together:
//   ldlq_prep_kernel  one CTA per tile: the compensation sum over the rows
//                     below (<= buf-16 of them, in shared memory), the
//                     cached product and W, written straight into the
//                     encoder's tile order;
//   the encoder       (exl3_quantize_tiles) on the concatenated tiles;
//   ldlq_post_kernel  one CTA per tile: reconstruction back to row order
//                     into W_q, states into `encoded`;
// plus, when a matrix finishes a span, ldlq_span_kernel: the trailing
// update, restricted to the rows above the span (the only ones read later),
// as a shared-memory tiled fp32 product (fixed summation order, so results
// are deterministic). Matrices shorter than the longest start at the step
// schedule_jobs picks, so that a column-sharded layer's short matrices fill
// steps that would otherwise encode a few tiles at the encoder's latency
// floor instead of pushing early steps into a second wave.
#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "encoder_shared.cuh"

namespace exl3 {
namespace {

constexpr int kMaxJobs = 32;

struct StepJob {
  const float* W;      // (k, n)
  const float* L;      // (k, k)
  float* Wq;           // (k, n)
  float* prod;         // (k, n) cached products
  int16_t* enc;        // (k/16, n/16, 256)
  int64_t k, n;
  int r0;              // first row of this step's block
  int below0, below1;  // rows [below0, below1) of the span below the block
  int tile0;           // first tile of this job in the step's batch
};

struct StepTable {
  int njobs;
  int total_tiles;
  StepJob j[kMaxJobs];
};

__constant__ int16_t c_perm[256];      // encoder position -> tile position (r*16+c)
__constant__ int16_t c_perm_inv[256];  // tile position -> encoder position

__device__ __forceinline__ int job_of(const StepTable& tab, int tile) {
  int jb = 0;
  while (jb + 1 < tab.njobs && tile >= tab.j[jb + 1].tile0) ++jb;
  return jb;
}

// one CTA (256 threads) per tile: thread = tile position (r, c)
__global__ void __launch_bounds__(256) ldlq_prep_kernel(const __grid_constant__ StepTable tab,
                                                        float* __restrict__ tiles) {
  __shared__ float Ls[112][16];
  __shared__ float Es[112][17];
  const int tile = blockIdx.x;
  const StepJob& J = tab.j[job_of(tab, tile)];
  const int tc = tile - J.tile0;
  const int t = threadIdx.x;
  const int nb = J.below1 - J.below0;
  // stage L[below, r0:r0+16] and (W - W_q)[below, tc*16 : tc*16+16]
  for (int i = t; i < nb * 16; i += 256) {
    const int s = i >> 4, q = i & 15;
    const int64_t row = J.below0 + s;
    Ls[s][q] = J.L[row * J.k + J.r0 + q];
    const int64_t off = row * J.n + (int64_t)tc * 16 + q;
    Es[s][q] = J.W[off] - J.Wq[off];
  }
  __syncthreads();
  const int r = t >> 4, c = t & 15;
  float acc = 0.f;
  for (int s = 0; s < nb; ++s) acc = fmaf(Ls[s][r], Es[s][c], acc);
  const int64_t off = (int64_t)(J.r0 + r) * J.n + (int64_t)tc * 16 + c;
  const float comp = J.prod[off] + acc;
  tiles[(size_t)tile * 256 + c_perm_inv[t]] = J.W[off] + comp;
}

__global__ void __launch_bounds__(256) ldlq_post_kernel(const __grid_constant__ StepTable tab,
                                                        const float* __restrict__ qw,
                                                        const int16_t* __restrict__ qi) {
  const int tile = blockIdx.x;
  const StepJob& J = tab.j[job_of(tab, tile)];
  const int tc = tile - J.tile0;
  const int t = threadIdx.x;  // tile position (r, c)
  const int r = t >> 4, c = t & 15;
  J.Wq[(int64_t)(J.r0 + r) * J.n + (int64_t)tc * 16 + c] = qw[(size_t)tile * 256 + c_perm_inv[t]];
  // encoder order is the container order: copy as is
  J.enc[((int64_t)(J.r0 >> 4) * (J.n >> 4) + tc) * 256 + t] = qi[(size_t)tile * 256 + t];
}

// prod[0:rows_above, :] += L[span, 0:rows_above]^T (W - W_q)[span, :]
// 64 x 64 output tile per CTA, 256 threads x (4 x 4) outputs, span rows in
// chunks of 16 staged in shared memory.
__global__ void __launch_bounds__(256) ldlq_span_kernel(const float* __restrict__ W,
                                                        const float* __restrict__ Wq,
                                                        const float* __restrict__ L,
                                                        float* __restrict__ prod, int64_t k,
                                                        int64_t n, int span0, int span_rows,
                                                        int rows_above) {
  __shared__ float As[16][64];  // As[s][r] = L[span0 + s][r0 + r]
  __shared__ float Bs[16][64];  // Bs[s][c] = (W - W_q)[span0 + s][c0 + c]
  const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
  const int t = threadIdx.x;
  const int tr = (t >> 4) * 4, tcl = (t & 15) * 4;
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
  for (int s0 = 0; s0 < span_rows; s0 += 16) {
    for (int i = t; i < 16 * 64; i += 256) {
      const int s = i >> 6, q = i & 63;
      const int64_t row = span0 + s0 + s;
      const int rr = r0 + q, cc = c0 + q;
      As[s][q] = (rr < rows_above) ? L[row * k + rr] : 0.f;
      Bs[s][q] = (cc < n) ? (W[row * n + cc] - Wq[row * n + cc]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int s = 0; s < 16; ++s) {
      float a[4], b[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        a[x] = As[s][tr + x];
        b[x] = Bs[s][tcl + x];
      }
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(a[x], b[y], acc[x][y]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int rr = r0 + tr + x;
    if (rr >= rows_above) continue;
#pragma unroll
    for (int y = 0; y < 4; ++y) {
      const int cc = c0 + tcl + y;
      if (cc < n) prod[(int64_t)rr * n + cc] += acc[x][y];
    }
  }
}

// tensor-core permutation (trellis_format.py:88-108)
void tc_perm(int16_t* perm, int16_t* inv) {
  for (int t = 0; t < 32; ++t) {
    const int r0 = (t % 4) * 2, c0 = t / 4;
    const int rows[4] = {r0, r0 + 1, r0 + 8, r0 + 9};
    const int cols[2] = {c0, c0 + 8};
    for (int j = 0; j < 2; ++j)
      for (int i = 0; i < 4; ++i) {
        const int q = t * 8 + 4 * j + i;
        perm[q] = (int16_t)(rows[i] * 16 + cols[j]);
      }
  }
  for (int q = 0; q < 256; ++q) inv[perm[q]] = (int16_t)q;
}

size_t align_up(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace
}  // namespace exl3

using namespace exl3;

namespace {

int check_jobs(const exl3_ldlq_job* jobs, int njobs, int buf, bool ptrs = true) {
  EXL3_REQUIRE(jobs != nullptr && njobs >= 1 && njobs <= kMaxJobs,
               "need 1..%d jobs, got %d", kMaxJobs, njobs);
  EXL3_REQUIRE(buf >= 16 && buf <= 128 && buf % 16 == 0,
               "buf_size_k must be a multiple of 16 in [16, 128], got %d", buf);
  for (int i = 0; i < njobs; ++i) {
    const exl3_ldlq_job& J = jobs[i];
    EXL3_REQUIRE(!ptrs || (J.W && J.L && J.W_q && J.encoded), "job %d: NULL pointer", i);
    EXL3_REQUIRE(J.k > 0 && J.k % buf == 0, "job %d: rows (%lld) must be a multiple of buf (%d)",
                 i, (long long)J.k, buf);
    EXL3_REQUIRE(J.n > 0 && J.n % 128 == 0, "job %d: columns (%lld) must be a multiple of 128", i,
                 (long long)J.n);
    EXL3_REQUIRE(J.k < (1ll << 24) && J.n < (1ll << 24), "job %d: matrix too large", i);
  }
  return EXL3_OK;
}

// workspace: per job prod (k*n f32); shared: tiles in (T*256 f32), recon
// (T*256 f32), states (T*256 i16), encoder workspace for T tiles
void ws_layout(const exl3_ldlq_job* jobs, int njobs, int K, size_t* prod_off, size_t* tiles_off,
               size_t* qw_off, size_t* qi_off, size_t* enc_off, size_t* enc_bytes,
               size_t* total) {
  size_t off = 0;
  int64_t T = 0;
  for (int i = 0; i < njobs; ++i) {
    prod_off[i] = off;
    off = align_up(off + (size_t)jobs[i].k * jobs[i].n * 4);
    T += jobs[i].n / 16;
  }
  *tiles_off = off;
  off = align_up(off + (size_t)T * 256 * 4);
  *qw_off = off;
  off = align_up(off + (size_t)T * 256 * 4);
  *qi_off = off;
  off = align_up(off + (size_t)T * 256 * 2);
  *enc_off = off;
  *enc_bytes = exl3_quantize_tiles_ws_bytes(T, K, 256);
  *total = off + *enc_bytes;
}

// Estimated device time (arbitrary units) of one LDLQ step that encodes
// `tiles` tiles at K bits: the encoder's latency floor by cluster split for
// few tile pairs (measured: ~0.45 at 8 CTAs per pair, ~0.6 at 8 CTAs per 2
// pairs, 0.57-0.78 at 4, 0.8 at 2), one unit per wave of one pair per SM
// beyond that.
void step_costs(int K, int max_tiles, std::vector<double>& cost) {
  cost.assign((size_t)max_tiles + 1, 0.0);
  const int sms = sm_count();
  for (int t = 1; t <= max_tiles; ++t) {
    if (K == 1) {
      cost[t] = 1.3 * (double)((t + sms - 1) / sms);
      continue;
    }
    const int pairs = (t + 1) / 2;
    int c = 1, pp = 1;
    cluster_choice(K, pairs, &c, &pp);
    if (c == 8) cost[t] = pp == 1 ? 0.45 : 0.6;
    else if (c == 4) cost[t] = K == 2 ? 0.78 : 0.57;
    else if (c == 2) cost[t] = 0.8;
    else cost[t] = (double)((pairs + sms - 1) / sms);
  }
}

// First step of each job. The longest job spans every step; the others are
// independent of it, so each may start at any step that lets it finish by
// the end. Jobs are placed longest first, then widest, each at the start
// that adds the least estimated time (earliest on ties): on one GPU this
// front-loads the short matrices into steps that already take several
// waves; on a column-sharded GPU it keeps a step out of a second wave by
// moving a matrix into steps that encode only a few tiles.
void schedule_jobs(const exl3_ldlq_job* jobs, int njobs, int K, int64_t* start) {
  int64_t H = 0, total = 0;
  for (int i = 0; i < njobs; ++i) {
    H = std::max<int64_t>(H, jobs[i].k / 16);
    total += jobs[i].n / 16;
  }
  std::vector<double> cost;
  step_costs(K, (int)total, cost);
  std::vector<int> order(njobs);
  for (int i = 0; i < njobs; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
    if (jobs[a].k != jobs[b].k) return jobs[a].k > jobs[b].k;
    return jobs[a].n > jobs[b].n;
  });
  std::vector<int64_t> load((size_t)H, 0);
  std::vector<double> delta((size_t)H + 1, 0.0);
  for (int i : order) {
    const int64_t len = jobs[i].k / 16, tl = jobs[i].n / 16;
    for (int64_t st = 0; st < H; ++st) delta[st + 1] = delta[st] + cost[load[st] + tl] - cost[load[st]];
    int64_t best = 0;
    double best_c = delta[len] - delta[0];
    for (int64_t s0 = 1; s0 + len <= H; ++s0) {
      const double c = delta[s0 + len] - delta[s0];
      if (c < best_c - 1e-9) {
        best_c = c;
        best = s0;
      }
    }
    start[i] = best;
    for (int64_t st = best; st < best + len; ++st) load[st] += tl;
  }
}

}  // namespace

extern "C" int exl3_ldlq_schedule(const exl3_ldlq_job* jobs, int njobs, int K, int buf,
                                  int64_t* start_steps) {
  if (int rc = check_jobs(jobs, njobs, buf, false)) return rc;
  EXL3_REQUIRE(K >= 1 && K <= 8, "K must be in 1..8, got %d", K);
  EXL3_REQUIRE(start_steps != nullptr, "start_steps is NULL");
  schedule_jobs(jobs, njobs, K, start_steps);
  return EXL3_OK;
}

extern "C" size_t exl3_ldlq_ws_bytes(const exl3_ldlq_job* jobs, int njobs, int K, int buf) {
  if (check_jobs(jobs, njobs, buf) != EXL3_OK || K < 1 || K > 8) return 0;
  size_t prod_off[kMaxJobs], t_off, qw_off, qi_off, e_off, e_bytes, total;
  ws_layout(jobs, njobs, K, prod_off, &t_off, &qw_off, &qi_off, &e_off, &e_bytes, &total);
  return e_bytes ? total : 0;
}

extern "C" int exl3_ldlq(const exl3_ldlq_job* jobs, int njobs, int K, int cb, int buf, void* ws,
                         size_t ws_bytes, exl3_stream_t stream) {
  if (int rc = check_jobs(jobs, njobs, buf)) return rc;
  EXL3_REQUIRE(K >= 1 && K <= 8, "K must be in 1..8, got %d", K);
  EXL3_REQUIRE(cb >= 0 && cb <= 2, "cb must be 0, 1 or 2, got %d", cb);
  EXL3_REQUIRE(ws != nullptr, "workspace is NULL");
  size_t prod_off[kMaxJobs], t_off, qw_off, qi_off, e_off, e_bytes, total;
  ws_layout(jobs, njobs, K, prod_off, &t_off, &qw_off, &qi_off, &e_off, &e_bytes, &total);
  EXL3_REQUIRE(ws_bytes >= total, "workspace of %zu bytes is smaller than the %zu needed",
               ws_bytes, total);
  cudaStream_t s = (cudaStream_t)stream;
  {
    static std::mutex mu;
    static uint32_t done = 0;  // permutation tables, one bit per device
    int dev = 0;
    EXL3_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> g(mu);
    if (dev >= 32 || !(done & (1u << dev))) {
      int16_t perm[256], inv[256];
      tc_perm(perm, inv);
      EXL3_CUDA(cudaMemcpyToSymbol(c_perm, perm, sizeof(perm)));
      EXL3_CUDA(cudaMemcpyToSymbol(c_perm_inv, inv, sizeof(inv)));
      if (dev < 32) done |= (1u << dev);
    }
  }
  uint8_t* base = static_cast<uint8_t*>(ws);
  float* tiles = reinterpret_cast<float*>(base + t_off);
  float* qw = reinterpret_cast<float*>(base + qw_off);
  int16_t* qi = reinterpret_cast<int16_t*>(base + qi_off);
  int64_t steps = 0;
  for (int i = 0; i < njobs; ++i) {
    EXL3_CUDA(cudaMemsetAsync(base + prod_off[i], 0, (size_t)jobs[i].k * jobs[i].n * 4, s));
    EXL3_CUDA(cudaMemsetAsync(jobs[i].W_q, 0, (size_t)jobs[i].k * jobs[i].n * 4, s));
    steps = std::max<int64_t>(steps, jobs[i].k / 16);
  }
  int64_t start[kMaxJobs];
  schedule_jobs(jobs, njobs, K, start);
  const int bps = buf / 16;  // blocks per span
  for (int64_t st = 0; st < steps; ++st) {
    StepTable tab;
    tab.njobs = 0;
    int tiles_now = 0;
    for (int i = 0; i < njobs; ++i) {
      const exl3_ldlq_job& J = jobs[i];
      const int64_t ls = st - start[i];  // the job's own step
      if (ls < 0 || ls >= J.k / 16) continue;
      const int span = (int)(ls / bps), blk = (int)(ls % bps);
      const int span0 = (int)(J.k - (int64_t)(span + 1) * buf);
      const int bi = buf - 16 * (blk + 1);
      StepJob& q = tab.j[tab.njobs++];
      q.W = J.W;
      q.L = J.L;
      q.Wq = J.W_q;
      q.prod = reinterpret_cast<float*>(base + prod_off[i]);
      q.enc = J.encoded;
      q.k = J.k;
      q.n = J.n;
      q.r0 = span0 + bi;
      q.below0 = span0 + bi + 16;
      q.below1 = span0 + buf;
      q.tile0 = tiles_now;
      tiles_now += (int)(J.n / 16);
    }
    tab.total_tiles = tiles_now;
    ldlq_prep_kernel<<<tiles_now, 256, 0, s>>>(tab, tiles);
    EXL3_LAUNCHED();
    if (int rc = exl3_quantize_tiles(tiles, qw, qi, nullptr, nullptr, tiles_now, K, cb, 256,
                                     base + e_off, e_bytes, stream))
      return rc;
    ldlq_post_kernel<<<tiles_now, 256, 0, s>>>(tab, qw, qi);
    EXL3_LAUNCHED();
    // spans that just finished: trailing update of the rows above them
    for (int i = 0; i < njobs; ++i) {
      const exl3_ldlq_job& J = jobs[i];
      const int64_t ls = st - start[i];
      if (ls < 0 || ls >= J.k / 16 || ls % bps != bps - 1) continue;
      const int span = (int)(ls / bps);
      const int span0 = (int)(J.k - (int64_t)(span + 1) * buf);
      if (span0 == 0) continue;  // nothing above
      const dim3 grid((unsigned)((J.n + 63) / 64), (unsigned)((span0 + 63) / 64));
      ldlq_span_kernel<<<grid, 256, 0, s>>>(J.W, J.W_q, J.L,
                                            reinterpret_cast<float*>(base + prod_off[i]), J.k,
                                            J.n, span0, buf, span0);
      EXL3_LAUNCHED();
    }
  }
  return EXL3_OK;
}
