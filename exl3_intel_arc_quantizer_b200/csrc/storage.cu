// EXL3 storage side on B200: unpack the trellis container and decode the
// original-basis weight in one pass.
//
// Reference: exl3_quant/serialization.py:65-84 (unpack_module_trellis) and
// :227-266 (decode_weight_from_storage: states -> codebook -> inverse tile
// permutation -> weight_from_quantized, hadamard.py:122-140).
//
// Container (trellis_format.py:120-174): a tile's 256*K-bit stream is its
// 16*K packed 16-bit words in order, each read MSB-first; storage exchanges
// the halves of every 32-bit word (SWAP16). Element t's 16-bit state is the
// window of the circular stream that ends at bit (t+1)*K.
//
// decode_weight_kernel: one CTA per 128x128 block of the (k, n) weight (8x8
// tiles). The block's container words are read once, each element is
// decoded into a padded fp32 shared tile at its tensor-core position, then
// the left rotation (columns, with the row scales su) and the right
// rotation (rows, with the column scales sv) run in shared memory and the
// block is written once: HBM traffic = K/8 B read + 4 B written per weight.
#include <cuda_fp16.h>

#include "common.cuh"
#include "hadamard.cuh"
#include "trellis_span.cuh"

namespace exl3 {
namespace {

constexpr int kDB = 128;          // block edge
constexpr int kDThreads = 256;   // unpack
constexpr int kDecThreads = 256; // decode: four spans per thread
constexpr int kUTiles = 16;       // tiles per unpack CTA (two per warp)

// unpack: one thread per span. A warp stages its two tiles' container words
// in shared memory with coalesced 32-bit loads, then each lane extracts the
// 16 states of one span and writes them as two 16-byte stores.
template <int K>
__global__ void __launch_bounds__(kDThreads)
unpack_trellis_kernel(const uint32_t* __restrict__ trellis, int16_t* __restrict__ states,
                      int64_t ntiles) {
  __shared__ uint16_t words[kUTiles * 16 * K];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int64_t tile0 = (int64_t)blockIdx.x * kUTiles + 2 * warp;  // this warp's first tile
  const int nt = (int)(ntiles - tile0 < 2 ? ntiles - tile0 : 2);
  if (nt <= 0) return;
  uint32_t* wsm = reinterpret_cast<uint32_t*>(words + 2 * warp * 16 * K);
  for (int i = lane; i < nt * 8 * K; i += 32) wsm[i] = trellis[tile0 * 8 * K + i];
  __syncwarp();
  const int tt = lane >> 4, sp = lane & 15;
  if (tt >= nt) return;
  const uint16_t* tw = words + (2 * warp + tt) * 16 * K;
  uint32_t st[16];
  span_states<K>([&](int j) { return (uint32_t)tw[j ^ 1]; }, sp, st);
  uint4* dst = reinterpret_cast<uint4*>(states + (tile0 + tt) * 256 + 16 * sp);
  dst[0] = make_uint4(st[0] | (st[1] << 16), st[2] | (st[3] << 16), st[4] | (st[5] << 16),
                      st[6] | (st[7] << 16));
  dst[1] = make_uint4(st[8] | (st[9] << 16), st[10] | (st[11] << 16), st[12] | (st[13] << 16),
                      st[14] | (st[15] << 16));
}

template <int SCALE_F32>
__device__ __forceinline__ float load_scale(const void* p, int64_t i) {
  if (SCALE_F32) return static_cast<const float*>(p)[i];
  return __half2float(static_cast<const __half*>(p)[i]);
}

// decode_weight_kernel: one CTA per 128x128 block of the (k, n) weight (8x8
// tiles). The block's container words are read once; each thread decodes
// four spans (16 states each, fixed tile positions) into an fp32 shared
// tile; the left rotation runs on columns, the right one on rows, and the
// block is written once: HBM traffic = K/8 B read + 4 B written per weight.
//
// Both rotations give each thread 64 elements of one column (or row) - the
// elements of one parity, its partner lane holding the other - so the
// stride-1 butterfly is one shuffle and the six wider ones run in registers
// (one shuffle per element per rotation instead of five). The shared tile is
// stored with the rows XOR-swizzled (column c of row r at c ^ dswz(r)) so
// that both thread mappings and the row-wise float4 copy-out are free of bank
// conflicts. Per element the steps and their roundings are those of
// hadamard.weight_from_quantized: butterflies in the order of strides
// 1, 2, ..., 64 (lower + upper, lower - upper), x 1/sqrt(128), x su, the row
// butterflies, x 1/sqrt(128), x sv.
__device__ __forceinline__ int dswz(int r) { return 2 * (((r & 1) << 3) | ((r >> 1) & 7)); }
__device__ __forceinline__ int dpos(int r, int c) { return r * kDB + (c ^ dswz(r)); }

// in-register butterflies of strides 1..32 over v[0..63] (element stride 2h in
// the block: the caller's stride-1 partner is another lane)
__device__ __forceinline__ void fwht64_regs(float (&v)[64]) {
#pragma unroll
  for (int h = 1; h < 64; h <<= 1) {
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      if (i & h) continue;
      const float lo = v[i], hi = v[i + h];
      v[i] = lo + hi;
      v[i + h] = lo - hi;
    }
  }
}

template <int K, int CB, int SCALE_F32>
__global__ void __launch_bounds__(kDecThreads, 2)
decode_weight_kernel(const uint16_t* __restrict__ trellis, const void* __restrict__ su,
                     const void* __restrict__ sv, float* __restrict__ out,
                     float* __restrict__ out_w_hat, int64_t tiles_n, int64_t n) {
  extern __shared__ __align__(16) uint8_t dsmem[];
  float* blk = reinterpret_cast<float*>(dsmem);                     // 128 x 128 fp32, swizzled
  uint16_t* words = reinterpret_cast<uint16_t*>(blk + kDB * kDB);   // 64 tiles x 16K
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t rb = blockIdx.y, cbk = blockIdx.x;
  constexpr int wpt = 16 * K;  // storage words per tile

  // 1. container words: each tile row of the block is one contiguous run of
  //    8 tiles (8 * 32K bytes), copied as 32-bit words
#pragma unroll
  for (int tr = 0; tr < 8; ++tr) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(
        trellis + ((rb * 8 + tr) * tiles_n + cbk * 8) * (int64_t)wpt);
    uint32_t* dst = reinterpret_cast<uint32_t*>(words + tr * 8 * wpt);
    for (int i = tid; i < 4 * wpt; i += kDecThreads) dst[i] = src[i];
  }
  __syncthreads();

  // 2. decode: four spans per thread; span s of tile tt holds elements
  //    16s..16s+15, whose tensor-core positions (trellis_format.py:88-108)
  //    are (4(s&1) + dr(u), (s>>1) + dc(u)) with compile-time dr, dc
#pragma unroll
  for (int q = 0; q < 1024 / kDecThreads; ++q) {
    const int spid = q * kDecThreads + tid;
    const int tt = spid >> 4, s = spid & 15;
    const uint16_t* tw = words + tt * wpt;
    uint32_t st[16];
    span_states<K>([&](int j) { return (uint32_t)tw[j ^ 1]; }, s, st);
    const int r0 = (tt >> 3) * 16 + 4 * (s & 1), c0 = (tt & 7) * 16 + (s >> 1);
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int dr = 2 * (u >> 3) + (u & 1) + 8 * ((u >> 1) & 1);
      const int dc = 8 * ((u >> 2) & 1);
      blk[dpos(r0 + dr, c0 + dc)] = __half2float(__ushort_as_half(cb_state_bits(CB, st[u])));
    }
  }
  __syncthreads();

  if (out_w_hat) {  // transformed-basis reconstruction, before the rotations
    for (int r = warp; r < kDB; r += kDecThreads / 32) {
      const int f = dswz(r);
      const float4 p = *reinterpret_cast<const float4*>(blk + r * kDB + ((4 * lane) ^ (f & ~3)));
      const float4 o = (f & 2) ? make_float4(p.z, p.w, p.x, p.y) : p;
      *reinterpret_cast<float4*>(out_w_hat + (rb * kDB + r) * n + cbk * kDB + 4 * lane) = o;
    }
  }

  float v[64];
  const int b = tid & 1;
  const float sign = b ? -1.0f : 1.0f;
  // 3. H_l on every column (thread pair per column: rows 2i + b), x 1/sqrt(128)
  {
    const int c = tid >> 1;
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = blk[dpos(2 * i + b, c)];
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = had_bfly(v[i], __shfl_xor_sync(0xFFFFFFFFu, v[i], 1), sign);
    fwht64_regs(v);
#pragma unroll
    for (int i = 0; i < 64; ++i) blk[dpos(2 * i + b, c)] = v[i] * kHad128Scale;
  }
  __syncthreads();
  // 4. x su, then H_r on every row (thread pair per row: columns 2i + b),
  //    x 1/sqrt(128)
  {
    const int r = tid >> 1;
    const float sur = load_scale<SCALE_F32>(su, rb * kDB + r);
    const int f = dswz(r);
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = blk[r * kDB + ((2 * i + b) ^ f)] * sur;
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = had_bfly(v[i], __shfl_xor_sync(0xFFFFFFFFu, v[i], 1), sign);
    fwht64_regs(v);
#pragma unroll
    for (int i = 0; i < 64; ++i) blk[r * kDB + ((2 * i + b) ^ f)] = v[i] * kHad128Scale;
  }
  __syncthreads();
  // 5. x sv (per column) and the block written row by row with float4 stores
  float svc[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) svc[e] = load_scale<SCALE_F32>(sv, cbk * kDB + 4 * lane + e);
  for (int r = warp; r < kDB; r += kDecThreads / 32) {
    const int f = dswz(r);
    const float4 p = *reinterpret_cast<const float4*>(blk + r * kDB + ((4 * lane) ^ (f & ~3)));
    const float4 o = (f & 2) ? make_float4(p.z, p.w, p.x, p.y) : p;
    *reinterpret_cast<float4*>(out + (rb * kDB + r) * n + cbk * kDB + 4 * lane) =
        make_float4(o.x * svc[0], o.y * svc[1], o.z * svc[2], o.w * svc[3]);
  }
}

constexpr size_t decode_smem_bytes(int K) {
  return (size_t)kDB * kDB * 4 + (size_t)64 * 16 * K * 2;
}

template <int K, int CB, int F32>
int launch_decode(const uint16_t* tw, const void* su, const void* sv, float* out, float* w_hat,
                  int64_t tiles_k, int64_t tiles_n, cudaStream_t stream) {
  static DeviceBits attr_done;
  int dev = 0;
  EXL3_CUDA(cudaGetDevice(&dev));
  if (!attr_done.has(dev)) {
    EXL3_CUDA(cudaFuncSetAttribute(decode_weight_kernel<K, CB, F32>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)decode_smem_bytes(K)));
    attr_done.set(dev);
  }
  const dim3 grid((unsigned)(tiles_n / 8), (unsigned)(tiles_k / 8));
  decode_weight_kernel<K, CB, F32><<<grid, kDecThreads, decode_smem_bytes(K), stream>>>(
      tw, su, sv, out, w_hat, tiles_n, tiles_n * 16);
  EXL3_LAUNCHED();
  return EXL3_OK;
}

template <int K>
int decode_k(int cb, int f32, const uint16_t* tw, const void* su, const void* sv, float* out,
             float* w_hat, int64_t tiles_k, int64_t tiles_n, cudaStream_t stream) {
  if (cb == 0)
    return f32 ? launch_decode<K, 0, 1>(tw, su, sv, out, w_hat, tiles_k, tiles_n, stream)
               : launch_decode<K, 0, 0>(tw, su, sv, out, w_hat, tiles_k, tiles_n, stream);
  if (cb == 1)
    return f32 ? launch_decode<K, 1, 1>(tw, su, sv, out, w_hat, tiles_k, tiles_n, stream)
               : launch_decode<K, 1, 0>(tw, su, sv, out, w_hat, tiles_k, tiles_n, stream);
  return f32 ? launch_decode<K, 2, 1>(tw, su, sv, out, w_hat, tiles_k, tiles_n, stream)
             : launch_decode<K, 2, 0>(tw, su, sv, out, w_hat, tiles_k, tiles_n, stream);
}

}  // namespace
}  // namespace exl3

using namespace exl3;

extern "C" int exl3_unpack_trellis(const int16_t* trellis, int16_t* states, int64_t ntiles, int K,
                                   exl3_stream_t stream) {
  EXL3_REQUIRE(K >= 1 && K <= 8, "K must be in 1..8, got %d", K);
  EXL3_REQUIRE(ntiles >= 0, "ntiles must be non-negative");
  if (ntiles == 0) return EXL3_OK;
  EXL3_REQUIRE(trellis && states, "NULL pointer argument");
  EXL3_REQUIRE(reinterpret_cast<uintptr_t>(trellis) % 4 == 0, "trellis must be 4-byte aligned");
  EXL3_REQUIRE(reinterpret_cast<uintptr_t>(states) % 16 == 0, "states must be 16-byte aligned");
  const int64_t blocks = (ntiles + kUTiles - 1) / kUTiles;
  EXL3_REQUIRE(blocks < (1ll << 31), "too many tiles");
  const uint32_t* tw = reinterpret_cast<const uint32_t*>(trellis);
  cudaStream_t s = (cudaStream_t)stream;
  EXL3_SWITCH_K(K, (unpack_trellis_kernel<KK><<<(unsigned)blocks, kDThreads, 0, s>>>(tw, states,
                                                                                     ntiles)));
  EXL3_LAUNCHED();
  return EXL3_OK;
}

extern "C" int exl3_decode_weight(const int16_t* trellis, const void* su, const void* sv,
                                  int scale_dtype, float* out, float* out_w_hat, int64_t tiles_k,
                                  int64_t tiles_n, int K, int cb, exl3_stream_t stream) {
  EXL3_REQUIRE(K >= 1 && K <= 8, "K must be in 1..8, got %d", K);
  EXL3_REQUIRE(cb >= 0 && cb <= 2, "codebook must be 0 (3INST), 1 (MCG) or 2 (MUL1), got %d", cb);
  EXL3_REQUIRE(scale_dtype == 0 || scale_dtype == 1,
               "scale_dtype must be 0 (fp16) or 1 (fp32), got %d", scale_dtype);
  EXL3_REQUIRE(tiles_k > 0 && tiles_n > 0 && tiles_k % 8 == 0 && tiles_n % 8 == 0,
               "weight dims (%lld x %lld) must be positive multiples of 128",
               (long long)(tiles_k * 16), (long long)(tiles_n * 16));
  EXL3_REQUIRE(trellis && su && sv && out, "NULL pointer argument");
  EXL3_REQUIRE(reinterpret_cast<uintptr_t>(trellis) % 4 == 0, "trellis must be 4-byte aligned");
  EXL3_REQUIRE(tiles_k / 8 < 65536, "too many row blocks");
  const uint16_t* tw = reinterpret_cast<const uint16_t*>(trellis);
  cudaStream_t s = (cudaStream_t)stream;
  int rc = EXL3_OK;
  EXL3_SWITCH_K(K, (rc = decode_k<KK>(cb, scale_dtype, tw, su, sv, out, out_w_hat, tiles_k,
                                      tiles_n, s)));
  return rc;
}
