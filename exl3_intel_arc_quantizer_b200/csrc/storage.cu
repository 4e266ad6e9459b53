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

namespace exl3 {
namespace {

constexpr int kDB = 128;          // block edge
constexpr int kDPitch = kDB + 1;  // padded row pitch (conflict-free column walks)
constexpr int kDThreads = 256;

// packed (un-swapped) word j of a tile whose storage starts at `st`
__device__ __forceinline__ uint32_t packed_word(const uint16_t* st, int j) {
  return st[j ^ 1];
}

// the 16-bit state of element t from a tile's storage words (16*K words)
__device__ __forceinline__ uint32_t tile_state(const uint16_t* st, int K, int t) {
  const int nbits = 256 * K;
  const int nwords = 16 * K;
  int b0 = (t + 1) * K - 16;
  if (b0 < 0) b0 += nbits;
  const int j = b0 >> 4;
  const int j1 = (j + 1 == nwords) ? 0 : j + 1;
  const uint32_t w = (packed_word(st, j) << 16) | packed_word(st, j1);
  return (w >> (16 - (b0 & 15))) & 0xFFFFu;
}

// tensor-core permutation: encoded element t sits at tile position r*16+c
// (trellis_format.py:88-108)
__device__ __forceinline__ void tc_position(int t, int& r, int& c) {
  const int g = t >> 3, w = t & 7;
  const int i = w & 3, j = w >> 2;
  const int r0 = (g & 3) * 2, c0 = g >> 2;
  r = r0 + (i & 1) + ((i >> 1) << 3);
  c = c0 + (j << 3);
}

__global__ void unpack_trellis_kernel(const uint16_t* __restrict__ trellis,
                                      int16_t* __restrict__ states, int64_t ntiles, int K) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= ntiles * 256) return;
  const int64_t tile = i >> 8;
  const int t = (int)(i & 255);
  states[i] = (int16_t)tile_state(trellis + tile * 16 * K, K, t);
}

template <int SCALE_F32>
__device__ __forceinline__ float load_scale(const void* p, int64_t i) {
  if (SCALE_F32) return static_cast<const float*>(p)[i];
  return __half2float(static_cast<const __half*>(p)[i]);
}

template <int SCALE_F32>
__global__ void __launch_bounds__(kDThreads)
decode_weight_kernel(const uint16_t* __restrict__ trellis, const void* __restrict__ su,
                     const void* __restrict__ sv, float* __restrict__ out,
                     float* __restrict__ out_w_hat, int64_t tiles_n, int64_t n, int K, int cb) {
  extern __shared__ __align__(16) uint8_t dsmem[];
  float* blk = reinterpret_cast<float*>(dsmem);                       // 128 x 129 fp32
  uint16_t* words = reinterpret_cast<uint16_t*>(blk + kDB * kDPitch);  // 64 tiles x 16K
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t rb = blockIdx.y, cbk = blockIdx.x;
  const int wpt = 16 * K;  // storage words per tile

  // 1. container words of the 8x8 tiles: each tile row of the block is one
  //    contiguous run of 8 tiles (8 * 32K bytes), copied as 32-bit words
  for (int tr = 0; tr < 8; ++tr) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(
        trellis + ((rb * 8 + tr) * tiles_n + cbk * 8) * (int64_t)wpt);
    uint32_t* dst = reinterpret_cast<uint32_t*>(words + tr * 8 * wpt);
    for (int i = tid; i < 4 * wpt; i += kDThreads) dst[i] = src[i];
  }
  __syncthreads();

  // 2. decode: warp-consecutive elements of one tile
  for (int i = tid; i < 64 * 256; i += kDThreads) {
    const int tt = i >> 8, t = i & 255;
    const uint32_t s = tile_state(words + tt * wpt, K, t);
    const float v = __half2float(__ushort_as_half(cb_state_bits(cb, s)));
    int r, c;
    tc_position(t, r, c);
    blk[((tt >> 3) * 16 + r) * kDPitch + (tt & 7) * 16 + c] = v;
  }
  __syncthreads();

  if (out_w_hat) {  // transformed-basis reconstruction, before the rotations
    for (int i = tid; i < kDB * kDB; i += kDThreads) {
      const int r = i >> 7, c = i & 127;
      out_w_hat[(rb * kDB + r) * n + cbk * kDB + c] = blk[r * kDPitch + c];
    }
  }

  // 3. H_l on every column, then x su (per row)
  for (int c = warp; c < kDB; c += kDThreads / 32) {
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = blk[(lane + 32 * q) * kDPitch + c];
    fwht128_warp(v, lane);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float h = v[q] * kHad128Scale;
      blk[(lane + 32 * q) * kDPitch + c] = h * load_scale<SCALE_F32>(su, rb * kDB + lane + 32 * q);
    }
  }
  __syncthreads();

  // 4. H_r on every row, then x sv (per column), written straight out
  for (int r = warp; r < kDB; r += kDThreads / 32) {
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = blk[r * kDPitch + lane + 32 * q];
    fwht128_warp(v, lane);
    float* dst = out + (rb * kDB + r) * n + cbk * kDB;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float h = v[q] * kHad128Scale;
      dst[lane + 32 * q] = h * load_scale<SCALE_F32>(sv, cbk * kDB + lane + 32 * q);
    }
  }
}

constexpr size_t decode_smem_bytes(int K) {
  return (size_t)kDB * kDPitch * 4 + (size_t)64 * 16 * K * 2;
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
  const int64_t total = ntiles * 256;
  const int64_t blocks = (total + 255) / 256;
  EXL3_REQUIRE(blocks < (1ll << 31), "too many tiles");
  unpack_trellis_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint16_t*>(trellis), states, ntiles, K);
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
  const size_t smem = decode_smem_bytes(K);
  static uint32_t attr_done[2] = {0u, 0u};
  int dev = 0;
  EXL3_CUDA(cudaGetDevice(&dev));
  const uint32_t bit = dev < 32 ? (1u << dev) : 0u;
  const dim3 grid((unsigned)(tiles_n / 8), (unsigned)(tiles_k / 8));
  const int64_t n = tiles_n * 16;
  const uint16_t* tw = reinterpret_cast<const uint16_t*>(trellis);
  if (scale_dtype == 0) {
    if (!(attr_done[0] & bit)) {
      EXL3_CUDA(cudaFuncSetAttribute(decode_weight_kernel<0>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)decode_smem_bytes(8)));
      attr_done[0] |= bit;
    }
    decode_weight_kernel<0><<<grid, kDThreads, smem, (cudaStream_t)stream>>>(
        tw, su, sv, out, out_w_hat, tiles_n, n, K, cb);
  } else {
    if (!(attr_done[1] & bit)) {
      EXL3_CUDA(cudaFuncSetAttribute(decode_weight_kernel<1>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)decode_smem_bytes(8)));
      attr_done[1] |= bit;
    }
    decode_weight_kernel<1><<<grid, kDThreads, smem, (cudaStream_t)stream>>>(
        tw, su, sv, out, out_w_hat, tiles_n, n, K, cb);
  }
  EXL3_LAUNCHED();
  return EXL3_OK;
}
