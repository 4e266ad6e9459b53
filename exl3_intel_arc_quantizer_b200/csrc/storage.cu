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
// decoded straight into the registers of the thread that rotates its column
// (left rotation, then x su), the right rotation runs on rows through a
// swizzled fp32 shared tile, and the block (x sv) is written once: HBM
// traffic = K/8 B read + 4 B written per weight.
#include <cuda_fp16.h>

#include "common.cuh"
#include "hadamard.cuh"
#include "trellis_span.cuh"

namespace exl3 {
namespace {

constexpr int kDB = 128;          // block edge
constexpr int kDThreads = 256;   // unpack
constexpr int kDecThreads = 256; // decode: two threads per column
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
// tiles); HBM traffic = K/8 B read + 4 B written per weight.
//
// 1. The block's container words become a table of 32-bit windows in shared
//    memory: window m of a tile holds stream words m and m + 1 (circular), so
//    the 16-bit state of element e is one bit-field extract of window
//    floor((K(e+1) - 16) / 16) at bit 16 - (K(e+1) mod 16). The table index
//    is padded per K (WinPad) so that a warp's reads spread over the banks.
// 2. Two threads per column (c, b) decode the 64 elements of column c in rows
//    4i + 2b and 4i + 2b + 1 straight into registers as pairs of adjacent
//    rows (tensor-core positions of trellis_format.py:88-108: consecutive
//    span elements u, u + 1; each tile gives a thread two spans x two pairs)
//    and apply the left rotation: row stride 1 inside each pair, stride 2
//    with the partner lane (one shuffle), strides 4..64 between pairs.
// 3. x su, the right rotation on rows (two threads per row, column pairs
//    4i + 2b, 4i + 2b + 1 read and written as 8-byte words, same scheme),
//    x sv and a row-wise float4 copy-out, through an fp32 shared tile whose
//    rows are XOR-swizzled (column c of row r at c ^ dswz(r)) so that the
//    column stores, the pair accesses and the copy-out are free of bank
//    conflicts.
// Butterflies and scalings run as packed f32x2 operations where two
// independent elements take the same step (each lane rounds like the scalar
// operation). Per element the steps and their roundings are those of
// hadamard.weight_from_quantized: butterflies in the order of strides
// 1, 2, ..., 64 (lower + upper, lower - upper), x 1/sqrt(128), x su, the row
// butterflies, x 1/sqrt(128), x sv.
__device__ __forceinline__ int dswz(int r) {
  return 16 * ((r >> 1) & 1) + 8 * (r & 1) + 4 * ((r >> 2) & 1);
}
__device__ __forceinline__ int dpos(int r, int c) { return r * kDB + (c ^ dswz(r)); }

// window table padding: index m is stored at m + A * (m >> S); (A, S) per K
// chosen so that a warp's reads (16 columns of one tile, both row classes)
// hit distinct banks for K = 1, 2, 4 and at most two-way conflicts otherwise
template <int K> struct WinPad { static constexpr int A = 0, S = 5; };
template <> struct WinPad<3> { static constexpr int A = 5, S = 5; };
template <> struct WinPad<4> { static constexpr int A = 4, S = 3; };
template <> struct WinPad<5> { static constexpr int A = 3, S = 2; };
template <> struct WinPad<7> { static constexpr int A = 1, S = 5; };
template <> struct WinPad<8> { static constexpr int A = 1, S = 2; };
template <int K>
__device__ __forceinline__ int wpad(int m) { return m + WinPad<K>::A * (m >> WinPad<K>::S); }
template <int K>
__host__ __device__ constexpr int win_stride() {
  return 16 * K + WinPad<K>::A * ((16 * K - 1) >> WinPad<K>::S);
}

__device__ __forceinline__ float2 f2_add(float2 a, float2 b) { return __fadd2_rn(a, b); }
// a - b with one rounding: (-1) * b is exact
__device__ __forceinline__ float2 f2_sub(float2 a, float2 b) {
  return __ffma2_rn(b, make_float2(-1.0f, -1.0f), a);
}

// 128-point butterflies over a line held by two lanes as pairs of adjacent
// elements w[p] = (v[4p + 2b], v[4p + 2b + 1]) (b = lane bit 0): stride 1
// inside each pair, stride 2 with the partner lane (lower = mine + other,
// upper = other - mine), strides 4..64 between pairs, x 1/sqrt(128)
__device__ __forceinline__ void fwht128_pair_line(float2 (&w)[32], float sign) {
#pragma unroll
  for (int p = 0; p < 32; ++p) {
    const float lo = w[p].x, hi = w[p].y;
    w[p] = make_float2(lo + hi, lo - hi);
  }
  const float2 sg = make_float2(sign, sign);
#pragma unroll
  for (int p = 0; p < 32; ++p) {
    // one 64-bit shuffle: both halves land in a register pair
    const unsigned long long mine = *reinterpret_cast<const unsigned long long*>(&w[p]);
    const unsigned long long theirs = __shfl_xor_sync(0xFFFFFFFFu, mine, 1);
    const float2 o = *reinterpret_cast<const float2*>(&theirs);
    w[p] = __ffma2_rn(sg, w[p], o);
  }
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
#pragma unroll
    for (int p = 0; p < 32; ++p) {
      if (p & h) continue;
      const float2 lo = w[p], hi = w[p + h];
      w[p] = f2_add(lo, hi);
      w[p + h] = f2_sub(lo, hi);
    }
  }
  const float2 sc = make_float2(kHad128Scale, kHad128Scale);
#pragma unroll
  for (int p = 0; p < 32; ++p) w[p] = __fmul2_rn(w[p], sc);
}

// two codebook values (the states' fp16 values widened to fp32)
template <int CB>
__device__ __forceinline__ float2 cb_decode2(uint32_t s0, uint32_t s1) {
  if constexpr (CB == 2) {
    // 0x6400 + byte sum of s * 0x83DCD12D (< 2^16), then h * inv + bias in
    // fp16 for both lanes at once
    const uint32_t h0 = __dp4a(s0 * 0x83DCD12Du, 0x01010101u, 0x6400u);
    const uint32_t h1 = __dp4a(s1 * 0x83DCD12Du, 0x01010101u, 0x6400u);
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(h0 | (h1 << 16)), "r"(0x1EEE1EEEu),
        "r"(0xC931C931u));
    return __half22float2(*reinterpret_cast<const __half2*>(&r));
  } else {
    return make_float2(half_bits_to_float(cb_state_bits(CB, s0)),
                       half_bits_to_float(cb_state_bits(CB, s1)));
  }
}

__device__ __forceinline__ uint32_t bits16_at(uint32_t w, uint32_t pos) {
  uint32_t r;
  asm("bfe.u32 %0, %1, %2, 16;" : "=r"(r) : "r"(w), "r"(pos));
  return r;
}

// K = 4 and K = 8: K (e + 1) mod 16 depends only on e mod 4 (K = 4: the
// thread's 2x + j, K = 8: j), so the window bit of slot k is a constant
template <int K>
__device__ __forceinline__ constexpr bool const_window_bit() { return K == 4 || K == 8; }
template <int K>
__device__ __forceinline__ constexpr uint32_t window_bit_of_slot(int k) {
  // slot k = 4x + 2sp + j; e = 16 * (...) + 2x + 8b + j + 4 (lc >> 3)
  return 16u - (uint32_t)((K * (2 * (k >> 2) + (k & 1) + 1)) & 15);
}

template <int K>
constexpr size_t decode_smem_bytes() {
  return (size_t)kDB * kDB * 4 + (size_t)64 * win_stride<K>() * 4;
}

template <int K, int CB, int SCALE_F32>
__global__ void __launch_bounds__(kDecThreads, 2)
decode_weight_kernel(const uint16_t* __restrict__ trellis, const void* __restrict__ su,
                     const void* __restrict__ sv, float* __restrict__ out,
                     float* __restrict__ out_w_hat, int64_t tiles_n, int64_t n) {
  extern __shared__ __align__(16) uint8_t dsmem[];
  float* blk = reinterpret_cast<float*>(dsmem);                    // 128 x 128 fp32, swizzled
  uint32_t* win = reinterpret_cast<uint32_t*>(blk + kDB * kDB);    // 64 tiles x win_stride
  constexpr int kW32 = 8 * K;          // 32-bit container words per tile
  constexpr int kWS = win_stride<K>();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t rb = blockIdx.y, cbk = blockIdx.x;

  // the scales are loaded first, so that their latency hides behind phase 1
  const int b = tid & 1, c = tid >> 1, lc = c & 15, tcb = c >> 4;
  const float sur = load_scale<SCALE_F32>(su, rb * kDB + c);
  float2 sv01, sv23;
  sv01.x = load_scale<SCALE_F32>(sv, cbk * kDB + 4 * lane);
  sv01.y = load_scale<SCALE_F32>(sv, cbk * kDB + 4 * lane + 1);
  sv23.x = load_scale<SCALE_F32>(sv, cbk * kDB + 4 * lane + 2);
  sv23.y = load_scale<SCALE_F32>(sv, cbk * kDB + 4 * lane + 3);

  // 1. windows. Each tile row of the block is one contiguous run of 8 tiles
  //    (8 * kW32 words); all 2K words a thread copies are loaded at once (one
  //    DRAM round trip per CTA, not one per tile row). Stored 32-bit word q is
  //    stream words 2q + 1, 2q (SWAP16), so window 2q is the word itself and
  //    window 2q + 1 joins its low half with the next word's high half; the
  //    next word comes from a shuffle where a tile fits in a warp (K = 1, 2,
  //    4), else from a copy staged in the fp32 tile's space (free until
  //    phase 2 has read the windows)
  {
    constexpr int kRun = 8 * kW32;
    static_assert(8 * kRun <= kDB * kDB, "the staged container must fit in the fp32 tile");
    uint32_t* stage = reinterpret_cast<uint32_t*>(blk);  // 64 tiles x kW32, block order
    uint32_t v[2 * K];
#pragma unroll
    for (int it = 0; it < 2 * K; ++it) {
      const int i = it * kDecThreads + tid, tr = i / kRun;
      v[it] = reinterpret_cast<const uint32_t*>(
          trellis + ((rb * 8 + tr) * tiles_n + cbk * 8) * (int64_t)(16 * K))[i - tr * kRun];
    }
    if constexpr (32 % kW32 == 0) {
      // K = 1, 2, 4: a tile's words sit in kW32 consecutive lanes of one
      // warp, so the next word (circular) is one shuffle away
#pragma unroll
      for (int it = 0; it < 2 * K; ++it) {
        const int i = it * kDecThreads + tid, t = i / kW32, q = i - t * kW32;
        const uint32_t nx = __shfl_sync(0xFFFFFFFFu, v[it], lane + 1, kW32);
        uint32_t* tw = win + t * kWS;
        tw[wpad<K>(2 * q)] = v[it];
        tw[wpad<K>(2 * q + 1)] = (v[it] << 16) | (nx >> 16);
      }
    } else {
#pragma unroll
      for (int it = 0; it < 2 * K; ++it) stage[it * kDecThreads + tid] = v[it];
      __syncthreads();
#pragma unroll
      for (int it = 0; it < 2 * K; ++it) {
        const int i = it * kDecThreads + tid, t = i / kW32, q = i - t * kW32;
        const uint32_t a = stage[i];
        const uint32_t nx = stage[t * kW32 + (q + 1 < kW32 ? q + 1 : 0)];
        uint32_t* tw = win + t * kWS;
        tw[wpad<K>(2 * q)] = a;
        tw[wpad<K>(2 * q + 1)] = (a << 16) | (nx >> 16);
      }
    }
  }
  __syncthreads();

  // 2. two threads per column: c = tid / 2, rows 4i + 2b + j. In tile row tr
  //    the column's local index lc takes spans s = 2 (lc & 7) + sp and span
  //    elements u = 4 (lc >> 3) + 2x + 8b + j; element e = 16 s + u sits at
  //    local row 4 sp + 8x + 2b + j, i.e. pair index 4 tr + sp + 2x
  int woff[8];
  uint32_t wbit[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {  // k = 4x + 2sp + j
    const int x = k >> 2, sp = (k >> 1) & 1, j = k & 1;
    const int e = 32 * (lc & 7) + 16 * sp + 4 * (lc >> 3) + 2 * x + 8 * b + j;
    const int be = K * (e + 1);  // the state is stream bits [be - 16, be)
    int m = (be + 256 * K - 16) >> 4;
    if (m >= 16 * K) m -= 16 * K;
    woff[k] = wpad<K>(m);
    wbit[k] = 16u - (uint32_t)(be & 15);
  }
  float2 w[32];  // w[p]: rows 4p + 2b, 4p + 2b + 1 of column c
#pragma unroll
  for (int tr = 0; tr < 8; ++tr) {
    const uint32_t* tw = win + (tr * 8 + tcb) * kWS;
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      uint32_t s0, s1;
      if constexpr (const_window_bit<K>()) {
        // one window holds both states of the pair (they overlap in 16 - K
        // bits; the first starts at most 16 - K bits into the window)
        constexpr uint32_t kMask = 0xFFFFu;
        const uint32_t win0 = tw[woff[k]];
        s0 = (win0 >> window_bit_of_slot<K>(k)) & kMask;
        s1 = (win0 >> (window_bit_of_slot<K>(k) - K)) & kMask;
      } else if constexpr (K == 1 || K == 2) {
        const uint32_t win0 = tw[woff[k]];
        s0 = bits16_at(win0, wbit[k]);
        s1 = bits16_at(win0, wbit[k] - K);
      } else {
        s0 = bits16_at(tw[woff[k]], wbit[k]);
        s1 = bits16_at(tw[woff[k + 1]], wbit[k + 1]);
      }
      const int x = k >> 2, sp = (k >> 1) & 1;
      w[4 * tr + sp + 2 * x] = cb_decode2<CB>(s0, s1);
    }
  }

  if (out_w_hat) {  // transformed-basis reconstruction, before the rotations
#pragma unroll
    for (int p = 0; p < 32; ++p) {
      blk[dpos(4 * p + 2 * b, c)] = w[p].x;
      blk[dpos(4 * p + 2 * b + 1, c)] = w[p].y;
    }
    __syncthreads();
    for (int r = warp; r < kDB; r += kDecThreads / 32) {
      const float4 o = *reinterpret_cast<const float4*>(blk + r * kDB + ((4 * lane) ^ dswz(r)));
      *reinterpret_cast<float4*>(out_w_hat + (rb * kDB + r) * n + cbk * kDB + 4 * lane) = o;
    }
    __syncthreads();
  }

  const float sign = b ? -1.0f : 1.0f;
  // left rotation on the column, x 1/sqrt(128)
  fwht128_pair_line(w, sign);
#pragma unroll
  for (int p = 0; p < 32; ++p) {
    blk[dpos(4 * p + 2 * b, c)] = w[p].x;
    blk[dpos(4 * p + 2 * b + 1, c)] = w[p].y;
  }
  __syncthreads();
  // 3. x su, then the right rotation on every row (two threads per row:
  //    column pairs 4i + 2b, 4i + 2b + 1), x 1/sqrt(128). Column pair p =
  //    8m + k sits at 32m + ((4k) ^ dswz(r)) + 2b: eight per-thread
  //    pointers, the rest immediate offsets
  {
    const int r = c;
    const float2 su2 = make_float2(sur, sur);
    const int f = dswz(r);
    float2* rp[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      rp[k] = reinterpret_cast<float2*>(blk + r * kDB + ((4 * k) ^ f) + 2 * b);
#pragma unroll
    for (int p = 0; p < 32; ++p) w[p] = __fmul2_rn(rp[p & 7][16 * (p >> 3)], su2);
    fwht128_pair_line(w, sign);
#pragma unroll
    for (int p = 0; p < 32; ++p) rp[p & 7][16 * (p >> 3)] = w[p];
  }
  __syncthreads();
  // x sv (per column) and the block written row by row with float4 stores
  for (int r = warp; r < kDB; r += kDecThreads / 32) {
    const float4 o = *reinterpret_cast<const float4*>(blk + r * kDB + ((4 * lane) ^ dswz(r)));
    const float2 lo = __fmul2_rn(make_float2(o.x, o.y), sv01);
    const float2 hi = __fmul2_rn(make_float2(o.z, o.w), sv23);
    *reinterpret_cast<float4*>(out + (rb * kDB + r) * n + cbk * kDB + 4 * lane) =
        make_float4(lo.x, lo.y, hi.x, hi.y);
  }
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
                                   (int)decode_smem_bytes<K>()));
    attr_done.set(dev);
  }
  const dim3 grid((unsigned)(tiles_n / 8), (unsigned)(tiles_k / 8));
  decode_weight_kernel<K, CB, F32><<<grid, kDecThreads, decode_smem_bytes<K>(), stream>>>(
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
