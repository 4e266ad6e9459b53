// Shared helpers for the libexl3k kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "../../include/exl3k.h"

namespace exl3 {

// ---------------------------------------------------------------------------
// Error reporting: every C entry point returns a status and leaves a message
// in a thread-local buffer read through exl3_last_error().
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);

#define EXL3_REQUIRE(cond, ...)                 \
  do {                                          \
    if (!(cond)) {                              \
      ::exl3::set_error(__VA_ARGS__);           \
      return EXL3_EINVAL;                       \
    }                                           \
  } while (0)

#define EXL3_CUDA(call)                                                   \
  do {                                                                    \
    cudaError_t err__ = (call);                                           \
    if (err__ != cudaSuccess) {                                           \
      ::exl3::set_error("%s failed: %s (%s:%d)", #call,                   \
                        cudaGetErrorString(err__), __FILE__, __LINE__);   \
      return EXL3_ECUDA;                                                  \
    }                                                                     \
  } while (0)

#define EXL3_LAUNCHED()                                                   \
  do {                                                                    \
    cudaError_t err__ = cudaGetLastError();                               \
    if (err__ != cudaSuccess) {                                           \
      ::exl3::set_error("kernel launch failed: %s (%s:%d)",               \
                        cudaGetErrorString(err__), __FILE__, __LINE__);   \
      return EXL3_ECUDA;                                                  \
    }                                                                     \
  } while (0)

int sm_count();  // SMs of the current device (cached per device)

// Per-device flags for one-time host set-up (kernel attributes, constant
// tables). Several host threads may make first calls at once: each set-up
// step is idempotent, so running it twice is harmless, and the atomic
// fetch_or never loses another thread's device bit.
class DeviceBits {
 public:
  bool has(int dev) const {
    return dev >= 0 && dev < 64 && ((bits_.load(std::memory_order_acquire) >> dev) & 1u);
  }
  void set(int dev) {
    if (dev >= 0 && dev < 64) bits_.fetch_or(uint64_t{1} << dev, std::memory_order_acq_rel);
  }

 private:
  std::atomic<uint64_t> bits_{0};
};

// ---------------------------------------------------------------------------
// Packed fp16x2 arithmetic with explicit IEEE round-to-nearest-even, so the
// compiler can neither contract nor reassociate the encoder's metric.
// Operands are raw 32-bit registers holding two binary16 lanes.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// The scalar forms (the tracebacks' candidate re-evaluation).
__device__ __forceinline__ uint16_t h_sub(uint16_t a, uint16_t b) {
  uint16_t r;
  asm("sub.rn.f16 %0, %1, %2;" : "=h"(r) : "h"(a), "h"(b));
  return r;
}
__device__ __forceinline__ uint16_t h_fma(uint16_t a, uint16_t b, uint16_t c) {
  uint16_t r;
  asm("fma.rn.f16 %0, %1, %2, %3;" : "=h"(r) : "h"(a), "h"(b), "h"(c));
  return r;
}
// {v, v} - w with v the low (HI = false) or high lane of `cb`. One asm block,
// so the lane broadcast cannot be hoisted away from the subtraction (keeping
// 128 broadcast copies of a thread's codebook live would exhaust registers).
template <bool HI>
__device__ __forceinline__ uint32_t h2_sub_bcast(uint32_t cb, uint32_t w) {
  uint32_t d;
  if (HI)
    asm("{\n\t.reg .b16 l, h;\n\t.reg .b32 v;\n\tmov.b32 {l, h}, %1;\n\t"
        "mov.b32 v, {h, h};\n\tsub.rn.f16x2 %0, v, %2;\n\t}"
        : "=r"(d) : "r"(cb), "r"(w));
  else
    asm("{\n\t.reg .b16 l, h;\n\t.reg .b32 v;\n\tmov.b32 {l, h}, %1;\n\t"
        "mov.b32 v, {l, l};\n\tsub.rn.f16x2 %0, v, %2;\n\t}"
        : "=r"(d) : "r"(cb), "r"(w));
  return d;
}
// IEEE minNum per lane; only used on NaN-free data.
__device__ __forceinline__ uint32_t h2_min(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// 0xFFFF per lane where a < b (ordered: false when either is NaN).
__device__ __forceinline__ uint32_t h2_lt_mask(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("set.lt.u32.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// Bitwise select: m ? a : b per bit.
__device__ __forceinline__ uint32_t bsel(uint32_t m, uint32_t a, uint32_t b) {
  return (a & m) | (b & ~m);
}
// Replicate the low / high lane into both lanes.
__device__ __forceinline__ uint32_t h2_lo2(uint32_t a) {
  return __byte_perm(a, 0, 0x1010);
}
__device__ __forceinline__ uint32_t h2_hi2(uint32_t a) {
  return __byte_perm(a, 0, 0x3232);
}

constexpr uint32_t kHInf2 = 0x7C007C00u;  // {+inf, +inf}
constexpr uint16_t kHInf = 0x7C00u;

// ---------------------------------------------------------------------------
// Procedural EXL3 codebooks (state -> fp16 bit pattern).
// Restates trellis_format.codebook_lut (exl3_quant/trellis_format.py:41-81):
//   MUL1:  x = s * 0x83DCD12D; h = fp16(1024 + bytesum(x)); fma(h, 0x1EEE, 0xC931)
//   MCG:   x = s * 0xCBAC1FED;       3INST: x = s * 89226354 + 64248484
//          x = (x & 0x8FFF8FFF) ^ 0x3B603B60; lo16 + hi16 (one rounding)
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t cb_mul1_bytesum(uint32_t s) {
  const uint32_t x = s * 0x83DCD12Du;
#ifdef __CUDA_ARCH__
  return __dp4a(x, 0x01010101u, 0u);  // the four bytes summed in one instruction
#else
  return (x & 0xFFu) + ((x >> 8) & 0xFFu) + ((x >> 16) & 0xFFu) + (x >> 24);
#endif
}

__device__ __forceinline__ uint16_t cb_state_bits(int cb, uint32_t s) {
  uint16_t r;
  if (cb == 2) {
    const uint16_t h = (uint16_t)(0x6400u + cb_mul1_bytesum(s));
    const uint16_t inv = 0x1EEEu, bias = 0xC931u;
    asm("fma.rn.f16 %0, %1, %2, %3;" : "=h"(r) : "h"(h), "h"(inv), "h"(bias));
    return r;
  }
  uint32_t x = (cb == 0) ? (s * 89226354u + 64248484u) : (s * 0xCBAC1FEDu);
  x = (x & 0x8FFF8FFFu) ^ 0x3B603B60u;
  const uint16_t lo = (uint16_t)(x & 0xFFFFu), hi = (uint16_t)(x >> 16);
  asm("add.rn.f16 %0, %1, %2;" : "=h"(r) : "h"(lo), "h"(hi));
  return r;
}

__device__ __forceinline__ float half_bits_to_float(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}

}  // namespace exl3
