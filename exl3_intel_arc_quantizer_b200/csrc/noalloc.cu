// Encoder entry point that allocates no device memory.
//
// For callers that cannot call cudaMalloc: a host embedded in another
// runtime whose allocator already owns all of the GPU's memory (a serving
// engine's pool), or a plain C/FFI host with no device allocator at all and
// that must not call cudaMalloc because it synchronizes the device. They pass
// inputs and outputs; the encoder's backpointer scratch comes from the fixed
// array below instead of a caller workspace.
//
//   * The array is a file-scope __device__ object of kNoAllocScratchBytes
//     (64 MiB + 4 KiB). Every GPU that loads this code holds it until the
//     process exits.
//   * With CUDA's default lazy module loading the array is committed on the
//     device by the first call on that device (its set-up, below, loads this
//     file's module); with CUDA_MODULE_LOADING=EAGER it is committed when the
//     library is loaded. A host whose memory pool claims the rest of HBM makes
//     one call before the pool does.
//   * Host code cannot use the symbol as a device address. The first call in
//     a CUDA context, with that context current, looks the address up with
//     cudaGetSymbolAddress and caches it under the device ordinal and the
//     context's unique id, so a cudaDeviceReset or another context on the
//     same device gets a fresh lookup, never a stale address. Make that first
//     call before any stream capture.
//   * All calls share the array and its contents persist between calls. The
//     encoder writes every scratch byte it later reads, so nothing has to
//     start at zero; calls that overlap on the GPU (different streams, or
//     different host threads) race on the array and must be serialized.
//   * A call needing more scratch than the array holds is rejected with
//     EXL3_EINVAL: at most 16 tiles at K=2 and L=256 (more at larger K).
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = (64u << 20) + (4u << 10);
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

CtxGetIdFn ctx_get_id_fn() {
  static std::once_flag once;
  static CtxGetIdFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetIdFn>(p);
  });
  return fn;
}

struct ScratchSlot {
  unsigned long long ctx_id = 0;  // 0: never resolved
  void* ptr = nullptr;
};

std::mutex g_noalloc_mu;
ScratchSlot g_noalloc_slot[64];

}  // namespace

extern "C" int exl3_quantize_tiles_noalloc(const float* in, float* out_w, int16_t* out_idx,
                                           int16_t* out_packed, float* out_cost, int64_t n,
                                           int K, int cb, int L, exl3_stream_t stream) {
  const size_t need = exl3_quantize_tiles_ws_bytes(n > 0 ? n : 1, K, L);
  EXL3_REQUIRE(need != 0, "K must be in 1..8 and L 256 or 160 (got K=%d, L=%d)", K, L);
  if (n > 0 && need > kNoAllocScratchBytes) {
    const size_t per_pair = exl3_quantize_tiles_ws_bytes(2, K, L);
    const long long max_tiles =
        K >= 2 ? (long long)(kNoAllocScratchBytes / per_pair) * 2
               : (long long)(kNoAllocScratchBytes / exl3_quantize_tiles_ws_bytes(1, K, L));
    exl3::set_error(
        "%lld tiles need %zu bytes of scratch but the no-alloc entry point has %zu; "
        "at most %lld tiles per call at K=%d, L=%d",
        (long long)n, need, kNoAllocScratchBytes, max_tiles, K, L);
    return EXL3_EINVAL;
  }
  int dev = 0;
  EXL3_CUDA(cudaGetDevice(&dev));
  EXL3_REQUIRE(dev >= 0 && dev < 64, "device ordinal %d out of range", dev);
  const CtxGetIdFn get_id = ctx_get_id_fn();
  EXL3_REQUIRE(get_id != nullptr, "the CUDA driver has no cuCtxGetId");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    ScratchSlot& slot = g_noalloc_slot[dev];
    unsigned long long ctx_id = 0;
    if (get_id(nullptr, &ctx_id) != CUDA_SUCCESS || ctx_id == 0 || slot.ctx_id != ctx_id) {
      // set-up for this context: the lookup also makes the device's primary
      // context current when none is yet
      void* p = nullptr;
      EXL3_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
      const CUresult cr = get_id(nullptr, &ctx_id);
      EXL3_REQUIRE(cr == CUDA_SUCCESS && ctx_id != 0, "cuCtxGetId failed (CUresult %d)", (int)cr);
      slot.ptr = p;
      slot.ctx_id = ctx_id;
    }
    scratch = slot.ptr;
  }
  return exl3_quantize_tiles(in, out_w, out_idx, out_packed, out_cost, n, K, cb, L, scratch,
                             kNoAllocScratchBytes, stream);
}
