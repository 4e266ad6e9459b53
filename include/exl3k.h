/*
 * exl3k.h — C ABI of libexl3k, the B200 (sm_100a) kernels behind the EXL3
 * conversion hot path: the 16x16-tile trellis Viterbi encoder, the LDLQ
 * block-feedback helpers and the Hessian calibration accumulation.
 *
 * Conventions (mirroring the reference op binding
 * csrc/quantize_xpu/quantize_xpu.cpp:73-101 of alpha2beta/EXL3_Intel_Arc_quantizer):
 *   - the caller owns every buffer; all pointers are device pointers on the
 *     current CUDA device unless a parameter says "host";
 *   - work is enqueued asynchronously on `stream` (NULL = legacy default
 *     stream); no entry point synchronizes the host;
 *   - every entry point returns 0 on success and a negative status otherwise;
 *     exl3_last_error() returns a thread-local description of the last
 *     failure. No C++ exception crosses this boundary.
 *
 * Codebook selectors follow the reference: 0 = 3INST, 1 = MCG, 2 = MUL1
 * (exl3_quant/trellis_format.py:33).
 */
#ifndef EXL3K_H
#define EXL3K_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* exl3_stream_t; /* == cudaStream_t */

enum {
  EXL3_OK = 0,
  EXL3_EINVAL = -22,   /* bad argument (shape, K, codebook, pointer) */
  EXL3_ENOMEM = -12,   /* workspace too small for even one tile */
  EXL3_ECUDA = -5,     /* a CUDA runtime call failed */
  EXL3_ENOTSUP = -95   /* configuration not supported on this device */
};

/* Description of the last failure on the calling host thread. */
const char* exl3_last_error(void);

/* Library version string. */
const char* exl3_version(void);

/* ------------------------------------------------------------------ */
/* Trellis encoder                                                     */
/* ------------------------------------------------------------------ */

/*
 * Decode all 65536 states of codebook `cb` into fp16 bit patterns.
 * Replaces decode_codebook(cb, out_lut) (quantize_xpu.cpp:105-110,
 * kernel quantize_kernels.sycl:51-73 / 236-243).
 */
int exl3_decode_codebook(int cb, uint16_t* out_lut, exl3_stream_t stream);

/*
 * Bytes of device workspace needed to encode `n` tiles in one chunk.
 * A smaller workspace is accepted by exl3_quantize_tiles, which then
 * processes the tiles in chunks of floor(ws_bytes / per-tile bytes).
 */
size_t exl3_quantize_tiles_ws_bytes(int64_t n, int K, int L);

/*
 * Fused two-pass tail-biting Viterbi encode of `n` tiles of length L
 * (256, or 160 with cb = MUL1), K bits per weight (1..8).
 * Replaces quantize_tiles(...) (quantize_xpu.cpp:112-167) and the fused
 * kernel FusedQuantizeKernel (quantize_kernels.sycl:245-360).
 *
 *   in          (n, L) float32, tile elements in encoder (tensor-core) order;
 *               each value is rounded to fp16 (round-to-nearest-even)
 *   out_w       (n, L) float32 reconstruction = codebook(state)
 *   out_idx     (n, L) int16 bit patterns of the 16-bit trellis states
 *   out_packed  (n, 16*K) int16, EXL3 bitstream words after SWAP16
 *               (trellis_format.pack_trellis + swap16_storage); may be NULL;
 *               only for L = 256
 *   out_cost    (n) float32 fp16 path cost of the emitted path; may be NULL
 *   ws          device workspace of ws_bytes bytes (see _ws_bytes)
 */
int exl3_quantize_tiles(const float* in, float* out_w, int16_t* out_idx,
                        int16_t* out_packed, float* out_cost, int64_t n, int K,
                        int cb, int L, void* ws, size_t ws_bytes,
                        exl3_stream_t stream);

/*
 * Reference-layout split passes, kept for the traceback placements of the
 * reference encoder (gpu_resident_split / d2h_cpu). They exchange the
 * reference's own scratch layout:
 *   temp_costs (B, 2, S) fp16 and temp_edges (B, L, S) int16 predecessor
 *   edges, S = 65536 >> K.
 *
 * Forward ACS pass over n <= B tiles with ring rotation `roll` and wrap
 * constraint pre_states[t] (-1 = none); writes every step's predecessor
 * into temp_edges and the final costs into temp_costs[:, cost_slot].
 * Replaces quantize_tiles_forward_pass (quantize_xpu.cpp:169-215).
 */
int exl3_forward_pass_ref_layout(const float* in, uint16_t* temp_costs,
                                 int16_t* temp_edges, const int32_t* pre_states,
                                 int64_t n, int K, int cb, int L, int roll,
                                 int cost_slot, exl3_stream_t stream);

/*
 * Traceback over the reference scratch layout. write_output = 0: argmin of
 * temp_costs[:, cost_slot] then walk back to ring index 0, writing
 * end_states. write_output = 1: walk back from end_states writing out_w and
 * out_idx. Replaces quantize_tiles_backward_pass (quantize_xpu.cpp:217-259).
 */
int exl3_backward_pass_ref_layout(const uint16_t* temp_costs,
                                  const int16_t* temp_edges, float* out_w,
                                  int16_t* out_idx, int32_t* end_states,
                                  int64_t n, int K, int cb, int L, int roll,
                                  int cost_slot, int write_output,
                                  exl3_stream_t stream);

/*
 * Pack 16-bit states into the EXL3 container on the device:
 * states (n, 256) int16 (16-byte aligned) -> packed (n, 16*K) int16
 * (4-byte aligned) (pack_trellis + SWAP16, trellis_format.py:120-174).
 */
int exl3_pack_trellis(const int16_t* states, int16_t* packed, int64_t n, int K,
                      exl3_stream_t stream);

/*
 * exl3_quantize_tiles without a caller workspace, for callers that cannot
 * allocate device memory (a host whose GPU memory is owned by another
 * runtime's pool, or a plain C/FFI host without a device allocator that
 * must not call cudaMalloc, which synchronizes the device). No counterpart
 * in the reference. Same arguments and outputs as exl3_quantize_tiles minus
 * the workspace; the scratch is a fixed 64 MiB + 4 KiB __device__ array held
 * by every GPU that loads the library, shared by all calls: at most 16 tiles
 * per call at K=2, L=256 (more at larger K), larger calls return EXL3_EINVAL.
 * The first call in a CUDA context resolves the array's address (make it
 * before any stream capture); under CUDA's default lazy module loading that
 * first call is also what commits the array on the device, so a host whose
 * memory pool later claims the rest of HBM makes one call first (or sets
 * CUDA_MODULE_LOADING=EAGER). Calls that overlap on the GPU race on the
 * scratch. Calls no cudaMalloc/cudaFree and no allocating library routine.
 */
int exl3_quantize_tiles_noalloc(const float* in, float* out_w, int16_t* out_idx,
                                int16_t* out_packed, float* out_cost, int64_t n, int K,
                                int cb, int L, exl3_stream_t stream);

/* ------------------------------------------------------------------ */
/* LDLQ block-feedback loop                                            */
/* ------------------------------------------------------------------ */

/* One weight matrix for exl3_ldlq. All pointers are device pointers on the
 * current device, row-major fp32 unless stated. */
typedef struct exl3_ldlq_job {
  const float* W;     /* (k, n) regularized weight (transformed basis) */
  const float* L;     /* (k, k) block-LDL factor (unit diagonal blocks) */
  float* W_q;         /* out (k, n): quantized weight in the same basis */
  int16_t* encoded;   /* out (k/16, n/16, 256): trellis states, encoder order */
  int64_t k, n;       /* k % buf == 0, n % 128 == 0 */
} exl3_ldlq_job;

/*
 * The LDLQ loop (spans of `buf` rows bottom-up, 16-row blocks bottom-up,
 * compensation through L, trailing update after each span) for 1..32
 * independent matrices advanced together: every step encodes the current
 * 16-row block of each matrix active at that step in one encoder launch.
 * The longest matrix runs from the first step to the last; every other one
 * starts at the step exl3_ldlq_schedule picks and then runs its own blocks
 * without a gap (each matrix's results do not depend on the placement).
 * Replaces ldlq (exl3_quant/ldlq.py:163-309) with the B200 encoder as its
 * tile encoder (make_xpu_tile_encoder, ldlq.py:344-387). exl3_ldlq_ws_bytes
 * returns the workspace size (0 on invalid arguments).
 */
size_t exl3_ldlq_ws_bytes(const exl3_ldlq_job* jobs, int njobs, int K, int buf);
int exl3_ldlq(const exl3_ldlq_job* jobs, int njobs, int K, int cb, int buf, void* ws,
              size_t ws_bytes, exl3_stream_t stream);

/*
 * The first step of each job in exl3_ldlq (host array of njobs): jobs go
 * longest first, then widest, to the start that adds the least estimated
 * encoder time, from
 * the current device's SM count and cluster capacity (earliest on ties).
 * Only the shapes (k, n) of the jobs are read; their pointers may be NULL.
 * No counterpart in the reference (its loop handles one matrix).
 */
int exl3_ldlq_schedule(const exl3_ldlq_job* jobs, int njobs, int K, int buf,
                       int64_t* start_steps);

/* ------------------------------------------------------------------ */
/* Storage side: container unpack and weight decode                    */
/* ------------------------------------------------------------------ */

/*
 * Container words -> 16-bit states: trellis (ntiles, 16*K) int16 in SWAP16
 * storage order (4-byte aligned) -> states (ntiles, 256) int16 (16-byte
 * aligned). Replaces unpack_module_trellis
 * (exl3_quant/serialization.py:65-84).
 */
int exl3_unpack_trellis(const int16_t* trellis, int16_t* states, int64_t ntiles, int K,
                        exl3_stream_t stream);

/*
 * Original-basis weight from the stored EXL3 parameters in one pass:
 * trellis (tiles_k, tiles_n, 16*K) int16 (4-byte aligned), su (k) and sv (n)
 * scales as fp16 (scale_dtype 0, the stored .suh/.svh) or fp32 (1) ->
 * out (k, n) fp32 row-major = H_l(w_hat) * su -> H_r -> * sv, with
 * k = 16*tiles_k and n = 16*tiles_n multiples of 128. out_w_hat (nullable)
 * receives the transformed-basis reconstruction w_hat. Replaces
 * decode_weight_from_storage (exl3_quant/serialization.py:227-266).
 */
int exl3_decode_weight(const int16_t* trellis, const void* su, const void* sv, int scale_dtype,
                       float* out, float* out_w_hat, int64_t tiles_k, int64_t tiles_n, int K,
                       int cb, exl3_stream_t stream);

/* ------------------------------------------------------------------ */
/* Floating-point stages                                               */
/* ------------------------------------------------------------------ */

/*
 * In-place blockwise orthonormal Sylvester Hadamard on a row-major fp32
 * (k, n) matrix: right = x @ H128/sqrt(128) on every 128-column block
 * (n % 128 == 0), left = H128/sqrt(128) @ x on every 128-row block
 * (k % 128 == 0). Replace blockwise_preapply_had_r_ / _l_
 * (exl3_quant/hadamard.py:94-119).
 */
int exl3_had128_right(float* x, int64_t k, int64_t n, exl3_stream_t stream);
int exl3_had128_left(float* x, int64_t k, int64_t n, exl3_stream_t stream);

/*
 * H += X^T X on the tensor cores (tcgen05, fp32 accumulation): X is a
 * row-major (T, d) fp16 (dtype 0) or bf16 (dtype 1) matrix, 16-byte aligned,
 * d % 8 == 0; H is a row-major fp32 (d, d) matrix, symmetric on entry (as
 * any sum of earlier calls is). Only tiles reaching the upper triangle are
 * multiplied and added; the lower triangle is then rewritten from the upper
 * one, so H is symmetric on return.
 * err_flag (device int) is set to 1 if a CTA gave up waiting on its own
 * tensor-core completion (it then skips its update). Replaces
 * HessianCollector._accumulate (exl3_quant/calibration.py:337-352).
 */
int exl3_hessian_accumulate(float* H, const void* X, int dtype, int64_t T, int64_t d,
                            int* err_flag, exl3_stream_t stream);

/*
 * Tile shape of exl3_hessian_accumulate in this process: 0 = chosen by d
 * (256 x 256 tiles for wide H, 128 x 256 otherwise; the default), 1 = always
 * 128 x 256, 2 = always 256 x 256. Results are bit-identical across shapes
 * (each element is summed over the same 8192-token segments in the same
 * order); the setting exists for tests and tuning. No reference counterpart.
 */
int exl3_hessian_set_tile(int mode);

/*
 * Hessian finalize in place on an fp32 (d, d) sum of X^T X over `count`
 * tokens: H /= count; diag += max(1e-8, lambda * mean(diag)); diagonal
 * entries with |d| < zero_floor become zero_floor. damp_out (device, may be
 * NULL) receives the damping added; scratch8 is 8 bytes of device scratch.
 * Replaces HessianCollector.finalize (exl3_quant/calibration.py:359-407).
 */
int exl3_hessian_finalize(float* H, int64_t d, int64_t count, float damping_lambda,
                          float zero_floor, float* damp_out, void* scratch8,
                          exl3_stream_t stream);

/*
 * Weight regularization of a (k, n) fp32 weight, k and n multiples of 128,
 * entirely on the device (no host round trip): the skew heuristic on
 * sqrt(h_diag) (h_diag may be NULL: no heuristic; its elements are
 * h_diag[i * h_diag_stride], e.g. stride k + 1 for the diagonal of H), the
 * 32-slice block RMS of every column, the output-scale decision
 * (force_out_scales -1 = automatic, 0 / 1 forced; q_fallback as the
 * reference), sv, W / sv and the right 128-block Hadamard, the row RMS, su,
 * work / su and the left 128-block Hadamard. Outputs: work (k, n), su_out
 * (k), sv_out (n), out_scales (n), in_scales (k) and 16 bytes of `info`
 * {int32 apply_out_scales, int32 zeros, float skew (NaN if not computed),
 * float mean}. Replaces regularize (exl3_quant/regularize.py:83-211) except
 * its global-scale step, which multiplies work and divides su afterwards.
 * exl3_regularize_ws_bytes returns the workspace size (0 on invalid shapes).
 */
size_t exl3_regularize_ws_bytes(int64_t k, int64_t n);
int exl3_regularize(const float* W, const float* su_in, const float* sv_in,
                    const float* h_diag, int64_t h_diag_stride, int force_out_scales,
                    int q_fallback, float* work, float* su_out, float* sv_out,
                    float* out_scales, float* in_scales, void* info, int64_t k, int64_t n,
                    void* ws, size_t ws_bytes, exl3_stream_t stream);

/*
 * Block-LDL fold: from the (n, n) lower Cholesky factor C (n % 16 == 0,
 * 16-byte aligned), L[:, b] = C[:, b] D_b^-1 for every 16-column block b with
 * D_b = C's 16x16 diagonal block, identity diagonal blocks and zeros above
 * them; `inverses` receives the (n/16, 16, 16) D_b^-1. Replaces the
 * fold of block_ldl (exl3_quant/ldlq.py:96-117); the factorization itself
 * stays cuSOLVER's potrf with the reference's retry schedule.
 */
int exl3_block_ldl_fold(const float* chol, float* L, float* inverses, int64_t n,
                        exl3_stream_t stream);

/* ------------------------------------------------------------------ */
/* Diagnostics                                                         */
/* ------------------------------------------------------------------ */

/*
 * Measured packed-fp16 FMA throughput of the current device (fp16 operations
 * per second, one fma.rn.f16x2 = 2). Synchronizes `stream`. The encoder's
 * add-compare-select runs on this pipe, so this is its roofline denominator.
 * No counterpart in the reference (its roofline had no measured peak).
 */
int exl3_probe_fp16x2_rate(double* fp16_ops_per_s, exl3_stream_t stream);

/*
 * fp16 FMA rounding probe: out[i] = dh[i] * dh[i] + cost[i] rounded once to
 * binary16 (round to nearest even), for the encoder's metric. Replaces
 * `probe_hfma(dh, cost, out, mode)` (csrc/probe_xpu/probe_xpu.cpp:47-62,
 * kernel csrc/probe_xpu/probe_kernels.sycl:45-70), whose tests
 * (tests/test_xpu_extension.py:64-80, exl3_quant/xpu_probe.py:153-270) check
 * it against an exact single rounding. mode 0: the packed fma.rn.f16x2 the
 * ACS kernels issue (elements 2j and 2j+1 share one instruction); mode 1: the
 * scalar fma.rn.f16 the tracebacks issue. Arrays hold binary16 bit patterns;
 * n == 0 is a no-op. Asynchronous on `stream`. EXL3_EINVAL for another mode,
 * a negative n or a NULL array with n > 0.
 */
int exl3_probe_hfma(const uint16_t* dh, const uint16_t* cost, uint16_t* out, int64_t n, int mode,
                    exl3_stream_t stream);

/*
 * Cluster split of the encoder's ACS passes (K = 2..6). A call with few
 * tile pairs (an LDLQ step of a column-sharded module: a few dozen tiles)
 * would leave most SMs idle with one pair per CTA; the encoder then spreads
 * each pair's cost vector over a thread-block cluster of 2, 4 or 8 CTAs that
 * exchange it every step through distributed shared memory. Outputs are
 * bit-identical either way. cluster_ctas: 0 = automatic (the largest size
 * whose clusters all fit on the device at once; off when the pairs fill the
 * SMs), 1 = never, 2 / 4 / 8 = always that size (tests, benchmarks).
 * Process-wide setting. No counterpart in the reference (its encoder runs one
 * work-group per tile).
 */
int exl3_encoder_set_cluster(int cluster_ctas);

/*
 * Tile pairs per cluster of the cluster-split ACS: 0 = automatic (one pair
 * per cluster while the clusters fit; at K = 2 then 2 pairs per cluster of 8
 * CTAs, which share one exchange round per step), 1 / 2 = always that many
 * (tests, benchmarks; 2 exists for clusters of 8 CTAs). Outputs are
 * bit-identical for every setting. Process-wide. No counterpart in the
 * reference.
 */
int exl3_encoder_set_cluster_pairs(int pairs_per_cluster);

/*
 * How many clusters of `cluster_ctas` CTAs (2, 4, 8) of the K-bit cluster
 * encoder the current device runs at once (0: that split is not available
 * for K, e.g. K = 1, 7, 8). Tile pairs beyond it take another wave. No
 * counterpart in the reference.
 */
int exl3_encoder_cluster_capacity(int K, int cluster_ctas, int* clusters);

/*
 * Number of encoder CTAs that gave up a bounded inter-CTA wait (2 s) since
 * the library loaded, on the current device; nonzero means the outputs of
 * those calls are not valid. Synchronizes the device. The asynchronous entry
 * points (exl3_quantize_tiles, exl3_ldlq) cannot return this error; a caller
 * reads the count before and after its work, as the Python layer drivers do
 * (they raise EncoderFault when it grew). No counterpart in the reference.
 */
int exl3_encoder_fault_count(unsigned int* count);

/*
 * Test hook for the error path above, process-wide. stop_sends_at_step in
 * [1, 254] makes every CTA of the cluster-split ACS stop sending cost words
 * from that step of each pass on (all CTAs at the same step, so no message is
 * left in flight); their next waits then run out after wait_limit_ns
 * ([1e5, 1e10] ns; <= 0 restores the 2 s default), the CTAs finish without
 * waiting, the outputs are invalid and the fault count grows. (-1, 0)
 * restores normal operation. No counterpart in the reference.
 */
int exl3_encoder_test_cluster_wait(long long wait_limit_ns, int stop_sends_at_step);

/*
 * Launch timing for benchmarks (off by default). After exl3_timing_begin,
 * every encoder kernel launch is bracketed by CUDA events on its own stream;
 * exl3_timing_end synchronizes those events and returns the summed device
 * time of the ACS passes and of the tracebacks, and the launch counts.
 * No counterpart in the reference.
 */
int exl3_timing_begin(void);
int exl3_timing_end(double* acs_ms, double* traceback_ms, int64_t* acs_launches,
                    int64_t* total_launches);

#ifdef __cplusplus
}
#endif

#endif /* EXL3K_H */
