// PyTorch binding of the floating-point stages (Hadamard, Hessian).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <vector>

#include "../../include/exl3k.h"

namespace {

exl3_stream_t cur_stream(const at::Tensor& t) {
  return reinterpret_cast<exl3_stream_t>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void check(int rc, const char* what) {
  TORCH_CHECK(rc == 0, what, " failed (status ", rc, "): ", exl3_last_error());
}

void check_f32_cuda_2d(const at::Tensor& x, const char* name) {
  TORCH_CHECK(x.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(x.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(x.scalar_type() == at::kFloat, name, " must be float32");
  TORCH_CHECK(x.dim() == 2, name, " must be 2-D");
}

}  // namespace

void had128_right_(at::Tensor x) {
  check_f32_cuda_2d(x, "x");
  TORCH_CHECK(x.size(1) % 128 == 0, "columns (", x.size(1), ") must be divisible by 128");
  c10::cuda::CUDAGuard g(x.device());
  check(exl3_had128_right(x.data_ptr<float>(), x.size(0), x.size(1), cur_stream(x)), "had128_right");
}

void had128_left_(at::Tensor x) {
  check_f32_cuda_2d(x, "x");
  TORCH_CHECK(x.size(0) % 128 == 0, "rows (", x.size(0), ") must be divisible by 128");
  c10::cuda::CUDAGuard g(x.device());
  check(exl3_had128_left(x.data_ptr<float>(), x.size(0), x.size(1), cur_stream(x)), "had128_left");
}

void hessian_finalize_(at::Tensor H, int64_t count, double damping_lambda, double zero_floor,
                       at::Tensor damp_out) {
  check_f32_cuda_2d(H, "H");
  TORCH_CHECK(H.size(0) == H.size(1), "H must be square");
  TORCH_CHECK(damp_out.is_cuda() && damp_out.scalar_type() == at::kFloat && damp_out.numel() == 1,
              "damp_out must be a 1-element float32 CUDA tensor");
  c10::cuda::CUDAGuard g(H.device());
  auto scratch = at::empty({1}, H.options().dtype(at::kDouble));
  check(exl3_hessian_finalize(H.data_ptr<float>(), H.size(0), count, (float)damping_lambda,
                              (float)zero_floor, damp_out.data_ptr<float>(), scratch.data_ptr(),
                              cur_stream(H)),
        "hessian_finalize");
}

void hessian_accumulate_(at::Tensor H, at::Tensor X, at::Tensor err_flag) {
  check_f32_cuda_2d(H, "H");
  TORCH_CHECK(H.size(0) == H.size(1), "H must be square");
  TORCH_CHECK(X.is_cuda() && X.is_contiguous() && X.dim() == 2, "X must be a contiguous 2-D CUDA tensor");
  TORCH_CHECK(X.device() == H.device(), "X and H must be on the same device");
  TORCH_CHECK(X.size(1) == H.size(0), "X must have H.size(0) columns");
  TORCH_CHECK(X.scalar_type() == at::kHalf || X.scalar_type() == at::kBFloat16,
              "X must be float16 or bfloat16");
  TORCH_CHECK(err_flag.is_cuda() && err_flag.scalar_type() == at::kInt && err_flag.numel() >= 1,
              "err_flag must be an int32 CUDA tensor");
  c10::cuda::CUDAGuard g(H.device());
  check(exl3_hessian_accumulate(H.data_ptr<float>(), X.data_ptr(),
                                X.scalar_type() == at::kBFloat16 ? 1 : 0, X.size(0), X.size(1),
                                err_flag.data_ptr<int>(), cur_stream(H)),
        "hessian_accumulate");
}

void unpack_trellis(at::Tensor trellis, at::Tensor states, int64_t K) {
  TORCH_CHECK(trellis.is_cuda() && trellis.is_contiguous() && trellis.scalar_type() == at::kShort,
              "trellis must be a contiguous int16 CUDA tensor");
  TORCH_CHECK(states.is_cuda() && states.is_contiguous() && states.scalar_type() == at::kShort,
              "states must be a contiguous int16 CUDA tensor");
  TORCH_CHECK(trellis.device() == states.device(), "trellis and states must be on the same device");
  TORCH_CHECK(K >= 1 && K <= 8, "K must be in 1..8");
  TORCH_CHECK(trellis.numel() % (16 * K) == 0, "trellis size must be a multiple of 16*K");
  const int64_t ntiles = trellis.numel() / (16 * K);
  TORCH_CHECK(states.numel() == ntiles * 256, "states must hold 256 entries per tile");
  c10::cuda::CUDAGuard g(trellis.device());
  check(exl3_unpack_trellis(trellis.data_ptr<int16_t>(), states.data_ptr<int16_t>(), ntiles,
                            (int)K, cur_stream(trellis)),
        "unpack_trellis");
}

void decode_weight(at::Tensor trellis, at::Tensor su, at::Tensor sv, at::Tensor out,
                   c10::optional<at::Tensor> out_w_hat, int64_t K, int64_t cb) {
  TORCH_CHECK(trellis.is_cuda() && trellis.is_contiguous() && trellis.scalar_type() == at::kShort &&
                  trellis.dim() == 3,
              "trellis must be a contiguous (tiles_k, tiles_n, 16*K) int16 CUDA tensor");
  TORCH_CHECK(trellis.size(2) == 16 * K, "trellis last dimension ", trellis.size(2),
              " does not match 16 * K = ", 16 * K);
  const int64_t k = trellis.size(0) * 16, n = trellis.size(1) * 16;
  TORCH_CHECK(su.is_cuda() && sv.is_cuda() && su.is_contiguous() && sv.is_contiguous(),
              "su and sv must be contiguous CUDA tensors");
  TORCH_CHECK(su.scalar_type() == sv.scalar_type() &&
                  (su.scalar_type() == at::kHalf || su.scalar_type() == at::kFloat),
              "su and sv must both be float16 or both float32");
  TORCH_CHECK(su.numel() == k && sv.numel() == n, "su must have ", k, " elements and sv ", n);
  check_f32_cuda_2d(out, "out");
  TORCH_CHECK(out.size(0) == k && out.size(1) == n, "out must be (", k, ", ", n, ")");
  float* wh = nullptr;
  if (out_w_hat.has_value()) {
    check_f32_cuda_2d(*out_w_hat, "out_w_hat");
    TORCH_CHECK(out_w_hat->size(0) == k && out_w_hat->size(1) == n, "out_w_hat must be (", k, ", ",
                n, ")");
    wh = out_w_hat->data_ptr<float>();
  }
  for (const at::Tensor* t : {&su, &sv, &out})
    TORCH_CHECK(t->device() == trellis.device(), "all tensors must be on the same device");
  c10::cuda::CUDAGuard g(trellis.device());
  check(exl3_decode_weight(trellis.data_ptr<int16_t>(), su.data_ptr(), sv.data_ptr(),
                           su.scalar_type() == at::kFloat ? 1 : 0, out.data_ptr<float>(), wh,
                           trellis.size(0), trellis.size(1), (int)K, (int)cb, cur_stream(out)),
        "decode_weight");
}

// LDLQ for several matrices in lockstep; the workspace comes from the
// caching allocator of the tensors' device.
void ldlq_(std::vector<at::Tensor> W, std::vector<at::Tensor> L, std::vector<at::Tensor> Wq,
           std::vector<at::Tensor> enc, int64_t K, int64_t cb, int64_t buf) {
  const size_t nj = W.size();
  TORCH_CHECK(nj >= 1 && L.size() == nj && Wq.size() == nj && enc.size() == nj,
              "W, L, W_q and encoded must be lists of the same non-zero length");
  std::vector<exl3_ldlq_job> jobs(nj);
  for (size_t i = 0; i < nj; ++i) {
    check_f32_cuda_2d(W[i], "W");
    check_f32_cuda_2d(L[i], "L");
    check_f32_cuda_2d(Wq[i], "W_q");
    const int64_t k = W[i].size(0), n = W[i].size(1);
    TORCH_CHECK(L[i].size(0) == k && L[i].size(1) == k, "L must be (", k, ", ", k, ")");
    TORCH_CHECK(Wq[i].size(0) == k && Wq[i].size(1) == n, "W_q must be (", k, ", ", n, ")");
    TORCH_CHECK(enc[i].is_cuda() && enc[i].is_contiguous() && enc[i].scalar_type() == at::kShort &&
                    enc[i].numel() == k * n,
                "encoded must be a contiguous int16 CUDA tensor of k*n elements");
    for (const at::Tensor* t : {&L[i], &Wq[i], &enc[i]})
      TORCH_CHECK(t->device() == W[0].device(), "all tensors must be on the same device");
    jobs[i] = {W[i].data_ptr<float>(), L[i].data_ptr<float>(), Wq[i].data_ptr<float>(),
               enc[i].data_ptr<int16_t>(), k, n};
  }
  c10::cuda::CUDAGuard g(W[0].device());
  const size_t bytes = exl3_ldlq_ws_bytes(jobs.data(), (int)nj, (int)K, (int)buf);
  TORCH_CHECK(bytes > 0, "ldlq: invalid arguments: ", exl3_last_error());
  auto ws = at::empty({(int64_t)bytes}, W[0].options().dtype(at::kByte));
  check(exl3_ldlq(jobs.data(), (int)nj, (int)K, (int)cb, (int)buf, ws.data_ptr(), bytes,
                  cur_stream(W[0])),
        "ldlq");
}

// Regularization on the device with no host synchronisation; returns the
// device info words {apply_out_scales, zeros, skew bits, mean bits} (int32).
at::Tensor regularize_device_(at::Tensor W, at::Tensor su_in, at::Tensor sv_in,
                              c10::optional<at::Tensor> h_diag_src, int64_t force_out_scales,
                              bool q_fallback, at::Tensor work, at::Tensor su_out,
                              at::Tensor sv_out, at::Tensor out_scales, at::Tensor in_scales) {
  check_f32_cuda_2d(W, "weight");
  check_f32_cuda_2d(work, "work");
  const int64_t k = W.size(0), n = W.size(1);
  TORCH_CHECK(work.size(0) == k && work.size(1) == n, "work must match the weight's shape");
  for (const auto* t : {&su_in, &sv_in, &su_out, &sv_out, &out_scales, &in_scales}) {
    TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->scalar_type() == at::kFloat,
                "scales must be contiguous float32 CUDA tensors");
    TORCH_CHECK(t->device() == W.device(), "all tensors must be on the weight's device");
  }
  TORCH_CHECK(su_in.numel() == k && su_out.numel() == k && in_scales.numel() == k,
              "su / in_scales must have ", k, " elements");
  TORCH_CHECK(sv_in.numel() == n && sv_out.numel() == n && out_scales.numel() == n,
              "sv / out_scales must have ", n, " elements");
  const float* hd = nullptr;
  int64_t stride = 1;
  at::Tensor hdt;
  if (h_diag_src.has_value() && h_diag_src->defined()) {
    hdt = *h_diag_src;
    TORCH_CHECK(hdt.is_cuda() && hdt.scalar_type() == at::kFloat && hdt.device() == W.device(),
                "H_diag must be a float32 tensor on the weight's device");
    TORCH_CHECK(hdt.dim() == 1 && hdt.size(0) == k, "H_diag must have ", k, " elements");
    stride = hdt.stride(0);
    hd = hdt.data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(W.device());
  const size_t bytes = exl3_regularize_ws_bytes(k, n);
  TORCH_CHECK(bytes > 0, "both dimensions must be divisible by 128, got (", k, ", ", n, ")");
  auto ws = at::empty({(int64_t)bytes}, W.options().dtype(at::kByte));
  auto info = at::empty({4}, W.options().dtype(at::kInt));
  check(exl3_regularize(W.data_ptr<float>(), su_in.data_ptr<float>(), sv_in.data_ptr<float>(), hd,
                        stride, (int)force_out_scales, q_fallback ? 1 : 0, work.data_ptr<float>(),
                        su_out.data_ptr<float>(), sv_out.data_ptr<float>(),
                        out_scales.data_ptr<float>(), in_scales.data_ptr<float>(),
                        info.data_ptr(), k, n, ws.data_ptr(), bytes, cur_stream(W)),
        "regularize");
  return info;
}

// Regularization on the device; returns (apply_out_scales, zeros, skew, mean)
// read back once (the only host synchronisation of the stage).
std::vector<double> regularize_(at::Tensor W, at::Tensor su_in, at::Tensor sv_in,
                                c10::optional<at::Tensor> h_diag_src, int64_t force_out_scales,
                                bool q_fallback, at::Tensor work, at::Tensor su_out,
                                at::Tensor sv_out, at::Tensor out_scales, at::Tensor in_scales) {
  auto host = regularize_device_(W, su_in, sv_in, h_diag_src, force_out_scales, q_fallback, work,
                                 su_out, sv_out, out_scales, in_scales)
                  .cpu();
  const int32_t* iv = host.data_ptr<int32_t>();
  float skew, mean;
  std::memcpy(&skew, iv + 2, 4);
  std::memcpy(&mean, iv + 3, 4);
  return {(double)iv[0], (double)iv[1], (double)skew, (double)mean};
}

void block_ldl_fold(at::Tensor chol, at::Tensor L, c10::optional<at::Tensor> inverses) {
  check_f32_cuda_2d(chol, "chol");
  check_f32_cuda_2d(L, "L");
  const int64_t n = chol.size(0);
  TORCH_CHECK(chol.size(1) == n && L.size(0) == n && L.size(1) == n, "square (n, n) matrices");
  TORCH_CHECK(L.device() == chol.device(), "chol and L must be on the same device");
  at::Tensor inv_t;
  if (inverses.has_value() && inverses->defined()) {
    inv_t = *inverses;
    TORCH_CHECK(inv_t.is_cuda() && inv_t.is_contiguous() && inv_t.scalar_type() == at::kFloat &&
                    inv_t.numel() == n * 16 && inv_t.device() == chol.device(),
                "inverses must be a contiguous float32 (n/16, 16, 16) tensor on chol's device");
  } else {
    inv_t = at::empty({n / 16, 16, 16}, chol.options());
  }
  float* inv = inv_t.data_ptr<float>();
  c10::cuda::CUDAGuard g(chol.device());
  check(exl3_block_ldl_fold(chol.data_ptr<float>(), L.data_ptr<float>(), inv, n, cur_stream(chol)),
        "block_ldl_fold");
}

void register_linalg_ops(pybind11::module& m) {
  m.def("regularize_device_", &regularize_device_, pybind11::arg("W"), pybind11::arg("su_in"),
        pybind11::arg("sv_in"), pybind11::arg("H_diag"), pybind11::arg("force_out_scales"),
        pybind11::arg("q_fallback"), pybind11::arg("work"), pybind11::arg("su_out"),
        pybind11::arg("sv_out"), pybind11::arg("out_scales"), pybind11::arg("in_scales"),
        "regularize_ without the host read-back: returns the int32 info words on the device");
  m.def("regularize_", &regularize_, pybind11::arg("W"), pybind11::arg("su_in"),
        pybind11::arg("sv_in"), pybind11::arg("H_diag"), pybind11::arg("force_out_scales"),
        pybind11::arg("q_fallback"), pybind11::arg("work"), pybind11::arg("su_out"),
        pybind11::arg("sv_out"), pybind11::arg("out_scales"), pybind11::arg("in_scales"),
        "Weight regularization on the device; returns (apply_out_scales, zeros, skew, mean)");
  m.def("block_ldl_fold", &block_ldl_fold, pybind11::arg("chol"), pybind11::arg("L"),
        pybind11::arg("inverses") = pybind11::none(),
        "L = C D^-1 per 16-column block with identity diagonal blocks");
  m.def("ldlq_", &ldlq_, pybind11::arg("W"), pybind11::arg("L"), pybind11::arg("W_q"),
        pybind11::arg("encoded"), pybind11::arg("K"), pybind11::arg("cb"), pybind11::arg("buf"),
        "LDLQ of several matrices in lockstep with the B200 encoder");
  m.def("unpack_trellis", &unpack_trellis, pybind11::arg("trellis"), pybind11::arg("states"),
        pybind11::arg("K"), "Container words -> 16-bit states");
  m.def("decode_weight", &decode_weight, pybind11::arg("trellis"), pybind11::arg("su"),
        pybind11::arg("sv"), pybind11::arg("out"), pybind11::arg("out_w_hat") = pybind11::none(),
        pybind11::arg("K"), pybind11::arg("cb"),
        "Original-basis weight from the EXL3 container and scales in one pass");
  m.def("hessian_accumulate_", &hessian_accumulate_, pybind11::arg("H"), pybind11::arg("X"),
        pybind11::arg("err_flag"), "In-place H += X^T X on the tensor cores");
  m.def("had128_right_", &had128_right_, "In-place x @ H128/sqrt(128) on 128-column blocks");
  m.def("had128_left_", &had128_left_, "In-place H128/sqrt(128) @ x on 128-row blocks");
  m.def("hessian_finalize_", &hessian_finalize_, pybind11::arg("H"), pybind11::arg("count"),
        pybind11::arg("damping_lambda"), pybind11::arg("zero_floor"), pybind11::arg("damp_out"),
        "In-place Hessian normalisation, damping and floor");
}
