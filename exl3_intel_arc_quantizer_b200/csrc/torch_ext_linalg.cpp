// PyTorch binding of the floating-point stages (Hadamard, Hessian).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

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

void register_linalg_ops(pybind11::module& m) {
  m.def("hessian_accumulate_", &hessian_accumulate_, pybind11::arg("H"), pybind11::arg("X"),
        pybind11::arg("err_flag"), "In-place H += X^T X on the tensor cores");
  m.def("had128_right_", &had128_right_, "In-place x @ H128/sqrt(128) on 128-column blocks");
  m.def("had128_left_", &had128_left_, "In-place H128/sqrt(128) @ x on 128-row blocks");
  m.def("hessian_finalize_", &hessian_finalize_, pybind11::arg("H"), pybind11::arg("count"),
        pybind11::arg("damping_lambda"), pybind11::arg("zero_floor"), pybind11::arg("damp_out"),
        "In-place Hessian normalisation, damping and floor");
}
