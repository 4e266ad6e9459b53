// PyTorch binding over the libexl3k C ABI.
//
// Mirrors the reference op binding csrc/quantize_xpu/quantize_xpu.cpp:
// same op names, argument order and meaning, TORCH_CHECK validation (surfaced
// in Python as RuntimeError), work enqueued on the current stream of the
// tensors' device. Device tensors are CUDA tensors here.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdint>

#include "../../include/exl3k.h"

namespace {

int64_t check_cuda_tensor(const at::Tensor& t, const char* name,
                          at::ScalarType expected_dtype, int64_t expected_ndim) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.device().index() >= 0, name, " must have a valid CUDA device index");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(t.scalar_type() == expected_dtype, name, " has wrong dtype");
  TORCH_CHECK(t.dim() == expected_ndim, name, " must be ", expected_ndim, "-D, got ",
              t.dim(), "-D");
  return t.device().index();
}

int64_t resolve_cb(bool mcg, bool mul1) {
  TORCH_CHECK(!(mcg && mul1), "mcg and mul1 cannot both be true (ambiguous codebook)");
  if (mul1) return 2;
  if (mcg) return 1;
  return 0;
}

void validate_common_params(int64_t K, int64_t cb, int64_t L, int64_t sg_size) {
  TORCH_CHECK(K >= 1 && K <= 8, "K must be in 1..8, got ", K);
  TORCH_CHECK(L == 256 || L == 160, "tile length L must be 256 or 160, got ", L);
  TORCH_CHECK(L != 160 || cb == 2, "tile length L=160 is only supported with mul1 (cb=2)");
  // The reference selects an Intel sub-group width; it has no meaning on
  // B200 but the same values are accepted (and others rejected).
  TORCH_CHECK(sg_size == 16 || sg_size == 32, "sg_size must be 16 or 32, got ", sg_size);
}

exl3_stream_t stream_of(int64_t dev) {
  return reinterpret_cast<exl3_stream_t>(
      at::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(dev)).stream());
}

void check_status(int rc, const char* what) {
  TORCH_CHECK(rc == 0, what, " failed (status ", rc, "): ", exl3_last_error());
}

}  // namespace

void register_linalg_ops(pybind11::module& m);  // torch_ext_linalg.cpp

void decode_codebook(int64_t cb, at::Tensor out_lut) {
  TORCH_CHECK(cb >= 0 && cb <= 2, "cb must be 0, 1, or 2");
  const int64_t dev = check_cuda_tensor(out_lut, "out_lut", at::kHalf, 1);
  TORCH_CHECK(out_lut.size(0) == 65536, "out_lut must have length 65536");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(dev));
  check_status(exl3_decode_codebook(static_cast<int>(cb),
                                    reinterpret_cast<uint16_t*>(out_lut.data_ptr()),
                                    stream_of(dev)),
               "decode_codebook");
}

// probe_hfma (probe_xpu.cpp:47-62): out = fma(dh, dh, cost) in fp16, mode 0 =
// the ACS kernels' packed instruction, mode 1 = the tracebacks' scalar one.
void probe_hfma(at::Tensor dh, at::Tensor cost, at::Tensor out, int64_t mode) {
  const int64_t dev = check_cuda_tensor(dh, "dh", at::kHalf, dh.dim());
  TORCH_CHECK(check_cuda_tensor(cost, "cost", at::kHalf, cost.dim()) == dev,
              "dh and cost must share a device");
  TORCH_CHECK(check_cuda_tensor(out, "out", at::kHalf, out.dim()) == dev,
              "dh and out must share a device");
  TORCH_CHECK(dh.numel() == cost.numel() && dh.numel() == out.numel(),
              "probe_hfma tensors must have equal numel");
  TORCH_CHECK(mode == 0 || mode == 1,
              "mode must be 0 (packed fma.rn.f16x2) or 1 (scalar fma.rn.f16)");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(dev));
  check_status(exl3_probe_hfma(reinterpret_cast<const uint16_t*>(dh.data_ptr()),
                               reinterpret_cast<const uint16_t*>(cost.data_ptr()),
                               reinterpret_cast<uint16_t*>(out.data_ptr()), dh.numel(),
                               static_cast<int>(mode), stream_of(dev)),
               "probe_hfma");
}

int64_t quantize_tiles_ws_bytes(int64_t n, int64_t K, int64_t L) {
  return static_cast<int64_t>(
      exl3_quantize_tiles_ws_bytes(n, static_cast<int>(K), static_cast<int>(L)));
}

// Native entry: caller-provided byte workspace, optional packed/cost outputs.
void encode_tiles(at::Tensor input_tiles, at::Tensor output_tiles, at::Tensor output_indices,
                  c10::optional<at::Tensor> output_packed, c10::optional<at::Tensor> output_cost,
                  at::Tensor workspace, int64_t K, int64_t cb) {
  const int64_t dev = check_cuda_tensor(input_tiles, "input_tiles", at::kFloat, 2);
  TORCH_CHECK(check_cuda_tensor(output_tiles, "output_tiles", at::kFloat, 2) == dev,
              "output_tiles must be on the same CUDA device as input_tiles");
  TORCH_CHECK(check_cuda_tensor(output_indices, "output_indices", at::kShort, 2) == dev,
              "output_indices must be on the same CUDA device as input_tiles");
  TORCH_CHECK(check_cuda_tensor(workspace, "workspace", at::kByte, 1) == dev,
              "workspace must be on the same CUDA device as input_tiles");
  const int64_t n = input_tiles.size(0), L = input_tiles.size(1);
  TORCH_CHECK(n > 0, "num_tiles must be positive, got ", n);
  validate_common_params(K, cb, L, 32);
  TORCH_CHECK(output_tiles.sizes() == input_tiles.sizes(), "output_tiles shape must match input_tiles");
  TORCH_CHECK(output_indices.sizes() == input_tiles.sizes(), "output_indices shape must match input_tiles");
  int16_t* packed = nullptr;
  if (output_packed.has_value() && output_packed->defined()) {
    TORCH_CHECK(check_cuda_tensor(*output_packed, "output_packed", at::kShort, 2) == dev,
                "output_packed must be on the same CUDA device");
    TORCH_CHECK(L == 256, "output_packed requires L=256");
    TORCH_CHECK(output_packed->size(0) == n && output_packed->size(1) == 16 * K,
                "output_packed must have shape (num_tiles, 16*K)");
    packed = output_packed->data_ptr<int16_t>();
  }
  float* cost = nullptr;
  if (output_cost.has_value() && output_cost->defined()) {
    TORCH_CHECK(check_cuda_tensor(*output_cost, "output_cost", at::kFloat, 1) == dev,
                "output_cost must be on the same CUDA device");
    TORCH_CHECK(output_cost->size(0) == n, "output_cost must have shape (num_tiles,)");
    cost = output_cost->data_ptr<float>();
  }
  TORCH_CHECK(reinterpret_cast<uintptr_t>(workspace.data_ptr()) % 16 == 0,
              "workspace must be 16-byte aligned");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(dev));
  check_status(exl3_quantize_tiles(input_tiles.data_ptr<float>(), output_tiles.data_ptr<float>(),
                                   output_indices.data_ptr<int16_t>(), packed, cost, n,
                                   static_cast<int>(K), static_cast<int>(cb),
                                   static_cast<int>(L), workspace.data_ptr(),
                                   static_cast<size_t>(workspace.numel()), stream_of(dev)),
               "encode_tiles");
}

// Reference op: quantize_tiles (quantize_xpu.cpp:112-167). temp_edges'
// storage is the encoder workspace (compact K-bit backpointers need at most
// 1/2 of the reference's int16 predecessor table per tile).
void quantize_tiles(at::Tensor input_tiles, at::Tensor output_tiles, at::Tensor output_indices,
                    at::Tensor temp_costs, at::Tensor temp_edges, int64_t K, bool mcg, bool mul1,
                    int64_t sg_size = 32, bool force_global_costs = false,
                    int64_t wave_cap_override = 0) {
  (void)force_global_costs;
  (void)wave_cap_override;
  const int64_t cb = resolve_cb(mcg, mul1);
  const int64_t dev = check_cuda_tensor(input_tiles, "input_tiles", at::kFloat, 2);
  TORCH_CHECK(check_cuda_tensor(output_tiles, "output_tiles", at::kFloat, 2) == dev,
              "output_tiles must be on the same CUDA device as input_tiles");
  TORCH_CHECK(check_cuda_tensor(output_indices, "output_indices", at::kShort, 2) == dev,
              "output_indices must be on the same CUDA device as input_tiles");
  TORCH_CHECK(check_cuda_tensor(temp_costs, "temp_costs", at::kHalf, 3) == dev,
              "temp_costs must be on the same CUDA device as input_tiles");
  TORCH_CHECK(check_cuda_tensor(temp_edges, "temp_edges", at::kShort, 3) == dev,
              "temp_edges must be on the same CUDA device as input_tiles");
  const int64_t num_tiles = input_tiles.size(0);
  const int64_t L = input_tiles.size(1);
  TORCH_CHECK(num_tiles > 0, "num_tiles must be positive, got ", num_tiles);
  validate_common_params(K, cb, L, sg_size);
  const int64_t edges = 65536 >> K;
  const int64_t batch_cap = temp_costs.size(0);
  TORCH_CHECK(batch_cap >= 1, "temp_costs batch dimension B must be >= 1");
  TORCH_CHECK(output_tiles.size(0) == num_tiles && output_tiles.size(1) == L,
              "output_tiles shape must match input_tiles");
  TORCH_CHECK(output_indices.size(0) == num_tiles && output_indices.size(1) == L,
              "output_indices shape must match input_tiles");
  TORCH_CHECK(temp_costs.size(1) == 2 && temp_costs.size(2) == edges,
              "temp_costs must have shape (B, 2, 65536 >> K)");
  TORCH_CHECK(temp_edges.size(0) == batch_cap && temp_edges.size(1) == L &&
                  temp_edges.size(2) == edges,
              "temp_edges must have shape (B, L, 65536 >> K)");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(temp_edges.data_ptr()) % 16 == 0,
              "temp_edges must be 16-byte aligned");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(dev));
  check_status(
      exl3_quantize_tiles(input_tiles.data_ptr<float>(), output_tiles.data_ptr<float>(),
                          output_indices.data_ptr<int16_t>(), nullptr, nullptr, num_tiles,
                          static_cast<int>(K), static_cast<int>(cb), static_cast<int>(L),
                          temp_edges.data_ptr(),
                          static_cast<size_t>(temp_edges.numel()) * sizeof(int16_t),
                          stream_of(dev)),
      "quantize_tiles");
}

// Reference op: quantize_tiles_forward_pass (quantize_xpu.cpp:169-215).
void quantize_tiles_forward_pass(at::Tensor input_tiles, at::Tensor temp_costs,
                                 at::Tensor temp_edges, at::Tensor pre_states, int64_t K,
                                 bool mcg, bool mul1, int64_t roll, int64_t cost_slot = 0,
                                 int64_t sg_size = 32, bool force_global_costs = false) {
  (void)force_global_costs;
  const int64_t cb = resolve_cb(mcg, mul1);
  const int64_t dev = check_cuda_tensor(input_tiles, "input_tiles", at::kFloat, 2);
  TORCH_CHECK(check_cuda_tensor(temp_costs, "temp_costs", at::kHalf, 3) == dev,
              "temp_costs must be on the same CUDA device");
  TORCH_CHECK(check_cuda_tensor(temp_edges, "temp_edges", at::kShort, 3) == dev,
              "temp_edges must be on the same CUDA device");
  TORCH_CHECK(check_cuda_tensor(pre_states, "pre_states", at::kInt, 1) == dev,
              "pre_states must be an int32 CUDA tensor");
  const int64_t num_tiles = input_tiles.size(0);
  const int64_t L = input_tiles.size(1);
  validate_common_params(K, cb, L, sg_size);
  const int64_t edges = 65536 >> K;
  TORCH_CHECK(num_tiles > 0 && num_tiles <= temp_costs.size(0), "num_tiles must be in 1..B");
  TORCH_CHECK(pre_states.size(0) >= num_tiles, "pre_states length must be >= num_tiles");
  TORCH_CHECK(temp_costs.size(1) == 2 && temp_costs.size(2) == edges,
              "temp_costs must have shape (B, 2, 65536 >> K)");
  TORCH_CHECK(temp_edges.size(0) >= num_tiles && temp_edges.size(1) == L &&
                  temp_edges.size(2) == edges,
              "temp_edges must have shape (B, L, 65536 >> K)");
  TORCH_CHECK(cost_slot == 0 || cost_slot == 1, "cost_slot must be 0 or 1");
  TORCH_CHECK(roll >= 0 && roll < L, "roll must be in [0, L)");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(dev));
  check_status(exl3_forward_pass_ref_layout(
                   input_tiles.data_ptr<float>(),
                   reinterpret_cast<uint16_t*>(temp_costs.data_ptr()),
                   temp_edges.data_ptr<int16_t>(), pre_states.data_ptr<int32_t>(), num_tiles,
                   static_cast<int>(K), static_cast<int>(cb), static_cast<int>(L),
                   static_cast<int>(roll), static_cast<int>(cost_slot), stream_of(dev)),
               "quantize_tiles_forward_pass");
}

// Reference op: quantize_tiles_backward_pass (quantize_xpu.cpp:217-259).
void quantize_tiles_backward_pass(at::Tensor temp_costs, at::Tensor temp_edges,
                                  at::Tensor output_tiles, at::Tensor output_indices,
                                  at::Tensor end_states, int64_t num_tiles, int64_t K, bool mcg,
                                  bool mul1, int64_t roll, int64_t cost_slot,
                                  bool write_output, int64_t sg_size = 32) {
  const int64_t cb = resolve_cb(mcg, mul1);
  const int64_t dev = check_cuda_tensor(temp_costs, "temp_costs", at::kHalf, 3);
  TORCH_CHECK(check_cuda_tensor(temp_edges, "temp_edges", at::kShort, 3) == dev,
              "temp_edges must be on the same CUDA device");
  TORCH_CHECK(check_cuda_tensor(output_tiles, "output_tiles", at::kFloat, 2) == dev,
              "output_tiles must be on the same CUDA device");
  TORCH_CHECK(check_cuda_tensor(output_indices, "output_indices", at::kShort, 2) == dev,
              "output_indices must be on the same CUDA device");
  TORCH_CHECK(check_cuda_tensor(end_states, "end_states", at::kInt, 1) == dev,
              "end_states must be an int32 CUDA tensor");
  const int64_t L = temp_edges.size(1);
  validate_common_params(K, cb, L, sg_size);
  TORCH_CHECK(num_tiles > 0 && num_tiles <= temp_costs.size(0), "num_tiles must be in 1..B");
  TORCH_CHECK(temp_edges.size(0) >= num_tiles && temp_edges.size(2) == (65536 >> K),
              "temp_edges must have shape (B, L, 65536 >> K)");
  TORCH_CHECK(end_states.size(0) >= num_tiles, "end_states length must be >= num_tiles");
  TORCH_CHECK(output_tiles.size(0) >= num_tiles && output_tiles.size(1) == L,
              "output_tiles must have shape (>=num_tiles, L)");
  TORCH_CHECK(output_indices.size(0) >= num_tiles && output_indices.size(1) == L,
              "output_indices must have shape (>=num_tiles, L)");
  TORCH_CHECK(cost_slot == 0 || cost_slot == 1, "cost_slot must be 0 or 1");
  TORCH_CHECK(roll >= 0 && roll < L, "roll must be in [0, L)");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(dev));
  check_status(exl3_backward_pass_ref_layout(
                   reinterpret_cast<const uint16_t*>(temp_costs.data_ptr()),
                   temp_edges.data_ptr<int16_t>(), output_tiles.data_ptr<float>(),
                   output_indices.data_ptr<int16_t>(), end_states.data_ptr<int32_t>(),
                   num_tiles, static_cast<int>(K), static_cast<int>(cb), static_cast<int>(L),
                   static_cast<int>(roll), static_cast<int>(cost_slot), write_output ? 1 : 0,
                   stream_of(dev)),
               "quantize_tiles_backward_pass");
}

void pack_trellis(at::Tensor states, at::Tensor packed, int64_t K) {
  const int64_t dev = check_cuda_tensor(states, "states", at::kShort, 2);
  TORCH_CHECK(check_cuda_tensor(packed, "packed", at::kShort, 2) == dev,
              "packed must be on the same CUDA device");
  TORCH_CHECK(K >= 1 && K <= 8, "K must be in 1..8, got ", K);
  TORCH_CHECK(states.size(1) == 256, "states must have shape (n, 256)");
  TORCH_CHECK(packed.size(0) == states.size(0) && packed.size(1) == 16 * K,
              "packed must have shape (n, 16*K)");
  const int64_t n = states.size(0);
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(dev));
  check_status(exl3_pack_trellis(states.data_ptr<int16_t>(), packed.data_ptr<int16_t>(), n,
                                 static_cast<int>(K), stream_of(dev)),
               "pack_trellis");
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("decode_codebook", &decode_codebook,
        "Decode all 65536 states of codebook cb into an fp16 CUDA tensor");
  m.def("probe_hfma", &probe_hfma, py::arg("dh"), py::arg("cost"), py::arg("out"), py::arg("mode"),
        "out[i] = fma(dh[i], dh[i], cost[i]) in fp16; mode 0 = packed fma.rn.f16x2 (ACS), "
        "mode 1 = scalar fma.rn.f16 (traceback)");
  m.def("quantize_tiles_ws_bytes", &quantize_tiles_ws_bytes, py::arg("n"), py::arg("K"),
        py::arg("L") = 256, "Workspace bytes for encode_tiles over n tiles");
  m.def("encode_tiles", &encode_tiles, py::arg("input_tiles"), py::arg("output_tiles"),
        py::arg("output_indices"), py::arg("output_packed"), py::arg("output_cost"),
        py::arg("workspace"), py::arg("K"), py::arg("cb"),
        "Fused 2-pass tail-biting Viterbi tile encoder (compact backpointers)");
  m.def("quantize_tiles", &quantize_tiles, py::arg("input_tiles"), py::arg("output_tiles"),
        py::arg("output_indices"), py::arg("temp_costs"), py::arg("temp_edges"), py::arg("K"),
        py::arg("mcg"), py::arg("mul1"), py::arg("sg_size") = 32,
        py::arg("force_global_costs") = false, py::arg("wave_cap_override") = 0,
        "Fused 2-pass circular Viterbi tile quantizer on CUDA");
  m.def("quantize_tiles_forward_pass", &quantize_tiles_forward_pass, py::arg("input_tiles"),
        py::arg("temp_costs"), py::arg("temp_edges"), py::arg("pre_states"), py::arg("K"),
        py::arg("mcg"), py::arg("mul1"), py::arg("roll"), py::arg("cost_slot") = 0,
        py::arg("sg_size") = 32, py::arg("force_global_costs") = false,
        "Single forward ACS pass on CUDA (reference scratch layout)");
  m.def("quantize_tiles_backward_pass", &quantize_tiles_backward_pass, py::arg("temp_costs"),
        py::arg("temp_edges"), py::arg("output_tiles"), py::arg("output_indices"),
        py::arg("end_states"), py::arg("num_tiles"), py::arg("K"), py::arg("mcg"),
        py::arg("mul1"), py::arg("roll"), py::arg("cost_slot"), py::arg("write_output"),
        py::arg("sg_size") = 32, "Single backward traceback pass on CUDA");
  m.def("pack_trellis", &pack_trellis, py::arg("states"), py::arg("packed"), py::arg("K"),
        "Pack 16-bit trellis states into the EXL3 container (SWAP16 storage)");
  register_linalg_ops(m);
}
