// Python binding of the per-call decode entry point, for callers that issue
// one quantized matmul per layer per token: the kernel takes a few
// microseconds, so the host cost of reaching it (argument checks, pointers,
// the caller's current stream) decides whether a decode step is host-bound.
// This module does those checks in C++ on the at::Tensor arguments and calls
// the C-ABI entry point b2_int4_matmul (include/b2.h) of libb2.so; it holds
// no kernels of its own.
//
// int4_matmul(input, weight, scales, group_size, out) mirrors the fast path of
// b200kern.quant.int4_matmul (the reference operator int4_matmul,
// triton_metal/codegen/_msl_templates.py:2682-2745, GPTQ layout, symmetric):
//   * returns None when the arguments are not that case (the Python operator
//     then takes its general path, with its own checks and messages);
//   * returns the output tensor on success;
//   * returns the nonzero b2 status as an int when the launch failed (the
//     Python operator raises the matching B2Error).
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "b2.h"

namespace {

py::object int4_matmul(const at::Tensor& x, const at::Tensor& w, const at::Tensor& s, int64_t group_size,
                       const c10::optional<at::Tensor>& out) {
  const auto st = x.scalar_type();
  int dt;
  if (st == at::kHalf)
    dt = B2_F16;
  else if (st == at::kBFloat16)
    dt = B2_BF16;
  else
    return py::none();
  if (w.scalar_type() != at::kInt || s.scalar_type() != st || !x.is_cuda() || !w.is_cuda() || !s.is_cuda())
    return py::none();
  if (x.dim() != 2 || w.dim() != 2 || s.dim() != 2 || !x.is_contiguous() || !w.is_contiguous() ||
      !s.is_contiguous())
    return py::none();
  const int64_t M = x.size(0), K = x.size(1), N = w.size(1);
  if (group_size <= 0 || w.size(0) * 8 != K || K % group_size || s.size(0) != K / group_size || s.size(1) != N)
    return py::none();
  at::Tensor res;
  bool into_out = false;
  if (out.has_value()) {
    const at::Tensor& o = *out;
    into_out = o.scalar_type() == st && o.is_cuda() && o.is_contiguous() && o.dim() == 2 && o.size(0) == M &&
               o.size(1) == N;
    if (into_out) res = o;
  }
  if (!into_out) res = at::empty({M, N}, x.options());
  if (M) {
    cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
    const int rc = b2_int4_matmul(x.data_ptr(), w.data_ptr(), res.data_ptr(), s.data_ptr(), nullptr, M, N, K,
                                  group_size, dt, (void*)stream);
    if (rc != 0) return py::int_(rc);
  }
  if (out.has_value() && !into_out) {
    // a caller-given output of another layout: filled by a copy, as the
    // Python path does
    out->copy_(res);
    return py::cast(*out);
  }
  return py::cast(res);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "C++ argument handling for the per-layer decode call of b2_int4_matmul";
  m.def("int4_matmul", &int4_matmul, py::arg("input"), py::arg("weight"), py::arg("scales"),
        py::arg("group_size"), py::arg("out") = py::none());
}
