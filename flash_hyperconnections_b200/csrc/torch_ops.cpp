// PyTorch operator registration over the fhx C ABI (include/fhx.h).
//
// Registers the reference's operator namespace and schemas unchanged
// (csrc/register.cpp:10-18):
//   flash_hypercons::_matrix_exp(Tensor input) -> Tensor
//   flash_hypercons::_frechet(Tensor input, Tensor direction) -> Tensor
// The CUDA implementations check their arguments like csrc/matrix_exp.cu:52-59, allocate the
// contiguous output (csrc/matrix_exp.cu:68) under a device guard (:60) and launch on the
// current stream (:16).  Instead of materialising padded FP32 copies (:35-44), they pass the
// input's strides and lazy negation bit straight to the C ABI.
#include <Python.h>

#include <ATen/core/Tensor.h>
#include <ATen/cuda/CUDAContext.h>
#include <ATen/ops/empty.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "fhx.h"

namespace {

int32_t dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return FHX_DTYPE_F32;
    case at::kBFloat16: return FHX_DTYPE_BF16;
    default: return FHX_DTYPE_F16;
  }
}

void check_input(const at::Tensor& a) {
  TORCH_CHECK(a.is_cuda() && a.layout() == at::kStrided && a.dim() == 3 && a.size(-1) == a.size(-2) &&
                  a.size(-1) > 1 && a.size(-1) <= FHX_MAX_N &&
                  (a.scalar_type() == at::kFloat || a.scalar_type() == at::kHalf ||
                   a.scalar_type() == at::kBFloat16),
              "expected a strided CUDA [B, N, N] tensor, 2 <= N <= 32, in float32, float16, or bfloat16");
}

at::Tensor run(const at::Tensor& a, const at::Tensor* direction) {
  check_input(a);
  if (direction != nullptr) {
    TORCH_CHECK(direction->sizes() == a.sizes() && direction->device() == a.device() &&
                    direction->scalar_type() == a.scalar_type() && direction->layout() == at::kStrided,
                "matrix exponential direction must match the input");
  }
  const c10::cuda::CUDAGuard guard(a.device());
  at::Tensor out = at::empty(a.sizes(), a.options().memory_format(at::MemoryFormat::Contiguous));
  if (a.numel() == 0) return out;
  void* stream = static_cast<void*>(at::cuda::getCurrentCUDAStream().stream());
  const int64_t batch = a.size(0);
  const int32_t n = static_cast<int32_t>(a.size(-1));
  int32_t status;
  if (direction == nullptr) {
    status = fhx_matrix_exp(a.const_data_ptr(), a.stride(0), a.stride(1), a.stride(2), a.is_neg() ? 1 : 0,
                            out.mutable_data_ptr(), batch, n, dtype_code(a), stream);
  } else {
    const at::Tensor& e = *direction;
    status = fhx_frechet(a.const_data_ptr(), a.stride(0), a.stride(1), a.stride(2), a.is_neg() ? 1 : 0,
                         e.const_data_ptr(), e.stride(0), e.stride(1), e.stride(2), e.is_neg() ? 1 : 0,
                         out.mutable_data_ptr(), batch, n, dtype_code(a), stream);
  }
  TORCH_CHECK(status == FHX_OK, "flash_hypercons kernel: ", fhx_status_string(status));
  return out;
}

at::Tensor matrix_exp_cuda(const at::Tensor& input) { return run(input, nullptr); }

at::Tensor frechet_cuda(const at::Tensor& input, const at::Tensor& direction) { return run(input, &direction); }

}  // namespace

TORCH_LIBRARY(flash_hypercons, m) {
  m.def("_matrix_exp(Tensor input) -> Tensor");
  m.def("_frechet(Tensor input, Tensor direction) -> Tensor");
}

TORCH_LIBRARY_IMPL(flash_hypercons, CUDA, m) {
  m.impl("_matrix_exp", &matrix_exp_cuda);
  m.impl("_frechet", &frechet_cuda);
}

static PyModuleDef module_def = {PyModuleDef_HEAD_INIT, "_C", "flash_hypercons operator registration", -1,
                                 nullptr};

PyMODINIT_FUNC PyInit__C() { return PyModule_Create(&module_def); }
