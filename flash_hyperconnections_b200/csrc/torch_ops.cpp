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
//
// The autograd formula of _matrix_exp is registered here, in C++ (the reference registers it from
// Python, flash_hypercons/ops/matrix_exp/__init__.py:61-77): the input is saved and the backward
// is _frechet(input.mT, grad).  With a forward-mode tangent on the input or the incoming gradient
// it is the differentiable float32 block formula exp([[A^T, G], [0, A^T]]) of native operators
// (__init__.py:32-37), as in the reference.  When a graph of the backward is built (grad mode on),
// the reference also takes that native formula; here _frechet itself carries an autograd
// formula, so second derivatives run through the kernels too (2n <= 32 for the second-order
// term).  Kept in C++ because the Python autograd wrapper cost about 60 us per forward +
// backward, which dominated small batches.
#include <Python.h>

#include <ATen/core/Tensor.h>
#include <ATen/cuda/CUDAContext.h>
#include <ATen/ops/cat.h>
#include <ATen/ops/empty.h>
#include <ATen/ops/linalg_matrix_exp.h>
#include <ATen/ops/matmul.h>
#include <ATen/ops/zeros_like.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <torch/csrc/autograd/custom_function.h>
#include <torch/csrc/autograd/forward_grad.h>
#include <torch/csrc/autograd/python_variable.h>
#include <torch/csrc/utils/pybind.h>
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

// Device workspace of the degree grouping (5 <= n <= 16), from the caching allocator; an
// undefined tensor when the size needs none.
at::Tensor workspace_for(const at::Tensor& a) {
  const size_t bytes = fhx_workspace_bytes(a.size(0), static_cast<int32_t>(a.size(-1)));
  if (bytes == 0) return at::Tensor();
  return at::empty({static_cast<int64_t>(bytes)}, a.options().dtype(at::kByte));
}

// Grouping handoff from the forward to the backward of MatrixExpFunction (5 <= n <= 8, where
// the operators group the batch by degree first): the forward's _matrix_exp call leaves its
// workspace -- keys and permutation of the grouping -- here, the autograd context keeps it, and
// the backward's _frechet call on input^T takes it back (fhx_frechet_grouped).  The backward then
// skips the grouping passes and runs every matrix at the (m, s) of the forward.  The
// classification of A and A^T is identical, so the results equal a fresh grouping's bit for bit.
// Thread-local, set and taken inside one MatrixExpFunction::forward / ::backward on the same
// thread, matched on data pointer, batch and n; plain CUDA tensors only.
struct GroupingHandoff {
  bool want = false;           // the next _matrix_exp call leaves its workspace
  at::Tensor ws;               // the workspace left by that call, or the one to reuse
  const void* data = nullptr;  // the matrices it groups
  int64_t batch = 0;
  int64_t n = 0;
};
thread_local GroupingHandoff g_handoff;

struct HandoffReset {
  ~HandoffReset() { g_handoff = GroupingHandoff(); }
};

bool plain_cuda(const at::Tensor& t) {
  return t.defined() && t.is_cuda() && t.layout() == at::kStrided &&
         !t.key_set().has_any(c10::DispatchKeySet({c10::DispatchKey::Python, c10::DispatchKey::PythonTLSSnapshot})) &&
         t.has_storage();
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
  const bool reuse = direction != nullptr && g_handoff.ws.defined() && g_handoff.data == a.const_data_ptr() &&
                     g_handoff.batch == batch && g_handoff.n == n;
  at::Tensor ws;
  if (reuse) {
    ws = std::move(g_handoff.ws);
    g_handoff = GroupingHandoff();
    // allocated on the forward's stream: keep it from reuse until this launch is done
    c10::cuda::CUDACachingAllocator::recordStream(ws.storage().data_ptr(), at::cuda::getCurrentCUDAStream());
  } else {
    ws = workspace_for(a);
  }
  void* ws_ptr = ws.defined() ? ws.mutable_data_ptr() : nullptr;
  const size_t ws_bytes = ws.defined() ? static_cast<size_t>(ws.numel()) : 0;
  int32_t status;
  if (direction == nullptr) {
    status = fhx_matrix_exp_ws(a.const_data_ptr(), a.stride(0), a.stride(1), a.stride(2), a.is_neg() ? 1 : 0,
                               out.mutable_data_ptr(), batch, n, dtype_code(a), ws_ptr, ws_bytes, stream);
    if (status == FHX_OK && g_handoff.want && ws.defined()) {
      g_handoff.want = false;
      g_handoff.ws = ws;
      g_handoff.data = a.const_data_ptr();
      g_handoff.batch = batch;
      g_handoff.n = n;
    }
  } else if (reuse) {
    const at::Tensor& e = *direction;
    status = fhx_frechet_grouped(a.const_data_ptr(), a.stride(0), a.stride(1), a.stride(2), a.is_neg() ? 1 : 0,
                                 e.const_data_ptr(), e.stride(0), e.stride(1), e.stride(2), e.is_neg() ? 1 : 0,
                                 out.mutable_data_ptr(), batch, n, dtype_code(a), ws_ptr, ws_bytes, stream);
  } else {
    const at::Tensor& e = *direction;
    status = fhx_frechet_ws(a.const_data_ptr(), a.stride(0), a.stride(1), a.stride(2), a.is_neg() ? 1 : 0,
                            e.const_data_ptr(), e.stride(0), e.stride(1), e.stride(2), e.is_neg() ? 1 : 0,
                            out.mutable_data_ptr(), batch, n, dtype_code(a), ws_ptr, ws_bytes, stream);
  }
  TORCH_CHECK(status == FHX_OK, "flash_hypercons kernel: ", fhx_status_string(status),
              status == FHX_ERR_CUDA ? std::string(" (") + fhx_last_cuda_error_string() + ")" : std::string());
  return out;
}

// (exp(A), L(A, E)) from one launch, or with `transposed` (exp(A^T)^T, L(A, E)): the forward
// and the backward of Y = exp(X) at A = X^T.
std::tuple<at::Tensor, at::Tensor> run_pair(const at::Tensor& a, const at::Tensor& e, bool transposed) {
  check_input(a);
  TORCH_CHECK(e.sizes() == a.sizes() && e.device() == a.device() && e.scalar_type() == a.scalar_type() &&
                  e.layout() == at::kStrided,
              "matrix exponential direction must match the input");
  const c10::cuda::CUDAGuard guard(a.device());
  const auto opts = a.options().memory_format(at::MemoryFormat::Contiguous);
  at::Tensor y = at::empty(a.sizes(), opts);
  at::Tensor l = at::empty(a.sizes(), opts);
  if (a.numel() == 0) return {y, l};
  void* stream = static_cast<void*>(at::cuda::getCurrentCUDAStream().stream());
  const at::Tensor ws = workspace_for(a);
  const int32_t status = fhx_matrix_exp_frechet(
      a.const_data_ptr(), a.stride(0), a.stride(1), a.stride(2), a.is_neg() ? 1 : 0, e.const_data_ptr(), e.stride(0),
      e.stride(1), e.stride(2), e.is_neg() ? 1 : 0, y.mutable_data_ptr(), transposed ? 1 : 0, l.mutable_data_ptr(),
      a.size(0), static_cast<int32_t>(a.size(-1)), dtype_code(a), ws.defined() ? ws.mutable_data_ptr() : nullptr,
      ws.defined() ? static_cast<size_t>(ws.numel()) : 0, stream);
  TORCH_CHECK(status == FHX_OK, "flash_hypercons kernel: ", fhx_status_string(status),
              status == FHX_ERR_CUDA ? std::string(" (") + fhx_last_cuda_error_string() + ")" : std::string());
  return {y, l};
}

std::tuple<at::Tensor, at::Tensor> matrix_exp_frechet_cuda(const at::Tensor& input, const at::Tensor& direction) {
  return run_pair(input, direction, false);
}

std::tuple<at::Tensor, at::Tensor> matrix_exp_and_grad_cuda(const at::Tensor& input, const at::Tensor& grad) {
  return run_pair(input.mT(), grad, true);
}

at::Tensor matrix_exp_cuda(const at::Tensor& input) { return run(input, nullptr); }

at::Tensor frechet_cuda(const at::Tensor& input, const at::Tensor& direction) { return run(input, &direction); }

// Differentiable L(input, direction): the upper-right block of the native exponential of
// [[A, E], [0, A]] in float32, cast back (reference __init__.py:32-37).
at::Tensor frechet_reference(const at::Tensor& input, const at::Tensor& direction) {
  const int64_t n = input.size(-1);
  const at::Tensor a = input.to(at::kFloat);
  const at::Tensor e = direction.to(at::kFloat);
  const at::Tensor top = at::cat({a, e}, -1);
  const at::Tensor bottom = at::cat({at::zeros_like(a), a}, -1);
  return at::linalg_matrix_exp(at::cat({top, bottom}, -2)).slice(-2, 0, n).slice(-1, n, 2 * n).to(input.scalar_type());
}

// A forward-mode tangent at any live forward-AD level (levels nest, so the live ones are
// 0, 1, ... up to the first released index).
bool has_tangent(const at::Tensor& t) {
  if (!t.defined()) return false;
  for (uint64_t level = 0; level < 64; ++level) {
    if (!torch::autograd::ForwardADLevel::try_get_by_idx(level)) break;
    if (t._fw_grad(level).defined()) return true;
  }
  return false;
}

// A tensor subclass that overrides __torch_function__ (the reference's has_torch_function
// check, flash_hypercons/ops/matrix_exp/__init__.py:66-72).  The reference then computes the
// gradient with the native block formula in Python, so the subclass sees every operator and
// the gradient comes back as the subclass.  Plain tensors (no Python object, or exactly
// torch.Tensor / Parameter) are recognised without the GIL.  Subclasses whose
// __torch_function__ is disabled -- __torch_dispatch__ subclasses, and the tracing tensors of
// torch.compile (FakeTensor, FunctionalTensor) -- do not count, as in the reference: they keep
// _frechet.
bool overrides_torch_function(const at::Tensor& t) {
  if (!t.defined()) return false;
  PyObject* obj = t.unsafeGetTensorImpl()->pyobj_slot()->load_pyobj();
  if (obj == nullptr || THPVariable_CheckTypeExact(Py_TYPE(obj))) return false;
  namespace py = pybind11;
  py::gil_scoped_acquire gil;
  try {
    // kept for the life of the process (never destroyed after the interpreter is gone)
    static const py::object* disabled =
        new py::object(py::module_::import("torch._C").attr("_disabled_torch_function_impl"));
    const py::object impl =
        py::getattr(py::handle(reinterpret_cast<PyObject*>(Py_TYPE(obj))), "__torch_function__", py::none());
    return !impl.is_none() && !impl.is(*disabled);
  } catch (const py::error_already_set&) {
    return false;
  }
}

// The native block formula called through Python (flash_hyperconnections_b200.ops.matrix_exp.
// _frechet_reference), so that __torch_function__ subclasses see its operators.
at::Tensor frechet_reference_python(const at::Tensor& input, const at::Tensor& direction) {
  namespace py = pybind11;
  py::gil_scoped_acquire gil;
  static const py::object* fn = new py::object(
      py::module_::import("flash_hyperconnections_b200.ops.matrix_exp").attr("_frechet_reference"));
  const py::object out = (*fn)(py::reinterpret_steal<py::object>(THPVariable_Wrap(input)),
                               py::reinterpret_steal<py::object>(THPVariable_Wrap(direction)));
  return THPVariable_Unpack(out.ptr());
}

const auto& frechet_op() {
  static const auto op = c10::Dispatcher::singleton()
                             .findSchemaOrThrow("flash_hypercons::_frechet", "")
                             .typed<at::Tensor(const at::Tensor&, const at::Tensor&)>();
  return op;
}

// Second-order Frechet derivative D^2 exp(X)[E1, E2] as the upper-right block of
// L(Z, W), Z = [[X, E1], [0, X]], W = [[E2, 0], [0, E2]] (d/dt of exp(Z + tW), whose upper-right
// block is L(X + tE2, E1)).  The 2n x 2n matrices go through the Frechet kernel while 2n <= 32;
// otherwise, or when a graph is needed, through the differentiable native block formula.
at::Tensor frechet_second(const at::Tensor& x, const at::Tensor& e1, const at::Tensor& e2, bool differentiable) {
  const int64_t n = x.size(-1);
  const at::Tensor zero = at::zeros_like(x);
  const at::Tensor z = at::cat({at::cat({x, e1}, -1), at::cat({zero, x}, -1)}, -2);
  const at::Tensor w = at::cat({at::cat({e2, zero}, -1), at::cat({zero, e2}, -1)}, -2);
  const at::Tensor l = (differentiable || 2 * n > FHX_MAX_N || !x.is_cuda()) ? frechet_reference(z, w)
                                                                               : frechet_op().call(z, w);
  return l.slice(-2, 0, n).slice(-1, n, 2 * n);
}

// Autograd formula of _frechet (used when a graph of the first backward is built): with
// Y = L(X, E) and upstream gradient H, dX = D^2 exp(X^T)[E^T, H] and dE = L(X^T, H) (adjoints
// of the first and second Frechet derivatives of exp).
struct FrechetFunction : public torch::autograd::Function<FrechetFunction> {
  static at::Tensor forward(torch::autograd::AutogradContext* ctx, const at::Tensor& input,
                            const at::Tensor& direction) {
    at::Tensor out;
    {
      at::AutoDispatchBelowADInplaceOrView below;
      out = frechet_op().call(input, direction);
    }
    ctx->save_for_backward({input, direction});
    return out;
  }

  static torch::autograd::variable_list backward(torch::autograd::AutogradContext* ctx,
                                                 torch::autograd::variable_list grads) {
    const auto saved = ctx->get_saved_variables();
    const at::Tensor& input = saved[0];
    const at::Tensor& direction = saved[1];
    const at::Tensor& grad = grads[0];
    const bool differentiable =
        at::GradMode::is_enabled() || has_tangent(input) || has_tangent(direction) || has_tangent(grad);
    at::Tensor d_input, d_direction;
    if (ctx->needs_input_grad(0)) d_input = frechet_second(input.mT(), direction.mT(), grad, differentiable);
    if (ctx->needs_input_grad(1)) {
      d_direction = differentiable ? frechet_reference(input.mT(), grad) : frechet_op().call(input.mT(), grad);
    }
    return {d_input, d_direction};
  }
};

at::Tensor frechet_autograd(const at::Tensor& input, const at::Tensor& direction) {
  return FrechetFunction::apply(input, direction);
}

struct MatrixExpFunction : public torch::autograd::Function<MatrixExpFunction> {
  static at::Tensor forward(torch::autograd::AutogradContext* ctx, const at::Tensor& input) {
    static const auto op = c10::Dispatcher::singleton()
                               .findSchemaOrThrow("flash_hypercons::_matrix_exp", "")
                               .typed<at::Tensor(const at::Tensor&)>();
    at::Tensor out;
    {
      const HandoffReset reset;
      g_handoff = GroupingHandoff();
      g_handoff.want = plain_cuda(input);
      {
        at::AutoDispatchBelowADInplaceOrView below;
        out = op.call(input);
      }
      if (g_handoff.ws.defined() && g_handoff.data == input.const_data_ptr()) ctx->saved_data["grouping"] = g_handoff.ws;
    }
    ctx->save_for_backward({input});
    return out;
  }

  static torch::autograd::variable_list backward(torch::autograd::AutogradContext* ctx,
                                                 torch::autograd::variable_list grads) {
    const at::Tensor input = ctx->get_saved_variables()[0];
    const at::Tensor& grad = grads[0];
    // Tensor subclasses that override __torch_function__ see the native formula's operators
    // in Python; forward-mode tangents need operators with forward derivatives: the native
    // formula.
    if (overrides_torch_function(input) || overrides_torch_function(grad))
      return {frechet_reference_python(input.mT(), grad)};
    if (has_tangent(input) || has_tangent(grad)) return {frechet_reference(input.mT(), grad)};
    // With grad mode on (a graph of this backward is being built) the call goes through the
    // autograd formula of _frechet above; otherwise straight to the kernel.  The forward's
    // grouping (if any) goes with it.
    const HandoffReset reset;
    const auto grouping = ctx->saved_data.find("grouping");
    if (grouping != ctx->saved_data.end() && plain_cuda(input) && plain_cuda(grad)) {
      g_handoff = GroupingHandoff();
      g_handoff.ws = grouping->second.toTensor();
      g_handoff.data = input.const_data_ptr();
      g_handoff.batch = input.size(0);
      g_handoff.n = input.size(-1);
    }
    return {frechet_op().call(input.mT(), grad)};
  }
};

at::Tensor matrix_exp_autograd(const at::Tensor& input) { return MatrixExpFunction::apply(input); }

// ---- hyper-connection stream mixing: Y = exp(H) X per token (fhx_stream_mix) ----

void check_mix(const at::Tensor& h, const at::Tensor& x) {
  auto ok = [](const at::Tensor& t) {
    return t.scalar_type() == at::kFloat || t.scalar_type() == at::kHalf || t.scalar_type() == at::kBFloat16;
  };
  TORCH_CHECK(h.is_cuda() && x.is_cuda() && h.device() == x.device() && h.layout() == at::kStrided &&
                  x.layout() == at::kStrided && h.dim() == 3 && x.dim() == 3 && h.size(1) == h.size(2) &&
                  h.size(1) >= 2 && h.size(1) <= FHX_MIX_MAX_N && x.size(0) == h.size(0) && x.size(1) == h.size(1) &&
                  ok(h) && ok(x),
              "expected CUDA tensors h [T, n, n] (2 <= n <= 4) and streams [T, n, D] on one device, in float32, "
              "float16, or bfloat16");
}

// Streams with a unit column stride and no lazy negation (the kernels' layout); a copy otherwise.
at::Tensor unit_columns(const at::Tensor& x) {
  at::Tensor r = x.is_neg() ? x.resolve_neg() : x;
  return (r.size(2) <= 1 || r.stride(2) == 1) ? r : r.contiguous();
}

at::Tensor mix_streams_cuda(const at::Tensor& h, const at::Tensor& x) {
  check_mix(h, x);
  const c10::cuda::CUDAGuard guard(h.device());
  const at::Tensor xs = unit_columns(x);
  at::Tensor y = at::empty(x.sizes(), x.options().memory_format(at::MemoryFormat::Contiguous));
  if (y.numel() == 0) return y;
  void* stream = static_cast<void*>(at::cuda::getCurrentCUDAStream().stream());
  const int32_t status = fhx_stream_mix(h.const_data_ptr(), h.stride(0), h.stride(1), h.stride(2), h.is_neg() ? 1 : 0,
                                        dtype_code(h), xs.const_data_ptr(), xs.stride(0), xs.stride(1), dtype_code(xs),
                                        y.mutable_data_ptr(), h.size(0), static_cast<int32_t>(h.size(1)), x.size(2),
                                        stream);
  TORCH_CHECK(status == FHX_OK, "flash_hypercons stream mixing: ", fhx_status_string(status),
              status == FHX_ERR_CUDA ? std::string(" (") + fhx_last_cuda_error_string() + ")" : std::string());
  return y;
}

std::tuple<at::Tensor, at::Tensor> mix_streams_backward_cuda(const at::Tensor& h, const at::Tensor& x,
                                                             const at::Tensor& grad) {
  check_mix(h, x);
  TORCH_CHECK(grad.sizes() == x.sizes() && grad.device() == x.device() && grad.scalar_type() == x.scalar_type() &&
                  grad.layout() == at::kStrided,
              "stream mixing gradient must match the streams");
  const c10::cuda::CUDAGuard guard(h.device());
  const at::Tensor xs = unit_columns(x);
  const at::Tensor gs = unit_columns(grad);
  at::Tensor dx = at::empty(x.sizes(), x.options().memory_format(at::MemoryFormat::Contiguous));
  at::Tensor dh = at::empty(h.sizes(), h.options().memory_format(at::MemoryFormat::Contiguous));
  if (dh.numel() == 0) return {dx, dh};
  void* stream = static_cast<void*>(at::cuda::getCurrentCUDAStream().stream());
  const size_t ws_bytes = fhx_stream_mix_workspace_bytes(h.size(0), static_cast<int32_t>(h.size(1)));
  at::Tensor ws = at::empty({static_cast<int64_t>(ws_bytes / sizeof(float))}, h.options().dtype(at::kFloat));
  const int32_t status = fhx_stream_mix_backward(
      h.const_data_ptr(), h.stride(0), h.stride(1), h.stride(2), h.is_neg() ? 1 : 0, dtype_code(h),
      xs.const_data_ptr(), xs.stride(0), xs.stride(1), dtype_code(xs), gs.const_data_ptr(), gs.stride(0), gs.stride(1),
      dx.mutable_data_ptr(), dh.mutable_data_ptr(), h.size(0), static_cast<int32_t>(h.size(1)), x.size(2),
      ws.mutable_data_ptr(), ws_bytes, stream);
  TORCH_CHECK(status == FHX_OK, "flash_hypercons stream mixing backward: ", fhx_status_string(status),
              status == FHX_ERR_CUDA ? std::string(" (") + fhx_last_cuda_error_string() + ")" : std::string());
  return {dx, dh};
}

// Differentiable native formula of the backward (float32 math, cast back): used when a graph
// of the backward is built, for forward-mode tangents and for __torch_function__ subclasses.
std::tuple<at::Tensor, at::Tensor> mix_streams_backward_native(const at::Tensor& h, const at::Tensor& x,
                                                               const at::Tensor& grad) {
  const at::Tensor hf = h.to(at::kFloat), xf = x.to(at::kFloat), gf = grad.to(at::kFloat);
  const at::Tensor e = at::linalg_matrix_exp(hf);
  const at::Tensor dx = at::matmul(e.mT(), gf).to(x.scalar_type());
  const at::Tensor dh = frechet_reference(h.mT(), at::matmul(gf, xf.mT()));
  return {dx, dh};
}

struct MixStreamsFunction : public torch::autograd::Function<MixStreamsFunction> {
  static at::Tensor forward(torch::autograd::AutogradContext* ctx, const at::Tensor& h, const at::Tensor& x) {
    static const auto op = c10::Dispatcher::singleton()
                               .findSchemaOrThrow("flash_hypercons::_mix_streams", "")
                               .typed<at::Tensor(const at::Tensor&, const at::Tensor&)>();
    at::Tensor out;
    {
      at::AutoDispatchBelowADInplaceOrView below;
      out = op.call(h, x);
    }
    ctx->save_for_backward({h, x});
    return out;
  }

  static torch::autograd::variable_list backward(torch::autograd::AutogradContext* ctx,
                                                 torch::autograd::variable_list grads) {
    static const auto op = c10::Dispatcher::singleton()
                               .findSchemaOrThrow("flash_hypercons::_mix_streams_backward", "")
                               .typed<std::tuple<at::Tensor, at::Tensor>(const at::Tensor&, const at::Tensor&,
                                                                         const at::Tensor&)>();
    const auto saved = ctx->get_saved_variables();
    const at::Tensor& h = saved[0];
    const at::Tensor& x = saved[1];
    const at::Tensor& grad = grads[0];
    if (!grad.defined()) return {at::Tensor(), at::Tensor()};
    const bool native = at::GradMode::is_enabled() || has_tangent(h) || has_tangent(x) || has_tangent(grad) ||
                        overrides_torch_function(h) || overrides_torch_function(x) || overrides_torch_function(grad);
    at::Tensor dx, dh;
    std::tie(dx, dh) = native ? mix_streams_backward_native(h, x, grad) : op.call(h, x, grad);
    return {ctx->needs_input_grad(0) ? dh : at::Tensor(), ctx->needs_input_grad(1) ? dx : at::Tensor()};
  }
};

at::Tensor mix_streams_autograd(const at::Tensor& h, const at::Tensor& x) { return MixStreamsFunction::apply(h, x); }

}  // namespace

TORCH_LIBRARY(flash_hypercons, m) {
  m.def("_matrix_exp(Tensor input) -> Tensor");
  m.def("_frechet(Tensor input, Tensor direction) -> Tensor");
  // Extensions of this package (no reference schema): both parts of one Frechet launch.
  // (exp(input), L(input, direction)) -- the primal and tangent of forward-mode AD.
  m.def("_matrix_exp_frechet(Tensor input, Tensor direction) -> (Tensor, Tensor)");
  // (exp(input), L(input^T, grad)) -- the forward and the backward of exp for a known grad.
  m.def("_matrix_exp_and_grad(Tensor input, Tensor grad) -> (Tensor, Tensor)");
  // exp(h) @ streams per token (hyper-connection stream mixing), and its backward
  // (d streams, d h).
  m.def("_mix_streams(Tensor h, Tensor streams) -> Tensor");
  m.def("_mix_streams_backward(Tensor h, Tensor streams, Tensor grad) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(flash_hypercons, CUDA, m) {
  m.impl("_matrix_exp", &matrix_exp_cuda);
  m.impl("_frechet", &frechet_cuda);
  m.impl("_matrix_exp_frechet", &matrix_exp_frechet_cuda);
  m.impl("_matrix_exp_and_grad", &matrix_exp_and_grad_cuda);
  m.impl("_mix_streams", &mix_streams_cuda);
  m.impl("_mix_streams_backward", &mix_streams_backward_cuda);
}

TORCH_LIBRARY_IMPL(flash_hypercons, Autograd, m) {
  m.impl("_matrix_exp", &matrix_exp_autograd);
  m.impl("_frechet", &frechet_autograd);
  m.impl("_mix_streams", &mix_streams_autograd);
}

static PyModuleDef module_def = {PyModuleDef_HEAD_INIT, "_C", "flash_hypercons operator registration", -1,
                                 nullptr};

PyMODINIT_FUNC PyInit__C() { return PyModule_Create(&module_def); }
