// C ABI of the fused hyper-connection stream mixing (kernels: stream_mix.cuh; declarations and
// status codes: include/fhx.h).
#include <cstdint>

#include "fhx.h"
#include "stream_mix.cuh"

namespace fhx {
namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_args(const void* h, int64_t h_s0, int64_t h_s1, int64_t h_s2, int32_t h_dtype, int32_t x_dtype,
               int64_t tokens, int32_t n, int64_t d) {
  if (n < 2 || n > FHX_MIX_MAX_N || tokens < 0 || d < 0) return FHX_ERR_SIZE;
  auto ok = [](int32_t t) { return t == FHX_DTYPE_F32 || t == FHX_DTYPE_BF16 || t == FHX_DTYPE_F16; };
  if (!ok(h_dtype) || !ok(x_dtype)) return FHX_ERR_DTYPE;
  if (tokens > 0 && h == nullptr) return FHX_ERR_POINTER;
  if (h_s0 < 0 || h_s1 < 0 || h_s2 < 0) return FHX_ERR_STRIDE;
  return FHX_OK;
}

int64_t mix_blocks(int64_t tokens) {
  const int64_t per_block = kMixThreads / 32;
  const int64_t blocks = (tokens + per_block - 1) / per_block;
  return blocks < 0x7fffffffLL ? blocks : 0x7fffffffLL;
}

template <typename XT>
int launch_forward(const View& h, int h_dtype, const void* x, int64_t x_s0, int64_t x_s1, void* y, int64_t tokens,
                   int n, int64_t d, cudaStream_t stream) {
  constexpr int V = Chunk<XT>::V;
  const int vec = d % V == 0 && x_s0 % V == 0 && x_s1 % V == 0 && aligned16(x) && aligned16(y);
  const Streams<XT> xs{static_cast<const XT*>(x), x_s0, x_s1};
  const unsigned blocks = unsigned(mix_blocks(tokens));
  XT* out = static_cast<XT*>(y);
  switch (n) {
    case 2: stream_mix_kernel<2, XT><<<blocks, kMixThreads, 0, stream>>>(h, h_dtype, xs, out, tokens, d, vec); break;
    case 3: stream_mix_kernel<3, XT><<<blocks, kMixThreads, 0, stream>>>(h, h_dtype, xs, out, tokens, d, vec); break;
    default: stream_mix_kernel<4, XT><<<blocks, kMixThreads, 0, stream>>>(h, h_dtype, xs, out, tokens, d, vec); break;
  }
  note_launches(1);
  return cuda_status(cudaGetLastError());
}

template <typename XT>
int launch_backward(const View& h, int h_dtype, const void* x, int64_t x_s0, int64_t x_s1, const void* dy,
                    int64_t dy_s0, int64_t dy_s1, void* dx, void* dh, float* gsum, int64_t tokens, int n, int64_t d,
                    cudaStream_t stream) {
  constexpr int V = Chunk<XT>::V;
  const int vec = d % V == 0 && x_s0 % V == 0 && x_s1 % V == 0 && dy_s0 % V == 0 && dy_s1 % V == 0 &&
                  aligned16(x) && aligned16(dy) && aligned16(dx);
  const Streams<XT> xs{static_cast<const XT*>(x), x_s0, x_s1};
  const Streams<XT> gs{static_cast<const XT*>(dy), dy_s0, dy_s1};
  const unsigned blocks = unsigned(mix_blocks(tokens));
  const int64_t dh_blocks64 = (tokens + kMixThreads - 1) / kMixThreads;
  if (dh_blocks64 > 0x7fffffffLL) return FHX_ERR_SIZE;
  const unsigned dh_blocks = unsigned(dh_blocks64);
  XT* out = static_cast<XT*>(dx);
  switch (n) {
    case 2:
      stream_mix_backward_kernel<2, XT><<<blocks, kMixThreads, 0, stream>>>(h, h_dtype, xs, gs, out, gsum, tokens, d, vec);
      stream_mix_dh_kernel<2><<<dh_blocks, kMixThreads, 0, stream>>>(h, h_dtype, gsum, dh, tokens);
      break;
    case 3:
      stream_mix_backward_kernel<3, XT><<<blocks, kMixThreads, 0, stream>>>(h, h_dtype, xs, gs, out, gsum, tokens, d, vec);
      stream_mix_dh_kernel<3><<<dh_blocks, kMixThreads, 0, stream>>>(h, h_dtype, gsum, dh, tokens);
      break;
    default:
      stream_mix_backward_kernel<4, XT><<<blocks, kMixThreads, 0, stream>>>(h, h_dtype, xs, gs, out, gsum, tokens, d, vec);
      stream_mix_dh_kernel<4><<<dh_blocks, kMixThreads, 0, stream>>>(h, h_dtype, gsum, dh, tokens);
      break;
  }
  note_launches(2);
  return cuda_status(cudaGetLastError());
}

}  // namespace
}  // namespace fhx

extern "C" {

int32_t fhx_stream_mix(const void* h, int64_t h_s0, int64_t h_s1, int64_t h_s2, int32_t h_negate, int32_t h_dtype,
                       const void* x, int64_t x_s0, int64_t x_s1, int32_t x_dtype, void* y, int64_t tokens, int32_t n,
                       int64_t d, void* stream) {
  using namespace fhx;
  int st = check_args(h, h_s0, h_s1, h_s2, h_dtype, x_dtype, tokens, n, d);
  if (st != FHX_OK) return st;
  if (tokens == 0 || d == 0) return FHX_OK;
  if (x == nullptr || y == nullptr) return FHX_ERR_POINTER;
  if (x_s0 < 0 || x_s1 < 0) return FHX_ERR_STRIDE;
  const View hv{h, h_s0, h_s1, h_s2, h_negate ? -1.f : 1.f};
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (x_dtype == FHX_DTYPE_F32) return launch_forward<float>(hv, h_dtype, x, x_s0, x_s1, y, tokens, n, d, s);
  if (x_dtype == FHX_DTYPE_BF16) return launch_forward<__nv_bfloat16>(hv, h_dtype, x, x_s0, x_s1, y, tokens, n, d, s);
  return launch_forward<__half>(hv, h_dtype, x, x_s0, x_s1, y, tokens, n, d, s);
}

size_t fhx_stream_mix_workspace_bytes(int64_t tokens, int32_t n) {
  if (tokens <= 0 || n < 2 || n > FHX_MIX_MAX_N) return 0;
  return size_t(tokens) * size_t(n) * size_t(n) * sizeof(float);
}

int32_t fhx_stream_mix_backward(const void* h, int64_t h_s0, int64_t h_s1, int64_t h_s2, int32_t h_negate,
                                int32_t h_dtype, const void* x, int64_t x_s0, int64_t x_s1, int32_t x_dtype,
                                const void* dy, int64_t dy_s0, int64_t dy_s1, void* dx, void* dh, int64_t tokens,
                                int32_t n, int64_t d, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace fhx;
  int st = check_args(h, h_s0, h_s1, h_s2, h_dtype, x_dtype, tokens, n, d);
  if (st != FHX_OK) return st;
  if (tokens == 0) return FHX_OK;
  if (dh == nullptr || (d > 0 && (x == nullptr || dy == nullptr || dx == nullptr))) return FHX_ERR_POINTER;
  if (x_s0 < 0 || x_s1 < 0 || dy_s0 < 0 || dy_s1 < 0) return FHX_ERR_STRIDE;
  if (workspace == nullptr || workspace_bytes < fhx_stream_mix_workspace_bytes(tokens, n) ||
      (reinterpret_cast<uintptr_t>(workspace) & 3u) != 0)
    return FHX_ERR_WORKSPACE;
  const View hv{h, h_s0, h_s1, h_s2, h_negate ? -1.f : 1.f};
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* gsum = static_cast<float*>(workspace);
  if (x_dtype == FHX_DTYPE_F32)
    return launch_backward<float>(hv, h_dtype, x, x_s0, x_s1, dy, dy_s0, dy_s1, dx, dh, gsum, tokens, n, d, s);
  if (x_dtype == FHX_DTYPE_BF16)
    return launch_backward<__nv_bfloat16>(hv, h_dtype, x, x_s0, x_s1, dy, dy_s0, dy_s1, dx, dh, gsum, tokens, n, d, s);
  return launch_backward<__half>(hv, h_dtype, x, x_s0, x_s1, dy, dy_s0, dy_s1, dx, dh, gsum, tokens, n, d, s);
}

}  // extern "C"
