// Hyper-connection stream mixing fused with the matrix exponential.
//
// A hyper-connection layer keeps n residual streams per token, X[t] of shape [n, D], and mixes
// them with a per-token n x n matrix.  With the mixing matrix parametrised as exp(H[t]), the
// unfused computation is one exp launch writing E = exp(H) to memory and a batched GEMM
// reading it back; for n <= 4 the exponential is a few hundred flops per token while the GEMM
// moves 2 n D elements, so the exp launch and the extra round trip are pure overhead.  Here one
// kernel does both:
//
//   forward   Y[t]  = exp(H[t]) X[t]
//   backward  dX[t] = exp(H[t])^T dY[t]
//             dH[t] = L(H[t]^T, dY[t] X[t]^T)      (the Frechet backward of exp)
//
// One warp per token (grid-stride over tokens).  Every lane evaluates exp(H[t]) -- and in the
// backward the Frechet pair -- in registers with the arithmetic of expm_reg_kernel
// (expm_regs), then the warp streams the D columns in 16-byte chunks: each lane reads the n
// stream rows of its chunk, writes the mixed rows, and in the backward accumulates its part of
// dY X^T, which a butterfly of warp shuffles reduces at the end (every lane ends with the same,
// bit-identical sums; the order is fixed, so results are deterministic).
//
// No reference counterpart: the reference package stops at exp (its name only refers to
// hyper-connections, README.md:1-5).
#pragma once

#include <cstring>
#include <type_traits>

#include "expm_common.cuh"
#include "expm_reg.cuh"

namespace fhx {

constexpr int kMixThreads = 256;
// Forward: three CTAs per SM (at most 85 registers; the exponential's code spills a little)
// and two 16-byte chunks per lane in flight -- measured 3 % faster than one CTA at 125
// registers and one chunk (0.748 against 0.772 ms on [65536, 4, 4096] bf16, 0.88 of HBM).
constexpr int kMixForwardMinBlocks = 3;
constexpr int kMixUnroll = 2;

// 16-byte chunks of a stream row as floats: V elements per chunk.
template <typename XT>
struct Chunk;

template <>
struct Chunk<float> {
  static constexpr int V = 4;
  __device__ static void load(const float* p, float (&v)[V]) {
    const float4 x = ld_f32x4(p);
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  }
  __device__ static void store(float* p, const float (&v)[V]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
  __device__ static float load1(const float* p) { return ld_f32(p); }
  __device__ static void store1(float* p, float v) { *p = v; }
};

__device__ __forceinline__ uint4 ld_u32x4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

template <typename H2, typename HT>
struct HalfChunk {
  static constexpr int V = 8;
  __device__ static float2 to_f2(unsigned w) {
    H2 h;
    memcpy(&h, &w, 4);
    if constexpr (std::is_same<HT, __nv_bfloat16>::value) return __bfloat1622float2(h);
    else return __half22float2(h);
  }
  __device__ static unsigned from_f2(float a, float b) {
    H2 h;
    if constexpr (std::is_same<HT, __nv_bfloat16>::value) h = __floats2bfloat162_rn(a, b);
    else h = __floats2half2_rn(a, b);
    unsigned w;
    memcpy(&w, &h, 4);
    return w;
  }
  __device__ static void load(const HT* p, float (&v)[V]) {
    const uint4 w = ld_u32x4(p);
    const unsigned ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = to_f2(ws[k]);
      v[2 * k] = f.x;
      v[2 * k + 1] = f.y;
    }
  }
  __device__ static void store(HT* p, const float (&v)[V]) {
    uint4 w;
    w.x = from_f2(v[0], v[1]);
    w.y = from_f2(v[2], v[3]);
    w.z = from_f2(v[4], v[5]);
    w.w = from_f2(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = w;
  }
  __device__ static float load1(const HT* p) {
    const unsigned short raw = ld_u16(reinterpret_cast<const unsigned short*>(p));
    if constexpr (std::is_same<HT, __nv_bfloat16>::value) return __bfloat162float(__ushort_as_bfloat16(raw));
    else return __half2float(__ushort_as_half(raw));
  }
  __device__ static void store1(HT* p, float v) {
    if constexpr (std::is_same<HT, __nv_bfloat16>::value) *p = __float2bfloat16_rn(v);
    else *p = __float2half_rn(v);
  }
};

template <>
struct Chunk<__nv_bfloat16> : HalfChunk<__nv_bfloat162, __nv_bfloat16> {};
template <>
struct Chunk<__half> : HalfChunk<__half2, __half> {};

// H[t] of a strided [tokens, n, n] view, in any of the three dtypes, as float registers.
template <int N, bool Pair>
__device__ __forceinline__ RMat<N, Pair> load_mix_matrix(const View& h, int h_dtype, int64_t t) {
  RMat<N, Pair> m;
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) {
      m.d[i * N + j] = h.sign * load_elem(h.data, h_dtype, t * h.s0 + i * h.s1 + j * h.s2);
      if constexpr (Pair) m.u[i * N + j] = 0.f;
    }
  return m;
}

// Stream rows: element (t, j, c) at x[t * s0 + j * s1 + c] (unit column stride).
template <typename XT>
struct Streams {
  const XT* data;
  int64_t s0, s1;
};

// Y[t] = exp(H[t]) X[t]; Y contiguous [tokens, N, D].  vec: every row start is 16-byte
// aligned and D is a multiple of the chunk width, so rows move in 16-byte chunks.
template <int N, typename XT>
__global__ void __launch_bounds__(kMixThreads, kMixForwardMinBlocks) stream_mix_kernel(View h, int h_dtype, Streams<XT> x, XT* __restrict__ y,
                                                                 int64_t tokens, int64_t d, int vec) {
  using C = Chunk<XT>;
  constexpr int V = C::V;
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t t = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; t < tokens; t += stride) {
    const RMat<N, false> e = expm_regs<N, false>(load_mix_matrix<N, false>(h, h_dtype, t));
    const XT* xt = x.data + t * x.s0;
    XT* yt = y + t * N * d;
    if (vec) {
      // U chunks per lane in flight: all loads of a round issue before its FMAs and stores
      constexpr int U = kMixUnroll;
#pragma unroll 1
      for (int64_t c0 = int64_t(lane) * V; c0 < d; c0 += 32 * V * U) {
        float xv[U][N][V];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t c = c0 + int64_t(u) * 32 * V;
          if (u == 0 || c < d) {
#pragma unroll
            for (int j = 0; j < N; ++j) C::load(xt + j * x.s1 + c, xv[u][j]);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t c = c0 + int64_t(u) * 32 * V;
          if (u > 0 && c >= d) break;
#pragma unroll
          for (int i = 0; i < N; ++i) {
            float yv[V];
#pragma unroll
            for (int v = 0; v < V; ++v) {
              float acc = 0.f;
#pragma unroll
              for (int j = 0; j < N; ++j) acc = fmaf(e.d[i * N + j], xv[u][j][v], acc);
              yv[v] = acc;
            }
            C::store(yt + i * d + c, yv);
          }
        }
      }
    } else {
#pragma unroll 1
      for (int64_t c = lane; c < d; c += 32) {
        float xv[N];
#pragma unroll
        for (int j = 0; j < N; ++j) xv[j] = C::load1(xt + j * x.s1 + c);
#pragma unroll
        for (int i = 0; i < N; ++i) {
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < N; ++j) acc = fmaf(e.d[i * N + j], xv[j], acc);
          C::store1(yt + i * d + c, acc);
        }
      }
    }
  }
}

// Backward, streaming part: dX[t] = exp(H[t])^T dY[t] (contiguous [tokens, N, D]) and
// G[t] = dY[t] X[t]^T (float32 [tokens, N, N], the caller's workspace).  vec: as in the forward, for
// X, dY and dX.  The Frechet derivative dH[t] = L(H[t]^T, G[t]) runs in a second, per-token kernel
// (stream_mix_dh_kernel): its register footprint in this kernel held the stream to one CTA
// per SM (measured 1.66 ms, 0.59 of HBM, on [65536, 4, 4096] bf16).
template <int N, typename XT>
__global__ void __launch_bounds__(kMixThreads) stream_mix_backward_kernel(View h, int h_dtype, Streams<XT> x,
                                                                          Streams<XT> dy, XT* __restrict__ dx,
                                                                          float* __restrict__ gsum, int64_t tokens,
                                                                          int64_t d, int vec) {
  using C = Chunk<XT>;
  constexpr int V = C::V;
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t t = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; t < tokens; t += stride) {
    const RMat<N, false> hm = load_mix_matrix<N, false>(h, h_dtype, t);
    const RMat<N, false> e = expm_regs<N, false>(hm);
    float g[N * N];  // this lane's part of dY X^T
#pragma unroll
    for (int k = 0; k < N * N; ++k) g[k] = 0.f;
    const XT* xt = x.data + t * x.s0;
    const XT* gt = dy.data + t * dy.s0;
    XT* dxt = dx + t * N * d;
    if (vec) {
#pragma unroll 1
      for (int64_t c = int64_t(lane) * V; c < d; c += 32 * V) {
        float xv[N][V], gv[N][V];
#pragma unroll
        for (int j = 0; j < N; ++j) {
          C::load(xt + j * x.s1 + c, xv[j]);
          C::load(gt + j * dy.s1 + c, gv[j]);
        }
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
          for (int j = 0; j < N; ++j)
#pragma unroll
            for (int v = 0; v < V; ++v) g[i * N + j] = fmaf(gv[i][v], xv[j][v], g[i * N + j]);
#pragma unroll
        for (int j = 0; j < N; ++j) {
          float r[V];
#pragma unroll
          for (int v = 0; v < V; ++v) {
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < N; ++i) acc = fmaf(e.d[i * N + j], gv[i][v], acc);
            r[v] = acc;
          }
          C::store(dxt + j * d + c, r);
        }
      }
    } else {
#pragma unroll 1
      for (int64_t c = lane; c < d; c += 32) {
        float xv[N], gv[N];
#pragma unroll
        for (int j = 0; j < N; ++j) {
          xv[j] = C::load1(xt + j * x.s1 + c);
          gv[j] = C::load1(gt + j * dy.s1 + c);
        }
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
          for (int j = 0; j < N; ++j) g[i * N + j] = fmaf(gv[i], xv[j], g[i * N + j]);
#pragma unroll
        for (int j = 0; j < N; ++j) {
          float acc = 0.f;
#pragma unroll
          for (int i = 0; i < N; ++i) acc = fmaf(e.d[i * N + j], gv[i], acc);
          C::store1(dxt + j * d + c, acc);
        }
      }
    }
    // Butterfly sums: partners add the same two operands, so every lane ends bit-identical.
#pragma unroll
    for (int k = 0; k < N * N; ++k)
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) g[k] += __shfl_xor_sync(0xffffffffu, g[k], off);
    if (lane < N * N) {
      float v = g[0];
#pragma unroll
      for (int k = 1; k < N * N; ++k)
        if (lane == k) v = g[k];
      gsum[t * (N * N) + lane] = v;
    }
  }
}

// dH[t] = L(H[t]^T, G[t]) in H's dtype, one thread per token, with the arithmetic of the n <= 4
// Frechet kernel (expm_regs).
template <int N>
__global__ void __launch_bounds__(kMixThreads) stream_mix_dh_kernel(View h, int h_dtype, const float* __restrict__ gsum,
                                                                    void* __restrict__ dh, int64_t tokens) {
  const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= tokens) return;
  const RMat<N, false> hm = load_mix_matrix<N, false>(h, h_dtype, t);
  RMat<N, true> p;
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) {
      p.d[i * N + j] = hm.d[j * N + i];
      p.u[i * N + j] = gsum[t * (N * N) + i * N + j];
    }
  const RMat<N, true> r = expm_regs<N, true>(p);
#pragma unroll
  for (int k = 0; k < N * N; ++k) store_elem(dh, h_dtype, t * (N * N) + k, r.u[k]);
}

}  // namespace fhx
