// One matrix per thread, everything in registers: the path for n <= 4.
//
// Each thread loads its n x n matrix (and, for the Frechet derivative, the direction E),
// picks (m, s) from min(||A||_1, ||A||_inf), evaluates the degree-m Taylor scheme on
// A / 2^s and squares s times.  In Frechet mode every quantity is the pair
// (X, dX) of the block-triangular matrix [[X, dX], [0, X]], so a product costs three
// n x n products: (X, dX)(Y, dY) = (XY, X dY + dX Y).
//
// Reference counterpart: the per-row warp kernel tiny::expm_kernel
// (csrc/MatrixExpSmall.cuh:115-173), which spreads one padded 4x4/8x8 matrix over N lanes
// and exchanges rows with one shuffle per FMA; here a thread owns a whole unpadded matrix,
// so products need no data exchange at all.
#pragma once

#include "expm_common.cuh"

namespace fhx {

template <int N, bool Pair>
struct RMat {
  float d[N * N];
  float u[Pair ? N * N : 1];
};

template <int N, bool Pair>
__device__ __forceinline__ RMat<N, Pair> rmul(const RMat<N, Pair>& x, const RMat<N, Pair>& y) {
  RMat<N, Pair> r;
  if constexpr (N % 2 == 0) {
    // pairs of adjacent columns with one paired FMA (FFMA2) each
#pragma unroll
    for (int i = 0; i < N; ++i) {
#pragma unroll
      for (int j = 0; j < N; j += 2) {
        float2 acc = make_float2(0.f, 0.f), accu = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < N; ++k) {
          const float2 xd = make_float2(x.d[i * N + k], x.d[i * N + k]);
          const float2 yd = make_float2(y.d[k * N + j], y.d[k * N + j + 1]);
          acc = __ffma2_rn(xd, yd, acc);
          if constexpr (Pair) {
            accu = __ffma2_rn(xd, make_float2(y.u[k * N + j], y.u[k * N + j + 1]), accu);
            accu = __ffma2_rn(make_float2(x.u[i * N + k], x.u[i * N + k]), yd, accu);
          }
        }
        r.d[i * N + j] = acc.x;
        r.d[i * N + j + 1] = acc.y;
        if constexpr (Pair) {
          r.u[i * N + j] = accu.x;
          r.u[i * N + j + 1] = accu.y;
        }
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float acc = 0.f;
        float accu = 0.f;
#pragma unroll
        for (int k = 0; k < N; ++k) {
          acc = fmaf(x.d[i * N + k], y.d[k * N + j], acc);
          if constexpr (Pair) {
            accu = fmaf(x.d[i * N + k], y.u[k * N + j], accu);
            accu = fmaf(x.u[i * N + k], y.d[k * N + j], accu);
          }
        }
        r.d[i * N + j] = acc;
        if constexpr (Pair) r.u[i * N + j] = accu;
      }
    }
  }
  return r;
}

// r = c0 * I
template <int N, bool Pair>
__device__ __forceinline__ RMat<N, Pair> rident(float c0) {
  RMat<N, Pair> r;
#pragma unroll
  for (int e = 0; e < N * N; ++e) {
    r.d[e] = (e / N == e % N) ? c0 : 0.f;
    if constexpr (Pair) r.u[e] = 0.f;
  }
  return r;
}

// r += c * x, element pairs with one paired FMA (FFMA2: two independent round-to-nearest FMAs,
// the same bits as fmaf on each element).
__device__ __forceinline__ void axpy_plane(float* r, float c, const float* x, int count) {
#pragma unroll
  for (int e = 0; e + 1 < count; e += 2) {
    const float2 v = __ffma2_rn(make_float2(c, c), make_float2(x[e], x[e + 1]), make_float2(r[e], r[e + 1]));
    r[e] = v.x;
    r[e + 1] = v.y;
  }
  if (count & 1) r[count - 1] = fmaf(c, x[count - 1], r[count - 1]);
}
template <int N, bool Pair>
__device__ __forceinline__ void raxpy(RMat<N, Pair>& r, float c, const RMat<N, Pair>& x) {
  axpy_plane(r.d, c, x.d, N * N);
  if constexpr (Pair) axpy_plane(r.u, c, x.u, N * N);
}

// r += x (paired adds, as above)
__device__ __forceinline__ void add_plane(float* r, const float* x, int count) {
#pragma unroll
  for (int e = 0; e + 1 < count; e += 2) {
    const float2 v = __fadd2_rn(make_float2(r[e], r[e + 1]), make_float2(x[e], x[e + 1]));
    r[e] = v.x;
    r[e + 1] = v.y;
  }
  if (count & 1) r[count - 1] += x[count - 1];
}
template <int N, bool Pair>
__device__ __forceinline__ void radd(RMat<N, Pair>& r, const RMat<N, Pair>& x) {
  add_plane(r.d, x.d, N * N);
  if constexpr (Pair) add_plane(r.u, x.u, N * N);
}

// Linear combination c[0] I + c[1] b1 + c[2] b2 + ... over up to four matrices.
template <int N, bool Pair, int K>
__device__ __forceinline__ RMat<N, Pair> rcomb(const float (&c)[K + 1], const RMat<N, Pair>* const (&b)[K]) {
  RMat<N, Pair> r = rident<N, Pair>(c[0]);
#pragma unroll
  for (int t = 0; t < K; ++t) {
    if (c[t + 1] != 0.f) raxpy(r, c[t + 1], *b[t]);
  }
  return r;
}

// The B1..B4 rows of every degree m <= 12 in the four-product structure of T12
// (expm_coeffs.h, t12u), for lanes that index them at run time.
struct T12UTable {
  float v[5][4][4];
};
__host__ __device__ constexpr T12UTable make_t12u_table() {
  T12UTable t{};
  for (int d = 0; d < 5; ++d)
    for (int r = 0; r < 4; ++r)
      for (int c = 0; c < 4; ++c) t.v[d][r][c] = t12u(d, r, c);
  return t;
}
__constant__ T12UTable kT12U = make_t12u_table();

// Degree-m Taylor scheme of Bader-Blanes-Casas (2019) on an already scaled matrix.  Every
// degree m <= 12 runs one code path, the four-product structure of T12 (A2, A3, A6 = B4 B4 + B3,
// T = (B2 + A6) A6 + B1) with its own coefficient rows: lanes of one warp whose matrices picked
// different degrees then run one program instead of one branch per degree (on config 2's
// degree-8/12 mix nearly every warp had both, 3 + 4 products).  Degree 18 has its own path.
template <int N, bool Pair>
__device__ __forceinline__ RMat<N, Pair> taylor(int m, const RMat<N, Pair>& a) {
  using M = RMat<N, Pair>;
  const M a2 = rmul(a, a);
  const M a3 = rmul(a2, a);
  if (m != 18) {
    const float(&t)[4][4] = kT12U.v[degree_index(m)];
    auto comb = [&](int r) {
      M x = rident<N, Pair>(t[r][0]);
      raxpy(x, t[r][1], a);
      raxpy(x, t[r][2], a2);
      raxpy(x, t[r][3], a3);
      return x;
    };
    const M b4 = comb(3);
    M a6 = rmul(b4, b4);
    radd(a6, comb(2));
    M left = comb(1);
    radd(left, a6);
    M r = rmul(left, a6);
    radd(r, comb(0));
    return r;
  }
  const M a6 = rmul(a3, a3);
  const M* basis[4] = {&a, &a2, &a3, &a6};
  const float c1[5] = {t18c(0, 0), t18c(0, 1), t18c(0, 2), t18c(0, 3), t18c(0, 4)};
  const float c2[5] = {t18c(1, 0), t18c(1, 1), t18c(1, 2), t18c(1, 3), t18c(1, 4)};
  const float c3[5] = {t18c(2, 0), t18c(2, 1), t18c(2, 2), t18c(2, 3), t18c(2, 4)};
  const float c4[5] = {t18c(3, 0), t18c(3, 1), t18c(3, 2), t18c(3, 3), t18c(3, 4)};
  const float c5[5] = {t18c(4, 0), t18c(4, 1), t18c(4, 2), t18c(4, 3), t18c(4, 4)};
  M a9 = rmul(rcomb<N, Pair, 4>(c1, basis), rcomb<N, Pair, 4>(c5, basis));
  radd(a9, rcomb<N, Pair, 4>(c4, basis));
  M left = rcomb<N, Pair, 4>(c3, basis);
  radd(left, a9);
  M r = rmul(left, a9);
  radd(r, rcomb<N, Pair, 4>(c2, basis));
  return r;
}

// exp of one n x n matrix held in registers -- with Pair, the pair (A, E) -> (exp(A), L(A, E))
// -- by the arithmetic of expm_reg_kernel below: float64 norms summed in the same order, the
// same (m, s), scaling, scheme and squarings.  Any non-finite entry makes both parts NaN.
// Used by the fused kernels that apply exp to other data (stream_mix.cuh).
template <int N, bool Pair>
__device__ __forceinline__ RMat<N, Pair> expm_regs(RMat<N, Pair> x) {
  bool bad = false;
  double col[N], row[N];
#pragma unroll
  for (int t = 0; t < N; ++t) col[t] = row[t] = 0.0;
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float v = x.d[i * N + j];
      bad |= !isfinite(v);
      const double av = fabs(double(v));
      col[j] += av;
      row[i] += av;
      if constexpr (Pair) bad |= !isfinite(x.u[i * N + j]);
    }
  if (bad) {
    RMat<N, Pair> r;
#pragma unroll
    for (int t = 0; t < N * N; ++t) {
      r.d[t] = __int_as_float(0x7fc00000);
      if constexpr (Pair) r.u[t] = __int_as_float(0x7fc00000);
    }
    return r;
  }
  double n1 = 0.0, ninf = 0.0;
#pragma unroll
  for (int t = 0; t < N; ++t) {
    n1 = fmax(n1, col[t]);
    ninf = fmax(ninf, row[t]);
  }
  int m, s;
  choose_degree(fmin(n1, ninf), &m, &s);
  if (s > 0) {
#pragma unroll
    for (int t = 0; t < N * N; ++t) {
      x.d[t] = scale_pow2(x.d[t], s);
      if constexpr (Pair) x.u[t] = scale_pow2(x.u[t], s);
    }
  }
  RMat<N, Pair> r = taylor<N, Pair>(m, x);
  for (int t = 0; t < s; ++t) r = rmul(r, r);
  return r;
}

// Row i of matrix b of a view as four elements (N == 4, row contiguous and aligned): one
// 128-bit (float32) or 64-bit (half types) load.
__device__ __forceinline__ float4 load_row4(const View& v, int dtype, int64_t off) {
  if (dtype == kF32) {
    const float4 x = ld_f32x4(static_cast<const float*>(v.data) + off);
    return make_float4(v.sign * x.x, v.sign * x.y, v.sign * x.z, v.sign * x.w);
  }
  const uint2 h = ld_u32x2(reinterpret_cast<const unsigned*>(static_cast<const unsigned short*>(v.data) + off));
  auto dec = [&](unsigned w) {
    const unsigned short u = static_cast<unsigned short>(w);
    return v.sign * (dtype == kBF16 ? __bfloat162float(__ushort_as_bfloat16(u)) : __half2float(__ushort_as_half(u)));
  };
  return make_float4(dec(h.x & 0xffffu), dec(h.x >> 16), dec(h.y & 0xffffu), dec(h.y >> 16));
}

// Threads per CTA of the register kernel.  With at least 8 CTAs per SM the compiler caps the
// kernel at 128 registers: the 4 x 4 Frechet kernel (204 registers uncapped, 8 warps per SM)
// then spills only in its degree-18 branch and runs 16 warps per SM.  Measured on B200: config 2
// backward 12.3 -> 10.3 us, a batch of degree-18 matrices unchanged, results bit-identical.
constexpr int kRegThreads = 64;

// flags: bit 0 = rows of A are one vector load each, bit 1 = same for E, bit 2 = output rows
// can be stored as one vector each (N == 4 only), bit 3 = write exp(A) to out2 transposed,
// bit 4 = out2 rows can be stored as one vector each (N == 4 only).
// out2 (Frechet launches only, may be null): exp(A), the value part of the pair.
template <int N, bool Pair>
__global__ void __launch_bounds__(kRegThreads, 8) expm_reg_kernel(View a, View e, void* __restrict__ out,
                                                       void* __restrict__ out2, int64_t batch, int dtype,
                                                       unsigned flags) {
  const int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  RMat<N, Pair> x;
  bool bad = false;
  double col[N], row[N];
#pragma unroll
  for (int t = 0; t < N; ++t) col[t] = row[t] = 0.0;
  const int64_t abase = b * a.s0;
  const int64_t ebase = b * e.s0;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float va[N], ve[N];
    if constexpr (N == 4) {
      if (flags & 1u) {
        const float4 r4 = load_row4(a, dtype, abase + i * a.s1);
        va[0] = r4.x; va[1] = r4.y; va[2] = r4.z; va[3] = r4.w;
      } else {
#pragma unroll
        for (int j = 0; j < N; ++j) va[j] = a.sign * load_elem(a.data, dtype, abase + i * a.s1 + j * a.s2);
      }
      if constexpr (Pair) {
        if (flags & 2u) {
          const float4 r4 = load_row4(e, dtype, ebase + i * e.s1);
          ve[0] = r4.x; ve[1] = r4.y; ve[2] = r4.z; ve[3] = r4.w;
        } else {
#pragma unroll
          for (int j = 0; j < N; ++j) ve[j] = e.sign * load_elem(e.data, dtype, ebase + i * e.s1 + j * e.s2);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        va[j] = a.sign * load_elem(a.data, dtype, abase + i * a.s1 + j * a.s2);
        if constexpr (Pair) ve[j] = e.sign * load_elem(e.data, dtype, ebase + i * e.s1 + j * e.s2);
      }
    }
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float v = va[j];
      x.d[i * N + j] = v;
      bad |= !isfinite(v);
      const double av = fabs(double(v));
      col[j] += av;
      row[i] += av;
      if constexpr (Pair) {
        x.u[i * N + j] = ve[j];
        bad |= !isfinite(ve[j]);
      }
    }
  }
  const int64_t obase = b * (N * N);
  if (bad) {
#pragma unroll
    for (int t = 0; t < N * N; ++t) {
      store_elem(out, dtype, obase + t, __int_as_float(0x7fc00000));
      if (Pair && out2 != nullptr) store_elem(out2, dtype, obase + t, __int_as_float(0x7fc00000));
    }
    return;
  }
  double n1 = 0.0, ninf = 0.0;
#pragma unroll
  for (int t = 0; t < N; ++t) {
    n1 = fmax(n1, col[t]);
    ninf = fmax(ninf, row[t]);
  }
  int m, s;
  choose_degree(fmin(n1, ninf), &m, &s);
  if (s > 0) {
#pragma unroll
    for (int t = 0; t < N * N; ++t) {
      x.d[t] = scale_pow2(x.d[t], s);
      if constexpr (Pair) x.u[t] = scale_pow2(x.u[t], s);
    }
  }
  RMat<N, Pair> r = taylor<N, Pair>(m, x);
  for (int t = 0; t < s; ++t) r = rmul(r, r);
  if constexpr (Pair) {
    if (out2 != nullptr) {
      const bool tr = flags & 8u;
      float v[N * N];
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int j = 0; j < N; ++j) v[i * N + j] = tr ? r.d[j * N + i] : r.d[i * N + j];
      if (N == 4 && (flags & 16u)) {
#pragma unroll
        for (int i = 0; i < N; ++i)
          store_chunk(out2, dtype, obase + 4 * i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
      } else {
#pragma unroll
        for (int t = 0; t < N * N; ++t) store_elem(out2, dtype, obase + t, v[t]);
      }
    }
  }
  const float* res = Pair ? r.u : r.d;
  if constexpr (N == 4) {
    if (flags & 4u) {
#pragma unroll
      for (int i = 0; i < N; ++i) store_chunk(out, dtype, obase + 4 * i, make_float4(res[4 * i], res[4 * i + 1], res[4 * i + 2], res[4 * i + 3]));
      return;
    }
  }
#pragma unroll
  for (int t = 0; t < N * N; ++t) store_elem(out, dtype, obase + t, res[t]);
}

}  // namespace fhx
