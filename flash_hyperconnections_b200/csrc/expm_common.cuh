// Shared device helpers of the batched small-matrix exponential: element load/store in the
// three I/O dtypes, the adaptive (degree, squarings) choice, and per-degree product counts.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "expm_coeffs.h"

namespace fhx {

enum : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

// A read-only strided [batch, n, n] view; `sign` is -1 for a lazily negated tensor.
struct View {
  const void* data;
  int64_t s0, s1, s2;
  float sign;
};

__device__ __forceinline__ float load_elem(const void* p, int dtype, int64_t off) {
  if (dtype == kF32) return __ldg(static_cast<const float*>(p) + off);
  const unsigned short raw = __ldg(static_cast<const unsigned short*>(p) + off);
  if (dtype == kBF16) return __bfloat162float(__ushort_as_bfloat16(raw));
  return __half2float(__ushort_as_half(raw));
}

__device__ __forceinline__ void store_elem(void* p, int dtype, int64_t off, float v) {
  if (dtype == kF32) {
    static_cast<float*>(p)[off] = v;
  } else if (dtype == kBF16) {
    static_cast<__nv_bfloat16*>(p)[off] = __float2bfloat16_rn(v);
  } else {
    static_cast<__half*>(p)[off] = __float2half_rn(v);
  }
}

// Number of matrix products of the degree-m scheme (Bader-Blanes-Casas 2019).
__host__ __device__ __forceinline__ int scheme_products(int m) {
  return m <= 1 ? 0 : m == 2 ? 1 : m == 4 ? 2 : m == 8 ? 3 : m == 12 ? 4 : 5;
}

// Adaptive choice: the smallest degree whose theta bounds nu; beyond theta_18, degree 18
// with s = ceil(log2(nu / theta_18)) squarings.  nu = min(||A||_1, ||A||_inf) is
// transpose-invariant, so exp(A) and the backward on A^T pick the same (m, s).
// The reference fixes m = 18 and takes s from ||A||_1 (csrc/MatrixExpSmall.cuh:141-157).
__host__ __device__ __forceinline__ void choose_degree(double nu, int* m, int* s) {
  *s = 0;
  if (nu <= kTheta1) {
    *m = 1;
  } else if (nu <= kTheta2) {
    *m = 2;
  } else if (nu <= kTheta4) {
    *m = 4;
  } else if (nu <= kTheta8) {
    *m = 8;
  } else if (nu <= kTheta12) {
    *m = 12;
  } else if (nu <= kTheta18) {
    *m = 18;
  } else {
    *m = 18;
    int e = 0;
    const double f = frexp(nu / kTheta18, &e);  // nu/theta = f * 2^e, f in [0.5, 1)
    *s = (f == 0.5) ? e - 1 : e;                  // exact ceil(log2(nu/theta))
  }
}

// x * 2^-s without forming a subnormal multiplier for large s.
__device__ __forceinline__ float scale_pow2(float x, int s) { return ldexpf(x, -s); }

}  // namespace fhx
