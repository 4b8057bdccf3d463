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

// The CUDA error behind the calling thread's last FHX_ERR_CUDA (fhx_last_cuda_error), and the
// status of a CUDA runtime result that remembers a failure there (both in fhx_expm.cu).
extern thread_local cudaError_t g_last_cuda_error;
int cuda_status(cudaError_t err);
// Kernels launched by this library in this process (fhx_launch_count; fhx_expm.cu).
void note_launches(int count);

// A read-only strided [batch, n, n] view; `sign` is -1 for a lazily negated tensor.
struct View {
  const void* data;
  int64_t s0, s1, s2;
  float sign;
};

// Global loads are volatile asm: the compiler may neither re-issue them at their point of
// use nor move them, so a load issued ahead of time stays in flight (prefetch).
__device__ __forceinline__ float ld_f32(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ unsigned short ld_u16(const unsigned short* p) {
  unsigned short v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ld_f32x4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ uint2 ld_u32x2(const unsigned* p) {
  uint2 v;
  asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

__device__ __forceinline__ float load_elem(const void* p, int dtype, int64_t off) {
  if (dtype == kF32) return ld_f32(static_cast<const float*>(p) + off);
  const unsigned short raw = ld_u16(static_cast<const unsigned short*>(p) + off);
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

// Four consecutive output elements at element offset off (16-byte aligned for float32,
// 8-byte aligned for the half types).
__device__ __forceinline__ void store_chunk(void* p, int dtype, int64_t off, float4 v) {
  if (dtype == kF32) {
    *reinterpret_cast<float4*>(static_cast<float*>(p) + off) = v;
  } else if (dtype == kBF16) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
    uint2 w;
    w.x = *reinterpret_cast<const unsigned*>(&lo);
    w.y = *reinterpret_cast<const unsigned*>(&hi);
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p) + off) = w;
  } else {
    const __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
    uint2 w;
    w.x = *reinterpret_cast<const unsigned*>(&lo);
    w.y = *reinterpret_cast<const unsigned*>(&hi);
    *reinterpret_cast<uint2*>(static_cast<__half*>(p) + off) = w;
  }
}

// Index of degree m in (1, 2, 4, 8, 12, 18), and back.
__host__ __device__ __forceinline__ int degree_index(int m) {
  return m == 1 ? 0 : m == 2 ? 1 : m == 4 ? 2 : m == 8 ? 3 : m == 12 ? 4 : 5;
}
__host__ __device__ __forceinline__ int degree_of_index(int i) {
  return i == 0 ? 1 : i == 1 ? 2 : i == 2 ? 4 : i == 3 ? 8 : i == 4 ? 12 : 18;
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

// x * 2^-s (s >= 0) by multiplications with exact, normal powers of two.
__device__ __forceinline__ float scale_pow2(float x, int s) {
  const int s1 = s < 126 ? s : 126;
  float r = x * __int_as_float((127 - s1) << 23);
  int rest = s - s1;
  while (rest > 0) {
    const int k = rest < 126 ? rest : 126;
    r *= __int_as_float((127 - k) << 23);
    rest -= k;
  }
  return r;
}

}  // namespace fhx
