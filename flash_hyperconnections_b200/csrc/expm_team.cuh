// Team kernel: padded sizes P = 8, 16, 32 (n = 5..32).
//
// A "team" of T = (P/4) * (P/8) lanes owns one matrix; lane (rb, cb) owns the 4 x 8 register
// tile at rows 4rb.., columns 8cb...  P = 32 is one matrix per warp, P = 16 four, P = 8
// sixteen.  Every polynomial step and every squaring is one product C = X Y (+ Z) of two
// shared-memory planes, computed as a register-tiled outer product: per k a lane reads 4
// values of column k of X and 8 of row k of Y (two 128-bit loads) for 32 FMAs (96 in
// Frechet mode, where (X, dX)(Y, dY) = (XY, X dY + dX Y)).  Planes are row-major with the
// 16-byte chunks of row i rotated by (i / 4), so the column reads of different row blocks
// fall in different banks and the row reads stay 16-byte aligned.
//
// Degree schemes (m = 2..18) are "step programs" over four plane slots s0..s3 and one
// register tile Z: each step is a product followed by a lane-local epilogue that forms
// the next operands as linear combinations of the powers.  All teams of a warp execute
// the product loop in lockstep (one __syncwarp after the product, one after the
// epilogue); a team whose own program is shorter simply idles, so every matrix gets
// exactly its own (m, s) and the result of a matrix never depends on its neighbours.
//
// Work is persistent: grid = resident CTAs, warp w takes warp items w, w + W, ...
//
// Reference counterpart: scalar::tiled_kernel (csrc/MatrixExpSmall.cuh:177-385), one CTA
// per padded 16x16/32x32 matrix with 2-8 elements per thread, operands restaged through
// shared memory with two __syncthreads per product and a fixed degree 18.
#pragma once

#include "expm_common.cuh"

namespace fhx {

template <int P, bool Pair>
struct TeamCfg {
  static constexpr int TM = 4;
  static constexpr int TN = 8;
  static constexpr int RB = P / TM;
  static constexpr int CB = P / TN;
  static constexpr int T = RB * CB;  // lanes per matrix
  static constexpr int TPW = 32 / T;  // matrices per warp
  static constexpr int PLANE = P * P;
  static constexpr int SLOT = (Pair ? 2 : 1) * PLANE;
  static constexpr int NSLOT = 4;
  // Team regions are skewed so that teams of one warp start in different banks.
  static constexpr int SKEW = P == 8 ? 8 : P == 16 ? 16 : 0;
  static constexpr int TEAM_FLOATS = NSLOT * SLOT + SKEW;
  static constexpr int WARP_FLOATS = TPW * TEAM_FLOATS;
  static_assert(TPW * T == 32, "team size must divide the warp");
};

// Offset of element (i, j) inside a plane.
template <int P>
__device__ __forceinline__ int pidx(int i, int j) {
  return i * P + ((((j >> 2) ^ (i >> 2)) & (P / 4 - 1)) << 2) + (j & 3);
}

template <bool Pair>
struct Tile {
  float d[4][8];
  float u[Pair ? 4 : 1][Pair ? 8 : 1];
};

template <bool Pair>
__device__ __forceinline__ void tile_zero(Tile<Pair>& t) {
#pragma unroll
  for (int ii = 0; ii < 4; ++ii)
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      t.d[ii][jj] = 0.f;
      if constexpr (Pair) t.u[ii][jj] = 0.f;
    }
}

// R = X Y (+ Z): X and Y point at the first (value) plane of a slot; the derivative
// plane follows at +PLANE.
template <int P, bool Pair>
__device__ __forceinline__ void team_product(const float* __restrict__ X, const float* __restrict__ Y, int i0,
                                             int j0, Tile<Pair>& R, const Tile<Pair>& Z, bool use_z) {
  constexpr int PLANE = P * P;
  if (use_z) {
    R = Z;
  } else {
    tile_zero(R);
  }
#pragma unroll 4
  for (int k = 0; k < P; ++k) {
    float x[4], xu[4];
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      x[ii] = X[pidx<P>(i0 + ii, k)];
      if constexpr (Pair) xu[ii] = X[PLANE + pidx<P>(i0 + ii, k)];
    }
    float y[8], yu[8];
    {
      const float4 v0 = *reinterpret_cast<const float4*>(Y + pidx<P>(k, j0));
      const float4 v1 = *reinterpret_cast<const float4*>(Y + pidx<P>(k, j0 + 4));
      y[0] = v0.x; y[1] = v0.y; y[2] = v0.z; y[3] = v0.w;
      y[4] = v1.x; y[5] = v1.y; y[6] = v1.z; y[7] = v1.w;
      if constexpr (Pair) {
        const float4 w0 = *reinterpret_cast<const float4*>(Y + PLANE + pidx<P>(k, j0));
        const float4 w1 = *reinterpret_cast<const float4*>(Y + PLANE + pidx<P>(k, j0 + 4));
        yu[0] = w0.x; yu[1] = w0.y; yu[2] = w0.z; yu[3] = w0.w;
        yu[4] = w1.x; yu[5] = w1.y; yu[6] = w1.z; yu[7] = w1.w;
      }
    }
#pragma unroll
    for (int ii = 0; ii < 4; ++ii)
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        R.d[ii][jj] = fmaf(x[ii], y[jj], R.d[ii][jj]);
        if constexpr (Pair) {
          R.u[ii][jj] = fmaf(x[ii], yu[jj], R.u[ii][jj]);
          R.u[ii][jj] = fmaf(xu[ii], y[jj], R.u[ii][jj]);
        }
      }
  }
}

// Operands of step `st` of the degree-m program: product slots and whether Z is added.
__device__ __forceinline__ void step_operands(int m, int st, int* xs, int* ys, bool* use_z) {
  *xs = 0;
  *ys = 0;
  *use_z = false;
  if (m == 4) {
    if (st == 1) { *xs = 2; *ys = 1; *use_z = true; }
  } else if (m == 8) {
    if (st == 1) { *xs = 2; *ys = 1; }
    else if (st == 2) { *xs = 3; *ys = 1; *use_z = true; }
  } else if (m == 12) {
    if (st == 1) { *xs = 1; *ys = 0; }
    else if (st == 2) { *xs = 2; *ys = 2; *use_z = true; }
    else if (st == 3) { *xs = 1; *ys = 2; *use_z = true; }
  } else if (m == 18) {
    if (st == 1) { *xs = 1; *ys = 0; }
    else if (st == 2) { *xs = 2; *ys = 2; }
    else if (st == 3) { *xs = 0; *ys = 1; }
    else if (st == 4) { *xs = 0; *ys = 1; *use_z = true; }
  }
}

// Lane-local epilogue of polynomial step `st`: reads the lane's own elements of the slots
// and of R, writes the lane's own elements of the next operands.  `part` 0 is the value
// plane (identity terms apply), part 1 the derivative plane.
template <int P, bool Pair>
__device__ __forceinline__ void step_epilogue(int m, int st, float* __restrict__ team, int i0, int j0,
                                              Tile<Pair>& R, Tile<Pair>& Z) {
  constexpr int PLANE = P * P;
  constexpr int SLOT = TeamCfg<P, Pair>::SLOT;
  constexpr int NPART = Pair ? 2 : 1;
#pragma unroll
  for (int part = 0; part < NPART; ++part) {
    float* s0 = team + 0 * SLOT + part * PLANE;
    float* s1 = team + 1 * SLOT + part * PLANE;
    float* s2 = team + 2 * SLOT + part * PLANE;
    float* s3 = team + 3 * SLOT + part * PLANE;
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int i = i0 + ii, j = j0 + jj;
        const int o = pidx<P>(i, j);
        const float id = (part == 0 && i == j) ? 1.f : 0.f;
        float& r = (part == 0) ? R.d[ii][jj] : R.u[Pair ? ii : 0][Pair ? jj : 0];
        float& z = (part == 0) ? Z.d[ii][jj] : Z.u[Pair ? ii : 0][Pair ? jj : 0];
        if (m == 2) {
          // T2 = I + A + A2 / 2
          r = id + s0[o] + 0.5f * r;
        } else if (m == 4) {
          if (st == 0) {
            const float a = s0[o], a2 = r;
            s1[o] = 0.5f * id + a * (1.f / 6.f) + a2 * (1.f / 24.f);
            s2[o] = a2;
            z = id + a;
          }
        } else if (m == 8) {
          if (st == 0) {
            const float a = s0[o], a2 = r;
            s1[o] = fmaf(kT8X1, a, kT8X2 * a2);
            s2[o] = a2;
            z = id + a + kT8Y2 * a2;
          } else if (st == 1) {
            const float a = s0[o], a2 = s2[o], a4 = r;
            s3[o] = fmaf(kT8X3, a2, a4);
            s1[o] = kT8X4 * id + kT8X5 * a + kT8X6 * a2 + kT8X7 * a4;
          }
        } else if (m == 12) {
          if (st == 0) {
            s1[o] = r;
          } else if (st == 1) {
            const float a = s0[o], a2 = s1[o], a3 = r;
            s2[o] = t12c(3, 0) * id + t12c(3, 1) * a + t12c(3, 2) * a2 + t12c(3, 3) * a3;
            z = t12c(2, 0) * id + t12c(2, 1) * a + t12c(2, 2) * a2 + t12c(2, 3) * a3;
            s3[o] = t12c(1, 0) * id + t12c(1, 1) * a + t12c(1, 2) * a2 + t12c(1, 3) * a3;
            s0[o] = t12c(0, 0) * id + t12c(0, 1) * a + t12c(0, 2) * a2 + t12c(0, 3) * a3;
          } else if (st == 2) {
            const float a6 = r;
            s1[o] = s3[o] + a6;
            s2[o] = a6;
            z = s0[o];
          }
        } else {  // m == 18
          if (st == 0) {
            s1[o] = r;
          } else if (st == 1) {
            s2[o] = r;
          } else if (st == 2) {
            const float a = s0[o], a2 = s1[o], a3 = s2[o], a6 = r;
            const float b1 = t18c(0, 0) * id + t18c(0, 1) * a + t18c(0, 2) * a2 + t18c(0, 3) * a3 + t18c(0, 4) * a6;
            const float b2 = t18c(1, 0) * id + t18c(1, 1) * a + t18c(1, 2) * a2 + t18c(1, 3) * a3 + t18c(1, 4) * a6;
            const float b3 = t18c(2, 0) * id + t18c(2, 1) * a + t18c(2, 2) * a2 + t18c(2, 3) * a3 + t18c(2, 4) * a6;
            const float b4 = t18c(3, 0) * id + t18c(3, 1) * a + t18c(3, 2) * a2 + t18c(3, 3) * a3 + t18c(3, 4) * a6;
            const float b5 = t18c(4, 0) * id + t18c(4, 1) * a + t18c(4, 2) * a2 + t18c(4, 3) * a3 + t18c(4, 4) * a6;
            s0[o] = b1;
            s1[o] = b5;
            s2[o] = b4;
            s3[o] = b3 + b4;
            z = b2;
          } else if (st == 3) {
            const float p = r;
            s1[o] = p + s2[o];  // A9 = B1 B5 + B4
            s0[o] = p + s3[o];  // B3 + A9
          }
        }
      }
    }
  }
}

template <int P, bool Pair>
__device__ __forceinline__ void tile_to_slot(float* __restrict__ slot, int i0, int j0, const Tile<Pair>& R) {
#pragma unroll
  for (int ii = 0; ii < 4; ++ii) {
    float4* p0 = reinterpret_cast<float4*>(slot + pidx<P>(i0 + ii, j0));
    float4* p1 = reinterpret_cast<float4*>(slot + pidx<P>(i0 + ii, j0 + 4));
    *p0 = make_float4(R.d[ii][0], R.d[ii][1], R.d[ii][2], R.d[ii][3]);
    *p1 = make_float4(R.d[ii][4], R.d[ii][5], R.d[ii][6], R.d[ii][7]);
    if constexpr (Pair) {
      float4* q0 = reinterpret_cast<float4*>(slot + P * P + pidx<P>(i0 + ii, j0));
      float4* q1 = reinterpret_cast<float4*>(slot + P * P + pidx<P>(i0 + ii, j0 + 4));
      *q0 = make_float4(R.u[ii][0], R.u[ii][1], R.u[ii][2], R.u[ii][3]);
      *q1 = make_float4(R.u[ii][4], R.u[ii][5], R.u[ii][6], R.u[ii][7]);
    }
  }
}

template <int P, bool Pair, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) expm_team_kernel(View a, View e, void* __restrict__ out,
                                                                  int64_t batch, int n, int dtype) {
  using C = TeamCfg<P, Pair>;
  extern __shared__ __align__(16) float smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int team_id = lane / C::T;
  const int t = lane % C::T;
  const int rb = t / C::CB, cb = t % C::CB;
  const int i0 = 4 * rb, j0 = 8 * cb;
  float* team = smem + warp * C::WARP_FLOATS + team_id * C::TEAM_FLOATS;
  const unsigned team_mask = (C::T == 32) ? 0xffffffffu : (((1u << C::T) - 1u) << (team_id * C::T));

  const int64_t n_items = (batch + C::TPW - 1) / C::TPW;
  const int64_t warps_total = int64_t(gridDim.x) * WARPS;
  for (int64_t item = int64_t(blockIdx.x) * WARPS + warp; item < n_items; item += warps_total) {
    const int64_t b = item * C::TPW + team_id;
    const bool valid = b < batch;

    // ---- load the lane's tile of A (and E), zero-padded to P x P ----
    Tile<Pair> R, Z;
    bool bad = false;
    double col[8], row[4];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) col[jj] = 0.0;
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) row[ii] = 0.0;
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int i = i0 + ii, j = j0 + jj;
        float v = 0.f, w = 0.f;
        if (valid && i < n && j < n) {
          v = a.sign * load_elem(a.data, dtype, b * a.s0 + i * a.s1 + j * a.s2);
          if constexpr (Pair) w = e.sign * load_elem(e.data, dtype, b * e.s0 + i * e.s1 + j * e.s2);
        }
        bad |= !isfinite(v);
        if constexpr (Pair) bad |= !isfinite(w);
        const double av = fabs(double(v));
        col[jj] += av;
        row[ii] += av;
        R.d[ii][jj] = v;
        if constexpr (Pair) R.u[ii][jj] = w;
      }
    }
    const bool team_bad = (__ballot_sync(0xffffffffu, bad) & team_mask) != 0u;
    // Column sums over the row blocks of the team, then the largest column.
#pragma unroll
    for (int off = C::CB; off < C::T; off <<= 1)
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) col[jj] += __shfl_xor_sync(0xffffffffu, col[jj], off);
#pragma unroll
    for (int off = 1; off < C::CB; off <<= 1)
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) row[ii] += __shfl_xor_sync(0xffffffffu, row[ii], off);
    double n1 = 0.0, ninf = 0.0;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) n1 = fmax(n1, col[jj]);
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) ninf = fmax(ninf, row[ii]);
#pragma unroll
    for (int off = 1; off < C::T; off <<= 1) {
      n1 = fmax(n1, __shfl_xor_sync(0xffffffffu, n1, off));
      ninf = fmax(ninf, __shfl_xor_sync(0xffffffffu, ninf, off));
    }
    int m = 1, s = 0;
    choose_degree(fmin(n1, ninf), &m, &s);
    const int poly = scheme_products(m);
    const int nsteps = (valid && !team_bad) ? poly + s : 0;

    // ---- scale by 2^-s and place A in slot 0 ----
    if (s > 0) {
#pragma unroll
      for (int ii = 0; ii < 4; ++ii)
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          R.d[ii][jj] = scale_pow2(R.d[ii][jj], s);
          if constexpr (Pair) R.u[ii][jj] = scale_pow2(R.u[ii][jj], s);
        }
    }
    tile_to_slot<P, Pair>(team, i0, j0, R);
    if (m == 1) {  // T1 = I + A (s == 0 here)
#pragma unroll
      for (int ii = 0; ii < 4; ++ii)
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) R.d[ii][jj] += (i0 + ii == j0 + jj) ? 1.f : 0.f;
    }
    tile_zero(Z);
    __syncwarp();

    // ---- polynomial steps, then squarings, in lockstep across the warp ----
    const int max_steps = __reduce_max_sync(0xffffffffu, nsteps);
    for (int st = 0; st < max_steps; ++st) {
      const bool active = st < nsteps;
      int xs = 0, ys = 0;
      bool use_z = false;
      if (st < poly) step_operands(m, st, &xs, &ys, &use_z);
      if (active) team_product<P, Pair>(team + xs * C::SLOT, team + ys * C::SLOT, i0, j0, R, Z, use_z);
      __syncwarp();
      if (active) {
        const bool last = st == nsteps - 1;
        if (st < poly) step_epilogue<P, Pair>(m, st, team, i0, j0, R, Z);
        if ((st >= poly - 1) && !last) tile_to_slot<P, Pair>(team, i0, j0, R);
      }
      __syncwarp();
    }

    // ---- store the n x n corner ----
    if (valid) {
      const int64_t obase = b * int64_t(n) * n;
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const int i = i0 + ii, j = j0 + jj;
          if (i < n && j < n) {
            float v;
            if constexpr (Pair) {
              v = R.u[ii][jj];
            } else {
              v = R.d[ii][jj];
            }
            if (team_bad) v = __int_as_float(0x7fc00000);
            store_elem(out, dtype, obase + int64_t(i) * n + j, v);
          }
        }
      }
    }
  }
}

}  // namespace fhx
