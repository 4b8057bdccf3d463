// Team kernel: padded sizes P = 8, 16, 32 (n = 5..32).
//
// A "team" of T = (P/TM) * (P/TN) threads owns one matrix; thread (rb, cb) of the team owns
// the TM x TN register tile at rows TM*rb.., columns TN*cb...  Teams of 4 threads (P = 8, 4 x 4
// tiles), 8 threads (P = 8 grouped Frechet, 2 x 4 tiles) or 16 threads (P = 16 forward) share a
// warp; the P = 16 Frechet team is one warp (2 x 4 tiles); at P = 32 a team is two warps
// (forward, 4 x 4 tiles) or four warps (Frechet, 2 x 4 tiles).  The matrix state lives in five
// shared-memory plane slots per team; registers hold only the accumulator tile of the product
// in flight.
//
// Every polynomial step and every squaring is one product R = X Y (+ Z) of slots X, Y (Z an
// optional slot added on the way in), computed as a register-tiled outer product: per four
// k a thread reads the TM x 4 block of X it needs (TM 128-bit loads) and per k the TN values
// of row k of Y (TN/4 128-bit loads), accumulating in float2 pairs with the paired FMA of
// sm_100 (FFMA2) -- three products at once in Frechet mode, where every matrix is the pair
// (M, dM) of the block-triangular [[M, dM], [0, M]] and (X, dX)(Y, dY) = (XY, X dY + dX Y).
// Planes are row-major with the 16-byte chunks of row i rotated by i/4, so the block reads of
// different row blocks hit different bank groups while every chunk stays 16-byte aligned.
//
// The degree-m schemes are table-driven "step programs" (step_def below): after each product
// the thread writes R into a slot and applies the step's element-wise linear combinations to
// its own tile (the next operands of the scheme), with the coefficients as compile-time
// immediates.  Multi-warp teams synchronise with a named barrier per team and square in
// ping-pong between two slots (one barrier per squaring).  Teams that share a warp run in
// lockstep with __syncwarp.  The eight 8 x 8 teams of a warp either run one program, the
// largest degree chosen in the warp (each matrix keeping its own number of squarings; a higher
// degree with the same scaling is at least as accurate), or -- grouped mode, with a workspace --
// take matrices pre-sorted by (degree, squarings) and run their own.  The two 16 x 16 forward
// teams of a warp run their own degrees (at most two epilogue paths).
//
// Loads are 16-byte chunks spread over the team and prefetched one matrix ahead into
// registers as raw bits (decoded when the next matrix starts); norms are read back from the
// slot; results leave in 16-byte chunks.
//
// Work is persistent: grid = resident CTAs, CTA c takes CTA items c, c + gridDim.x, ...
//
// Reference counterpart: scalar::tiled_kernel (csrc/MatrixExpSmall.cuh:177-385) -- one CTA
// per padded 16x16 / 32x32 matrix with 2-8 elements per thread, operands restaged through
// shared memory with two __syncthreads per product, fixed degree 18.
#pragma once

#include "expm_common.cuh"
#include "expm_sort.cuh"

namespace fhx {

constexpr int kSlots = 5;

#ifndef FHX_FRECHET8_MINBLOCKS
#define FHX_FRECHET8_MINBLOCKS 16
#endif

// Layout flags of a launch (computed on the host from strides, dtype and alignment).
// A view is moved in 16-byte chunks: four consecutive elements of a row ("row chunks",
// when the elements of a row are closest in memory, s2 <= s1) or of a column ("column
// chunks", s1 < s2).  "Vec": the chunk is contiguous and aligned (16 bytes for float32, 8 for
// the half types) and n == P, so it is one 128-bit or 64-bit load.
enum : unsigned {
  kARows = 1u,    // input: row chunks
  kAVec = 2u,     // input: one vector load per chunk
  kERows = 4u,    // direction: row chunks
  kEVec = 8u,     // direction: one vector load per chunk
  kOutVec = 16u,  // output: n % 4 == 0 and 16-byte (float32) / 8-byte (half types) aligned
  kOut2T = 32u,   // Frechet launches with a second output: write exp(A) transposed there
  kOut2Vec = 64u, // second output: as kOutVec
};
constexpr int kMaxIn = 4;
constexpr int kMaxOut = 5;

// One step of a degree program: R = slot[x] * slot[y] (+ slot[z] if z >= 0), R -> slot[r],
// then nout outputs out[o] = coef[o][0] * I + sum_j coef[o][1 + j] * slot[in[j]], evaluated
// element-wise on the lane's own tile with every input read before any output is written.
struct Step {
  signed char x, y, z, r;
  signed char nin, nout;
  signed char in[kMaxIn];
  signed char out[kMaxOut];
  float coef[kMaxOut][kMaxIn + 1];
};

// Programs for m = 2, 4, 8, 12, 18 (steps numbered from 0; the result ends in slot 0).
// Slots: 0 holds A on entry.  Coefficients: BBC 2019 schemes, expm_coeffs.h.
constexpr int kNumSteps = 15;
__host__ __device__ constexpr Step step_def(int index) {
  constexpr Step tab[kNumSteps] = {
      // m = 2: A2 -> s1; s0 = I + A + A2/2
      {0, 0, -1, 1, 2, 1, {0, 1}, {0}, {{1.f, 1.f, 0.5f}}},
      // m = 4: A2 -> s1; s2 = I/2 + A/6 + A2/24, s3 = I + A
      {0, 0, -1, 1, 2, 2, {0, 1}, {2, 3}, {{0.5f, 1.f / 6.f, 1.f / 24.f}, {1.f, 1.f, 0.f}}},
      //         s0 = A2 * s2 + s3
      {1, 2, 3, 0, 0, 0, {}, {}, {}},
      // m = 8: A2 -> s1; s2 = x1 A + x2 A2 (C1), s3 = I + A + y2 A2 (F)
      {0, 0, -1, 1, 2, 2, {0, 1}, {2, 3}, {{0.f, kT8X1, kT8X2}, {1.f, 1.f, kT8Y2}}},
      //         A4 = A2 * C1 -> s4; s2 = x3 A2 + A4 (L), s0 = x4 I + x5 A + x6 A2 + x7 A4 (R)
      {1, 2, -1, 4, 3, 2, {0, 1, 4}, {2, 0}, {{0.f, 0.f, kT8X3, 1.f}, {kT8X4, kT8X5, kT8X6, kT8X7}}},
      //         s0 = L * R + F
      {2, 0, 3, 0, 0, 0, {}, {}, {}},
      // m = 12: A2 -> s1
      {0, 0, -1, 1, 0, 0, {}, {}, {}},
      //          A3 -> s2; s3 = B4, s4 = B3, s1 = B2, s0 = B1 (on I, A, A2, A3)
      {1, 0, -1, 2, 3, 4, {0, 1, 2}, {3, 4, 1, 0},
       {{t12c(3, 0), t12c(3, 1), t12c(3, 2), t12c(3, 3)},
        {t12c(2, 0), t12c(2, 1), t12c(2, 2), t12c(2, 3)},
        {t12c(1, 0), t12c(1, 1), t12c(1, 2), t12c(1, 3)},
        {t12c(0, 0), t12c(0, 1), t12c(0, 2), t12c(0, 3)}}},
      //          A6 = B4 * B4 + B3 -> s2; s1 = B2 + A6
      {3, 3, 4, 2, 2, 1, {1, 2}, {1}, {{0.f, 1.f, 1.f}}},
      //          s0 = (B2 + A6) * A6 + B1
      {1, 2, 0, 0, 0, 0, {}, {}, {}},
      // m = 18: A2 -> s1
      {0, 0, -1, 1, 0, 0, {}, {}, {}},
      //          A3 -> s2
      {1, 0, -1, 2, 0, 0, {}, {}, {}},
      //          A6 -> s3; s0 = B1, s1 = B5, s2 = B4, s3 = B3 + B4, s4 = B2 (on I, A, A2, A3, A6)
      {2, 2, -1, 3, 4, 5, {0, 1, 2, 3}, {0, 1, 2, 3, 4},
       {{t18c(0, 0), t18c(0, 1), t18c(0, 2), t18c(0, 3), t18c(0, 4)},
        {t18c(4, 0), t18c(4, 1), t18c(4, 2), t18c(4, 3), t18c(4, 4)},
        {t18c(3, 0), t18c(3, 1), t18c(3, 2), t18c(3, 3), t18c(3, 4)},
        {t18c(2, 0) + t18c(3, 0), t18c(2, 1) + t18c(3, 1), t18c(2, 2) + t18c(3, 2), t18c(2, 3) + t18c(3, 3),
         t18c(2, 4) + t18c(3, 4)},
        {t18c(1, 0), t18c(1, 1), t18c(1, 2), t18c(1, 3), t18c(1, 4)}}},
      //          P = B1 * B5 -> s0; s1 = P + B4 (A9), s0 = P + B3 + B4
      {0, 1, -1, 0, 3, 2, {0, 2, 3}, {1, 0}, {{0.f, 1.f, 1.f, 0.f}, {0.f, 1.f, 0.f, 1.f}}},
      //          s0 = (B3 + A9) * A9 + B2
      {0, 1, 4, 0, 0, 0, {}, {}, {}},
  };
  return tab[index];
}

// Device copy for the step machine (operand slots, output count); the epilogues take their
// coefficients from step_def at compile time.
__constant__ Step kSteps[kNumSteps] = {step_def(0),  step_def(1),  step_def(2),  step_def(3),  step_def(4),
                                       step_def(5),  step_def(6),  step_def(7),  step_def(8),  step_def(9),
                                       step_def(10), step_def(11), step_def(12), step_def(13), step_def(14)};

__host__ __device__ __forceinline__ int program_offset(int m) {
  return m == 2 ? 0 : m == 4 ? 1 : m == 8 ? 3 : m == 12 ? 6 : 10;
}

// Last step of the program that contains step S.
__host__ __device__ constexpr int program_last(int S) { return S == 0 ? 0 : S <= 2 ? 2 : S <= 5 ? 5 : S <= 9 ? 9 : 14; }

__host__ __device__ constexpr bool step_reads(const Step& st, int slot, bool epilogue) {
  if (!epilogue) return st.x == slot || st.y == slot || st.z == slot;
  for (int t = 0; t < st.nin; ++t)
    if (st.in[t] == slot) return true;
  return false;
}
__host__ __device__ constexpr bool step_writes_out(const Step& st, int slot) {
  for (int o = 0; o < st.nout; ++o)
    if (st.out[o] == slot) return true;
  return false;
}

// Whether the product result of step S must go to its slot r: not when S's own epilogue
// overwrites r (it reads the result from registers), nor when no later step of the program
// reads r before writing it (the program's result, slot 0 after the last step, is always
// kept).  E.g. m = 18: A6 (step 12) and B1 * B5 (step 13) live only in their epilogues.
__host__ __device__ constexpr bool product_store_needed(int S) {
  const Step st = step_def(S);
  if (step_writes_out(st, st.r)) return false;
  for (int k = S + 1; k <= program_last(S); ++k) {
    const Step nx = step_def(k);
    if (step_reads(nx, st.r, false)) return true;
    if (nx.r == st.r) return false;
    if (step_reads(nx, st.r, true)) return true;
    if (step_writes_out(nx, st.r)) return false;
  }
  return st.r == 0;
}
static_assert(!product_store_needed(12) && !product_store_needed(13) && product_store_needed(14) &&
                  product_store_needed(11) && !product_store_needed(7) && product_store_needed(8) &&
                  !product_store_needed(4) && !product_store_needed(0) && product_store_needed(1),
              "product-store liveness");


template <int P, int TM, int TN, bool Pair>
struct TeamCfg {
  static constexpr int RB = P / TM;
  static constexpr int CB = P / TN;
  static constexpr int T = RB * CB;  // threads per matrix
  static constexpr int PLANE = P * P;
  static constexpr int NPART = Pair ? 2 : 1;
  static constexpr int SLOT = NPART * PLANE;
  // Teams that share a warp start in different banks (4 floats of per-team scratch included):
  // 16 banks apart, except the four 8-thread teams of the 8 x 8 Frechet kernel, which start 8
  // apart and so cover all four offsets (measured 1.2-1.5 % faster on config 3; the eight 4 x 4
  // forward teams ran 5 % slower at 8 apart).
  static constexpr int SKEW = T >= 32 ? 0 : (P == 8 && T == 8 ? 8 : 16);
  static constexpr int TEAM_FLOATS = kSlots * SLOT + 4 + (SKEW ? SKEW - 4 : 12);
  static_assert(32 % T == 0 || (T % 32 == 0 && T <= 256), "team must divide a warp or be whole warps");
  // Thread -> tile map: each quarter-warp (8 threads) covers QR row blocks x QC column
  // blocks, and the chunks it reads together fall in distinct bank groups.  Measured on B200
  // (ncu shared-load wavefronts): a 128-bit load costs 2 wavefronts per warp both when every
  // quarter-warp reads the same four chunks (the X blocks of the 32 x 32 kernels) and when each
  // reads two and the warp eight (their Y rows); different chunks in one bank group cost more.
  static constexpr int QR = (T < 8) ? 1 : (TN >= TM ? (RB >= 4 ? 4 : RB) : 2);
  static constexpr int QC = (T < 8) ? 1 : 8 / QR;
  static_assert(T < 8 || (RB % QR == 0 && CB % QC == 0 && QR * QC == 8), "quarter-warp tiling");
  // Row blocks of one quarter-warp are RB / QR apart (e.g. 0, 4, 8, 12 of 16), so that with
  // TM = 2 they still fall in different 4-row rotation groups.
  // (At P = 8 a row spans 8 banks: row blocks 2 rows apart, e.g. 0, 2, 4, 6 with TM = 2, still
  // start in four different bank groups.)
  static_assert(T < 8 || TM * (RB / QR) >= 4 || QR == 1 || P == 8, "quarter rows must span rotation groups");
  static_assert(TEAM_FLOATS % 4 == 0, "16-byte aligned team regions");
};

// Physical row of logical row i.  A row of a P <= 16 plane covers only half of the 32 banks
// (P = 16) or a quarter (P = 8), and the rows that one quarter-warp touches together (one per
// 4-row group: i0, i0 + 4, ...) would all start in the same bank half.  Swapping the two rows of
// each pair in every other 4-row group puts them in both halves, which makes the tile-chunk
// accesses of the epilogues and squarings conflict-free (measured before: 28-41 % of the shared
// wavefronts of the 8 x 8 and 16 x 16 kernels were bank-conflict replays).  Used where it
// measured faster on B200: the 8 x 8 kernels (config 3: forward -16 %, Frechet -7 %) and the
// 16 x 16 Frechet kernel (2 x 4 tiles); the 16 x 16 forward (4 x 4 tiles, 96 registers) spilled
// and ran slower with it (2.97 against 2.38 ms on 1,048,576 matrices).
template <int P, int TM>
__host__ __device__ __forceinline__ constexpr bool swapped_rows() {
  return P == 8 || (P == 16 && TM == 2);
}
template <int P, int TM>
__host__ __device__ __forceinline__ constexpr int prow(int i) {
  return swapped_rows<P, TM>() ? (i ^ ((i >> 2) & 1)) : i;
}

// Offset of element (i, j) inside a plane: 16-byte chunk (j / 4) of row i is stored at
// chunk position (j / 4) ^ (i / 4) of physical row prow(i).  Rows of one 4-row group share a
// rotation, so a thread reads a row chunk of Y for four consecutive k with one address
// computation; the thread -> tile map spreads the row blocks of a quarter-warp over different
// 4-row groups, so their X reads hit different bank groups.  (TM is kept as a parameter of the
// call sites.)
template <int P, int TM>
__device__ __forceinline__ int pidx(int i, int j) {
  return prow<P, TM>(i) * P + ((((j >> 2) ^ (i >> 2)) & (P / 4 - 1)) << 2) + (j & 3);
}

// The row whose |a| sum thread l of the norm phase takes.  At P = 32 rows 4 (l % 8) + l / 8, so
// that the eight threads of a quarter-warp read rows of different chunk rotations (consecutive
// rows share one, and their 128-bit reads collided 4-way): 32 x 32 forward 2.8 % and Frechet
// 0.4 % faster on B200.  A permutation of the rows; only the maximum of the row sums is used.
// (At P = 16 the same idea, rows 4 (l % 4) + l / 4, measured 1.2 % slower on the forward.)
template <int P>
__device__ __forceinline__ int norm_row(int l) {
  if constexpr (P == 32) return 4 * (l & 7) + (l >> 3);
  return l;
}

template <int T>
__device__ __forceinline__ void team_sync(int team_in_cta) {
  if constexpr (T <= 32) {
    __syncwarp();
  } else {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + team_in_cta), "r"(T) : "memory");
  }
}

// Accumulators in float2 pairs along j: one paired FMA (FFMA2, sm_100) updates two of them.
template <int TM, int TN, bool Pair>
struct Acc {
  float2 d[TM][TN / 2];
  float2 u[Pair ? TM : 1][Pair ? TN / 2 : 1];
};

template <int TM, int TN, bool Pair>
__device__ __forceinline__ void acc_zero(Acc<TM, TN, Pair>& R) {
#pragma unroll
  for (int ii = 0; ii < TM; ++ii)
#pragma unroll
    for (int jj = 0; jj < TN / 2; ++jj) {
      R.d[ii][jj] = make_float2(0.f, 0.f);
      if constexpr (Pair) R.u[ii][jj] = make_float2(0.f, 0.f);
    }
}

// Thread-own tile <-> slot.  Own chunks: rows i0..i0+TM-1, chunks j0/4 .. j0/4 + TN/4 - 1.
template <int P, int TM, int TN, bool Pair>
__device__ __forceinline__ void acc_store(float* __restrict__ slot, int i0, int j0, const Acc<TM, TN, Pair>& R) {
#pragma unroll
  for (int ii = 0; ii < TM; ++ii)
#pragma unroll
    for (int c = 0; c < TN / 4; ++c) {
      const int o = pidx<P, TM>(i0 + ii, j0 + 4 * c);
      *reinterpret_cast<float4*>(slot + o) =
          make_float4(R.d[ii][2 * c].x, R.d[ii][2 * c].y, R.d[ii][2 * c + 1].x, R.d[ii][2 * c + 1].y);
      if constexpr (Pair)
        *reinterpret_cast<float4*>(slot + P * P + o) =
            make_float4(R.u[ii][2 * c].x, R.u[ii][2 * c].y, R.u[ii][2 * c + 1].x, R.u[ii][2 * c + 1].y);
    }
}

template <int P, int TM, int TN, bool Pair>
__device__ __forceinline__ void acc_load(const float* __restrict__ slot, int i0, int j0, Acc<TM, TN, Pair>& R) {
#pragma unroll
  for (int ii = 0; ii < TM; ++ii)
#pragma unroll
    for (int c = 0; c < TN / 4; ++c) {
      const int o = pidx<P, TM>(i0 + ii, j0 + 4 * c);
      const float4 a = *reinterpret_cast<const float4*>(slot + o);
      R.d[ii][2 * c] = make_float2(a.x, a.y);
      R.d[ii][2 * c + 1] = make_float2(a.z, a.w);
      if constexpr (Pair) {
        const float4 b = *reinterpret_cast<const float4*>(slot + P * P + o);
        R.u[ii][2 * c] = make_float2(b.x, b.y);
        R.u[ii][2 * c + 1] = make_float2(b.z, b.w);
      }
    }
}

__device__ __forceinline__ float f4get(const float4& v, int r) { return r == 0 ? v.x : r == 1 ? v.y : r == 2 ? v.z : v.w; }

// 128-bit shared-memory load from a 32-bit shared address.  Written as explicit ld.shared:
// for the product's access pattern this costs one shared-memory wavefront per load, where the
// compiler's own code for the same float4 dereference measured about 3.3 (ncu,
// l1tex__data_pipe_lsu_wavefronts_mem_shared_op_ld) and saturated the shared-memory pipe.
__device__ __forceinline__ float4 lds128(unsigned addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ unsigned smem_addr(const float* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

// R += X Y.  X, Y: first (value) plane of a slot; the derivative plane follows at +PLANE.
// Per group of four k: the TM x 4 block of X (TM 128-bit loads) and, for each of the
// thread's TN/4 column chunks, rows 4q..4q+3 of Y at one rotated chunk position.  The Y
// addresses of a group are one base register per chunk plus immediate row offsets (a
// per-k address computation measured 8 % slower on the 32 x 32 kernels).  A variant that
// issued the loads of k + 1 into a second register buffer before the FMAs of k (software
// pipelining) measured no faster on any shape: the loop is not latency-bound.
template <int P, int TM, int TN, bool Pair>
__device__ __forceinline__ void team_product(const float* __restrict__ X, const float* __restrict__ Y, int i0, int j0,
                                             Acc<TM, TN, Pair>& R) {
  constexpr unsigned PLANE_B = P * P * 4;  // bytes
  constexpr unsigned ROW_B = P * 4;
  constexpr unsigned MASK16 = unsigned(P / 4 - 1) << 4;
  constexpr bool swapped = swapped_rows<P, TM>();
  const unsigned rx16 = unsigned(i0 >> 2) << 4;  // rotation of the thread's X rows (bytes)
  const unsigned c016 = unsigned(j0 >> 2) << 4;  // first column chunk of the tile (bytes)
  const unsigned xrow = smem_addr(X) + unsigned(i0) * ROW_B;
  // with swapped rows, rows i0 .. i0 + TM - 1 (TM even, i0 a multiple of TM) sit at physical
  // rows i0 + (ii ^ xs), and rows 4q + r of Y at 4q + (r ^ (q & 1))
  static_assert(!swapped || TM % 2 == 0, "row pairs");
  const unsigned xs = swapped ? unsigned(prow<P, TM>(i0) - i0) : 0u;
  unsigned yrow = smem_addr(Y);
  // Frechet: R.u accumulates X dY and dX Y, interleaved per k.
#pragma unroll(Pair ? (P == 32 ? 2 : 1) : (P == 32 ? 4 : 2))
  for (unsigned q16 = 0; q16 < unsigned(P / 4) * 16u; q16 += 16u) {
    const unsigned xa = xrow + ((rx16 ^ q16) & MASK16);
    float4 xb[TM], xub[TM];
#pragma unroll
    for (int ii = 0; ii < TM; ++ii) {
      const unsigned xo = (swapped ? (unsigned(ii) ^ xs) : unsigned(ii)) * ROW_B;
      xb[ii] = lds128(xa + xo);
      if constexpr (Pair) xub[ii] = lds128(xa + PLANE_B + xo);
    }
    unsigned ya[TN / 4];
#pragma unroll
    for (int c = 0; c < TN / 4; ++c) ya[c] = yrow + (((c016 + unsigned(c) * 16u) ^ q16) & MASK16);
    const unsigned ys = swapped ? (q16 >> 4) & 1u : 0u;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const unsigned yo = (swapped ? (unsigned(r) ^ ys) : unsigned(r)) * ROW_B;
      float2 y[TN / 2], yu[TN / 2];
#pragma unroll
      for (int c = 0; c < TN / 4; ++c) {
        const float4 v = lds128(ya[c] + yo);
        y[2 * c] = make_float2(v.x, v.y);
        y[2 * c + 1] = make_float2(v.z, v.w);
        if constexpr (Pair) {
          const float4 w = lds128(ya[c] + PLANE_B + yo);
          yu[2 * c] = make_float2(w.x, w.y);
          yu[2 * c + 1] = make_float2(w.z, w.w);
        }
      }
#pragma unroll
      for (int ii = 0; ii < TM; ++ii) {
        const float x = f4get(xb[ii], r);
        const float2 x2 = make_float2(x, x);
#pragma unroll
        for (int jj = 0; jj < TN / 2; ++jj) {
          R.d[ii][jj] = __ffma2_rn(x2, y[jj], R.d[ii][jj]);
          if constexpr (Pair) R.u[ii][jj] = __ffma2_rn(x2, yu[jj], R.u[ii][jj]);
        }
      }
      if constexpr (Pair) {
        // second derivative term after every other FMA of this k: the two updates of R.u are
        // a whole pass apart
#pragma unroll
        for (int ii = 0; ii < TM; ++ii) {
          const float xu = f4get(xub[ii], r);
          const float2 xu2 = make_float2(xu, xu);
#pragma unroll
          for (int jj = 0; jj < TN / 2; ++jj) R.u[ii][jj] = __ffma2_rn(xu2, y[jj], R.u[ii][jj]);
        }
      }
    }
    yrow += 4u * ROW_B;
  }
}

// Whether a kernel shape takes each step's product into its epilogue from registers (and skips
// the stores product_store_needed rules out).  Measured on B200 against storing every product:
// 8 x 8 forward and Frechet 2 % faster, 16 x 16 Frechet 0.5 % faster; the 32 x 32 Frechet 1.2 %
// slower (same registers, other scheduling), and the 16 x 16 forward, held to 96 registers for
// 20 CTAs per SM, spills with the accumulator live through the epilogue.
template <int P, int TM, int TN, bool Pair>
__host__ __device__ constexpr bool feed_product() {
  return P == 8 || (P == 16 && Pair);
}

// Whether the element-wise phases (step epilogues, the 2^-s scaling) walk the plane in
// row-major chunks t, t + T, ... instead of the thread's own tile.  For the 16 x 16 forward (4 x 4
// tiles, no row swap) the own-tile chunks of a quarter-warp fall on the same banks in pairs
// (rows 4rb + ii of one ii start in the same bank half), while two consecutive rows of a
// 16-float plane cover all 32 banks; the team (half a warp) then needs a __syncwarp between the
// product store and the epilogue.
template <int P, int TM, int TN, bool Pair>
__host__ __device__ constexpr bool rowmap_elementwise() {
  return P == 16 && !Pair;
}
static_assert(!(rowmap_elementwise<16, 4, 4, false>() && feed_product<16, 4, 4, false>()),
              "the product feed needs own-tile epilogues");

// Chunk c (0 <= c < TM * TN / 4) of the element-wise phases: elements (i, j .. j + 3) at plane
// offset off = pidx(i, j).
template <int P, int TM, int TN, bool Pair>
__device__ __forceinline__ void ew_chunk(int c, int t, int i0, int j0, int& i, int& j, int& off) {
  if constexpr (rowmap_elementwise<P, TM, TN, Pair>()) {
    // rows t / (P/4) + (T / (P/4)) c, and in each the chunk whose rotated position is t % (P/4):
    // off = i * P + 4 (t % (P/4)), one base plus an immediate per c
    constexpr int CPR = P / 4;  // chunks per row
    constexpr int RSTEP = TeamCfg<P, TM, TN, Pair>::T / CPR;
    static_assert(TeamCfg<P, TM, TN, Pair>::T * TM * TN == P * P, "row-major map covers the plane");
    static_assert(!swapped_rows<P, TM>(), "physical rows are logical rows");
    i = t / CPR + RSTEP * c;
    j = 4 * ((t % CPR) ^ ((i >> 2) & (CPR - 1)));
    off = (t / CPR) * P + 4 * (t % CPR) + RSTEP * P * c;
  } else {
    i = i0 + c / (TN / 4);
    j = j0 + 4 * (c % (TN / 4));
    off = pidx<P, TM>(i, j);
  }
}

// Element-wise linear combinations of step S on the thread's own TM x TN tile, with the
// coefficients of step_def(S) as compile-time constants: zero terms vanish, and each term is
// one FMA per element with an immediate coefficient (paired FMAs at P <= 16).  Terms are
// accumulated in the table's order, identity first.  The input that is the step's own product
// (slot r) is taken from the accumulator R, which holds the same values.
template <int P, int TM, int TN, bool Pair, int S>
__device__ __forceinline__ void epilogue_step(float* __restrict__ team, int t_in_team, int i0, int j0,
                                              const Acc<TM, TN, Pair>& R) {
  constexpr Step st = step_def(S);
  constexpr int PLANE = P * P;
  constexpr int SLOT = TeamCfg<P, TM, TN, Pair>::SLOT;
  constexpr int CH = TM * TN / 4;  // own 16-byte chunks per plane
#pragma unroll
  for (int part = 0; part < (Pair ? 2 : 1); ++part) {
    float4 in[st.nin > 0 ? st.nin : 1][CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      int i, j, o;
      ew_chunk<P, TM, TN, Pair>(c, t_in_team, i0, j0, i, j, o);
      const int off = part * PLANE + o;
#pragma unroll
      for (int t = 0; t < st.nin; ++t) {
        if (feed_product<P, TM, TN, Pair>() && st.in[t] == st.r) {
          const int ii = c / (TN / 4), cc = c % (TN / 4);
          float2 lo = R.d[ii][2 * cc], hi = R.d[ii][2 * cc + 1];
          if constexpr (Pair) {
            if (part == 1) {
              lo = R.u[ii][2 * cc];
              hi = R.u[ii][2 * cc + 1];
            }
          }
          in[t][c] = make_float4(lo.x, lo.y, hi.x, hi.y);
        } else {
          in[t][c] = *reinterpret_cast<const float4*>(team + st.in[t] * SLOT + off);
        }
      }
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      int i, j, o;
      ew_chunk<P, TM, TN, Pair>(c, t_in_team, i0, j0, i, j, o);
      const int off = part * PLANE + o;
      const int dj = part == 0 ? i - j : -1;  // identity pattern of this chunk (value plane only)
      const float4 id = make_float4(dj == 0 ? 1.f : 0.f, dj == 1 ? 1.f : 0.f, dj == 2 ? 1.f : 0.f, dj == 3 ? 1.f : 0.f);
#pragma unroll
      for (int o = 0; o < st.nout; ++o) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if constexpr (P <= 16) {
          // (x, y) and (z, w) halves, two lanes per paired FMA: at small P these O(P^2)
          // combinations are a large share of the work per matrix.
          float2 lo = make_float2(0.f, 0.f), hi = make_float2(0.f, 0.f);
          bool first = true;
          if (st.coef[o][0] != 0.f) {
            const float c0 = st.coef[o][0];
            lo = make_float2(c0 * id.x, c0 * id.y);
            hi = make_float2(c0 * id.z, c0 * id.w);
            first = false;
          }
#pragma unroll
          for (int t = 0; t < st.nin; ++t) {
            const float cf = st.coef[o][1 + t];
            if (cf == 0.f) continue;
            const float2 xl = make_float2(in[t][c].x, in[t][c].y), xh = make_float2(in[t][c].z, in[t][c].w);
            const float2 c2 = make_float2(cf, cf);
            if (first) {
              lo = cf == 1.f ? xl : __fmul2_rn(c2, xl);
              hi = cf == 1.f ? xh : __fmul2_rn(c2, xh);
              first = false;
            } else if (cf == 1.f) {
              lo = __fadd2_rn(lo, xl);
              hi = __fadd2_rn(hi, xh);
            } else {
              lo = __ffma2_rn(c2, xl, lo);
              hi = __ffma2_rn(c2, xh, hi);
            }
          }
          v = make_float4(lo.x, lo.y, hi.x, hi.y);
        } else {
          bool first = true;
          if (st.coef[o][0] != 0.f) {
            const float c0 = st.coef[o][0];
            v = make_float4(c0 * id.x, c0 * id.y, c0 * id.z, c0 * id.w);
            first = false;
          }
#pragma unroll
          for (int t = 0; t < st.nin; ++t) {
            const float cf = st.coef[o][1 + t];
            if (cf == 0.f) continue;
            const float4 x = in[t][c];
            if (first) {
              v = cf == 1.f ? x : make_float4(cf * x.x, cf * x.y, cf * x.z, cf * x.w);
              first = false;
            } else if (cf == 1.f) {
              v.x += x.x; v.y += x.y; v.z += x.z; v.w += x.w;
            } else {
              v.x = fmaf(cf, x.x, v.x);
              v.y = fmaf(cf, x.y, v.y);
              v.z = fmaf(cf, x.z, v.z);
              v.w = fmaf(cf, x.w, v.w);
            }
          }
        }
        *reinterpret_cast<float4*>(team + st.out[o] * SLOT + off) = v;
      }
    }
  }
}

// The end of polynomial step S, dispatched on the runtime step index: the product R to slot r
// where a later step reads it, then the step's epilogue (inlined: measured faster than an
// out-of-line call, which moves registers across the call boundary).  Shapes without
// feed_product store R before the call and use only the epilogues.
template <int P, int TM, int TN, bool Pair>
__device__ __forceinline__ void team_epilogue(int step_index, float* __restrict__ team, int t_in_team, int i0, int j0,
                                              const Acc<TM, TN, Pair>& R) {
  constexpr int SLOT = TeamCfg<P, TM, TN, Pair>::SLOT;
  switch (step_index) {
#define FHX_EPI(S)                                                                                  \
  case S:                                                                                           \
    if constexpr (feed_product<P, TM, TN, Pair>() && product_store_needed(S)) acc_store<P, TM, TN, Pair>(team + step_def(S).r * SLOT, i0, j0, R); \
    if constexpr (step_def(S).nout > 0) epilogue_step<P, TM, TN, Pair, S>(team, t_in_team, i0, j0, R);      \
    break;
    FHX_EPI(0) FHX_EPI(1) FHX_EPI(2) FHX_EPI(3) FHX_EPI(4) FHX_EPI(5) FHX_EPI(6) FHX_EPI(7)
    FHX_EPI(8) FHX_EPI(9) FHX_EPI(10) FHX_EPI(11) FHX_EPI(12) FHX_EPI(13) FHX_EPI(14)
#undef FHX_EPI
    default:
      break;
  }
}

// Raw bits of one chunk of matrix b of a view (zero outside the n x n matrix): elements
// (r, c..c+3) for a row chunk, (r..r+3, c) for a column chunk; float32 bits, or a 16-bit
// value in the low half of each word.  Nothing is computed from the loaded values here, so a
// prefetch never waits for its own loads; decode_chunk converts at the point of use.
__device__ __forceinline__ uint4 load_chunk_raw(const View& v, int dtype, int64_t b, int r, int c, int n, bool rowc,
                                                bool vec) {
  const int64_t base = b * v.s0 + int64_t(r) * v.s1 + int64_t(c) * v.s2;
  if (vec) {
    if (dtype == kF32) {
      const float4 x = ld_f32x4(static_cast<const float*>(v.data) + base);
      return make_uint4(__float_as_uint(x.x), __float_as_uint(x.y), __float_as_uint(x.z), __float_as_uint(x.w));
    }
    // four 16-bit elements in one 64-bit load, each moved to the low half of a word
    const uint2 h = ld_u32x2(reinterpret_cast<const unsigned*>(static_cast<const unsigned short*>(v.data) + base));
    return make_uint4(h.x & 0xffffu, h.x >> 16, h.y & 0xffffu, h.y >> 16);
  }
  const int64_t step = rowc ? v.s2 : v.s1;
  unsigned w[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    w[u] = 0u;
    if ((rowc ? r : r + u) < n && (rowc ? c + u : c) < n) {
      const int64_t off = base + u * step;
      w[u] = dtype == kF32 ? __float_as_uint(ld_f32(static_cast<const float*>(v.data) + off))
                           : unsigned(ld_u16(static_cast<const unsigned short*>(v.data) + off));
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Chunk q of a P x P matrix: row chunks enumerate (row, column block) row-major, column chunks
// (column, row block) column-major, so consecutive threads read consecutive addresses.
template <int P>
__device__ __forceinline__ void chunk_coords(int q, bool rowc, int* r, int* c) {
  if (rowc) {
    *r = q / (P / 4);
    *c = 4 * (q % (P / 4));
  } else {
    *r = 4 * (q % (P / 4));
    *c = q / (P / 4);
  }
}

__device__ __forceinline__ float decode_elem(unsigned w, int dtype, float sign) {
  if (dtype == kF32) return sign * __uint_as_float(w);
  const unsigned short h = static_cast<unsigned short>(w);
  return sign * (dtype == kBF16 ? __bfloat162float(__ushort_as_bfloat16(h)) : __half2float(__ushort_as_half(h)));
}

__device__ __forceinline__ float4 decode_chunk(const uint4& w, int dtype, float sign) {
  return make_float4(decode_elem(w.x, dtype, sign), decode_elem(w.y, dtype, sign), decode_elem(w.z, dtype, sign),
                     decode_elem(w.w, dtype, sign));
}

__device__ __forceinline__ bool finite4(const float4& x) {
  return isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w);
}

// Resident CTAs per SM the shared-memory footprint allows; passed to __launch_bounds__ so
// that register allocation does not become the tighter limit.
template <int P, int TM, int TN, bool Pair, int WARPS>
constexpr int team_min_blocks() {
  constexpr int smem = (WARPS * 32 / TeamCfg<P, TM, TN, Pair>::T) * TeamCfg<P, TM, TN, Pair>::TEAM_FLOATS * 4 + 1024;
  // Frechet teams smaller than a warp keep their registers (measured: the bound costs more in
  // spills than the extra resident warps return), except the 8 x 8 Frechet with 2 x 4 tiles,
  // which fits 128 registers without spills (16 CTAs of one warp).  The 32 x 32 forward runs 8
  // CTAs (16 warps) at 128 registers rather than 10 at 96 (measured 3 % faster on config 5: no
  // spills in the per-matrix phases); the 16 x 16 forward runs 20 CTAs (measured 4 % faster than
  // the shared-memory bound of 16).  Every other shape gets the shared-memory bound.
  if constexpr (Pair && P == 8 && TM == 2) return FHX_FRECHET8_MINBLOCKS;
  if constexpr (Pair && TeamCfg<P, TM, TN, Pair>::T < 32) return 1;
  if constexpr (P == 32 && !Pair && TM * TN == 16) return 8;
  if constexpr (P == 16 && !Pair) return 20;
  return (228 * 1024) / smem > 16 ? 16 : (228 * 1024) / smem;
}

// The n x n matrix of plane `res` to a contiguous [batch, n, n] output, 16-byte chunks spread
// over the team; `transposed`: element (r, c) of the output is element (c, r) of the plane.
template <int P, int TM, int T>
__device__ __forceinline__ void store_plane(const float* __restrict__ res, void* __restrict__ out, int dtype, int64_t b,
                                            int n, int t, bool vec, bool transposed, bool bad) {
  const float nanv = __int_as_float(0x7fc00000);
#pragma unroll 1
  for (int idx = t; idx < n * (P / 4); idx += T) {
    const int r = idx / (P / 4);
    const int c = 4 * (idx % (P / 4));
    if (c >= n) continue;
    float4 v;
    if (transposed) {
      v = make_float4(res[pidx<P, TM>(c, r)], res[pidx<P, TM>(c + 1, r)], res[pidx<P, TM>(c + 2, r)],
                      res[pidx<P, TM>(c + 3, r)]);
    } else {
      v = *reinterpret_cast<const float4*>(res + pidx<P, TM>(r, c));
    }
    if (bad) v = make_float4(nanv, nanv, nanv, nanv);
    const int64_t o = (b * n + r) * int64_t(n) + c;
    if (vec) {
      store_chunk(out, dtype, o, v);
    } else {
      const float vals[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c + u < n) store_elem(out, dtype, o + u, vals[u]);
    }
  }
}

__device__ __forceinline__ int ld_s32(const int* p) {
  int v;
  asm volatile("ld.global.nc.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// out: the result (exp(A), or L(A, E) for Frechet launches); out2 (Frechet launches only,
// may be null): exp(A) of the same launch -- the value part of the pair -- transposed when
// flags has kOut2T.
// Grouped (keys set; expm_sort.cuh): each matrix's (m, s) comes from its key instead of the
// in-kernel norms, and no degree is shared between teams.  With perm (the 5 <= n <= 8 grouping)
// the team's k-th matrix is perm[k] instead of k and its key keys[perm[k]]; without (keyed mode,
// the keys a forward launch stored) it is matrix k with key keys[k].  A template parameter, so
// that the ungrouped kernel carries none of it in registers.
// KeysOut (ungrouped launches): every matrix's key, make_key(m, s) or kKeyBad, is stored in
// keys_out for a later keyed launch on the same matrices or their transposes.  A separate
// instantiation, so that the other launches compile as without it.
template <int P, int TM, int TN, bool Pair, int WARPS, bool Grouped, bool KeysOut = false>
__global__ void __launch_bounds__(WARPS * 32, (team_min_blocks<P, TM, TN, Pair, WARPS>())) expm_team_kernel(View a, View e, void* __restrict__ out,
                                                                  void* __restrict__ out2, const int* __restrict__ perm,
                                                                  const unsigned short* __restrict__ keys,
                                                                  unsigned short* __restrict__ keys_out,
                                                                  int64_t batch, int n, int dtype, unsigned flags) {
  const bool a_rows = flags & kARows, a_vec = flags & kAVec;
  const bool e_rows = flags & kERows, e_vec = flags & kEVec;
  const bool out_vec = flags & kOutVec;
  using C = TeamCfg<P, TM, TN, Pair>;
  constexpr int T = C::T;
  constexpr int TPC = WARPS * 32 / T;  // teams per CTA
  static_assert(TPC >= 1, "CTA too small for one team");
  extern __shared__ __align__(16) float smem[];
  const int tic = threadIdx.x / T;  // team index in the CTA
  const int t = threadIdx.x % T;
  int rb, cb;
  if constexpr (T < 8) {
    rb = t / C::CB;
    cb = t % C::CB;
  } else {
    const int u = t / 8, v = t % 8;  // quarter-warp u, thread v within it
    rb = (v / C::QC) * (C::RB / C::QR) + u / (C::CB / C::QC);
    cb = (u % (C::CB / C::QC)) * C::QC + v % C::QC;
  }
  const int i0 = TM * rb, j0 = TN * cb;
  float* team = smem + tic * C::TEAM_FLOATS;
  int* scratch = reinterpret_cast<int*>(team + kSlots * C::SLOT);
  if (t == 0) scratch[3] = 0;
  __syncthreads();

  // Every thread moves 16-byte chunks of A (and E); chunks are enumerated row-major for
  // row-contiguous views and column-major otherwise, so that consecutive threads read
  // consecutive addresses.
  constexpr int CHUNKS = P * P / 4;
  constexpr int PER_THREAD = (CHUNKS * C::NPART + T - 1) / T;
  uint4 vals[PER_THREAD];
  int64_t pf_b = 0;     // matrix index of the prefetched matrix (grouped mode)
  unsigned pf_key = 0;  // and its key
  constexpr bool grouped = Grouped;
  auto fetch = [&](int64_t next_item) {
    int64_t nb = next_item * TPC + tic;
    bool ok = nb < batch;
    if constexpr (grouped) {
      if (ok) {
        if (perm != nullptr) {
          nb = ld_s32(perm + nb);
          ok = nb >= 0 && nb < batch;  // an entry outside the batch (a foreign workspace) is skipped
        }
        pf_key = ok ? ld_u16(keys + nb) : 0u;
      }
      pf_b = ok ? nb : -1;
    }
#pragma unroll
    for (int k = 0; k < PER_THREAD; ++k) {
      const int idx = t + k * T;
      const int part = idx / CHUNKS;
      const int q = idx % CHUNKS;
      const bool rowc = part == 0 ? a_rows : e_rows;
      int r, c;
      chunk_coords<P>(q, rowc, &r, &c);
      vals[k] = make_uint4(0u, 0u, 0u, 0u);
      if (ok && idx < CHUNKS * C::NPART) {
        vals[k] = part == 0 ? load_chunk_raw(a, dtype, nb, r, c, n, rowc, a_vec)
                            : load_chunk_raw(e, dtype, nb, r, c, n, rowc, e_vec);
      }
    }
  };
  fetch(blockIdx.x);
  for (int64_t item = blockIdx.x; item * TPC < batch; item += gridDim.x) {
    const bool valid = item * TPC + tic < batch && (!grouped || pf_b >= 0);
    const int64_t b = grouped ? pf_b : item * TPC + tic;
    const unsigned key = pf_key;

    // ---- A (and E) of this matrix, prefetched during the previous one, into slot 0 ----
    bool bad = false;
#pragma unroll
    for (int k = 0; k < PER_THREAD; ++k) {
      const int idx = t + k * T;
      if (idx < CHUNKS * C::NPART) {
        const int part = idx / CHUNKS;
        const int q = idx % CHUNKS;
        const bool rowc = part == 0 ? a_rows : e_rows;
        int r, c;
        chunk_coords<P>(q, rowc, &r, &c);
        const float4 x = decode_chunk(vals[k], dtype, part == 0 ? a.sign : e.sign);
        bad |= !finite4(x);
        float* plane = team + part * C::PLANE;
        if (rowc) {
          *reinterpret_cast<float4*>(plane + pidx<P, TM>(r, c)) = x;
        } else {
          plane[pidx<P, TM>(r, c)] = x.x;
          plane[pidx<P, TM>(r + 1, c)] = x.y;
          plane[pidx<P, TM>(r + 2, c)] = x.z;
          plane[pidx<P, TM>(r + 3, c)] = x.w;
        }
      }
    }
    fetch(item + gridDim.x);  // next matrix of this team: loads stay in flight during the steps
    if (bad) scratch[3] = 1;
    team_sync<T>(tic);
    int m = 1, s = 0, nsteps = 0;
    if constexpr (grouped) {
      if (key != kKeyBad) {
        m = degree_of_index(int(key & 7u));
        s = int(key >> 3);
      }
    } else {
      // ---- norms: sums of |row| and |column| of A, maxima over the team ----
      // Sums of |a| in four float32 partial sums combined in float64; a partial sum that
      // overflows float32 (entries near the float32 limit) is redone in float64.  Multi-warp
      // teams split the work: threads 0..P-1 rows, P..2P-1 columns.
      auto line_sum = [&](int l, bool column) {
        // element k of line l: a[l][k] for a row, a[k][l] for a column
        auto at = [&](int k) { return team[column ? pidx<P, TM>(k, l) : pidx<P, TM>(l, k)]; };
        float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < P; ++k) ps[k & 3] += fabsf(at(k));
        double sum = (double(ps[0]) + double(ps[1])) + (double(ps[2]) + double(ps[3]));
        if (!isfinite(sum)) {
          sum = 0.0;
#pragma unroll 1
          for (int k = 0; k < P; ++k) sum += fabs(double(at(k)));
        }
        return sum;
      };
      static_assert(T <= 32 || (P == 32 && T >= 2 * P), "team norm split");
      double nrow = 0.0, ncol = 0.0;
      // row l with 128-bit loads; same partial sums (element k into ps[k % 4], k ascending)
      auto row_sum = [&](int l) {
        float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c4 = 0; c4 < P / 4; ++c4) {
          const float4 x = *reinterpret_cast<const float4*>(team + pidx<P, TM>(l, 4 * c4));
          ps[0] += fabsf(x.x);
          ps[1] += fabsf(x.y);
          ps[2] += fabsf(x.z);
          ps[3] += fabsf(x.w);
        }
        const double sum = (double(ps[0]) + double(ps[1])) + (double(ps[2]) + double(ps[3]));
        return isfinite(sum) ? sum : line_sum(l, false);
      };
      if constexpr (T > 32) {
        if (t < P) {
          nrow = row_sum(norm_row<P>(t));
        } else if (t < 2 * P) {
          ncol = line_sum(t - P, true);
        }
      } else {
        for (int l = t; l < P; l += T) {
          nrow = fmax(nrow, row_sum(norm_row<P>(l)));
          ncol = fmax(ncol, line_sum(l, true));
        }
      }
      if constexpr (T <= 32) {
        // Max over all T lanes of the team: every lane must end with the team's (m, s).  Lanes
        // t >= P (teams wider than the matrix) hold no line and contribute 0.
#pragma unroll
        for (int off = 1; off < T; off <<= 1) {
          nrow = fmax(nrow, __shfl_xor_sync(0xffffffffu, nrow, off));
          ncol = fmax(ncol, __shfl_xor_sync(0xffffffffu, ncol, off));
        }
      } else {
        // warp 0 holds the row sums, warp 1 the column sums (P = 32)
        double* maxima = reinterpret_cast<double*>(scratch + 4);
        if (t < 64) {
          double v = t < 32 ? nrow : ncol;
#pragma unroll
          for (int off = 1; off < 32; off <<= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, off));
          if ((t & 31) == 0) maxima[t >> 5] = v;
        }
        team_sync<T>(tic);  // also: every column read is done before tiles are rescaled
        nrow = maxima[0];
        ncol = maxima[1];
      }
      choose_degree(fmin(nrow, ncol), &m, &s);
      if constexpr (P == 8) {
        // The eight teams of a warp run one program, of the largest degree chosen in the warp:
        // the step epilogues of different degrees would otherwise run one after another
        // (measured: 30% of the 8 x 8 Frechet time on mixed-degree batches).  A team keeps its
        // own s, which stays valid for a higher degree (theta_m grows with m), so accuracy never
        // drops; the degree of a matrix then depends on the aligned group of 8 matrices that
        // shares its warp.  (The grouped mode, with a workspace, avoids both.)  The two teams of
        // a 16 x 16 forward warp keep their own degrees: at most two epilogue paths, and the
        // Frechet kernel, whose teams are whole warps, then repeats the forward's (m, s).
        m = int(__reduce_max_sync(0xffffffffu, unsigned(m)));
      }
    }
    {
      const bool bad_team = scratch[3] != 0;
      nsteps = (valid && !bad_team) ? scheme_products(m) + s : (bad_team ? -1 : 0);
    }
    const bool team_bad = nsteps < 0;
    if (team_bad) nsteps = 0;
    if constexpr (KeysOut && !grouped) {
      // every lane of the team stores the same key (one transaction, no divergent branch)
      if (valid) keys_out[b] = team_bad ? kKeyBad : make_key(m, s);
    }
    const int poly = scheme_products(m);
    const int prog = program_offset(m);
    if constexpr (T <= 32) team_sync<T>(tic);  // every column read is done before tiles are rescaled

    // ---- A / 2^s (the element-wise chunks), identity for the degree-1 polynomial ----
    if (s > 0 || m == 1) {
#pragma unroll 1
      for (int part = 0; part < C::NPART; ++part) {
#pragma unroll
        for (int c = 0; c < TM * TN / 4; ++c) {
          int i, j, o;
          ew_chunk<P, TM, TN, Pair>(c, t, i0, j0, i, j, o);
          float4* p = reinterpret_cast<float4*>(team + part * C::PLANE + o);
          float4 v = *p;
          v.x = scale_pow2(v.x, s);
          v.y = scale_pow2(v.y, s);
          v.z = scale_pow2(v.z, s);
          v.w = scale_pow2(v.w, s);
          if (m == 1 && part == 0) {
            const int dj = i - j;
            v.x += dj == 0 ? 1.f : 0.f;
            v.y += dj == 1 ? 1.f : 0.f;
            v.z += dj == 2 ? 1.f : 0.f;
            v.w += dj == 3 ? 1.f : 0.f;
          }
          *p = v;
        }
      }
    }
    // Multi-warp teams skip this barrier when nothing was rescaled (team-uniform condition).
    if (T <= 32 || s > 0 || m == 1) team_sync<T>(tic);

    // ---- polynomial steps, then squarings ----
    // Whole-warp teams square in ping-pong between slots 0 and 1: the slot written in a
    // squaring step is not read in it, so one barrier per squaring suffices.  Teams that
    // share a warp keep the lockstep two-barrier form.
    constexpr bool kPingPong = T >= 32;
    int max_steps = nsteps;
    if constexpr (T < 32) max_steps = __reduce_max_sync(0xffffffffu, nsteps);
    int cur = 0;  // slot holding the current value during the squarings
    for (int st = 0; st < max_steps; ++st) {
      const bool active = st < nsteps;
      const bool is_poly = st < poly;
      const Step* step = &kSteps[prog + (is_poly ? st : 0)];
      const int xs = is_poly ? step->x : cur;
      const int ys = is_poly ? step->y : cur;
      const int zs = is_poly ? step->z : -1;
      const int rs = is_poly ? step->r : (kPingPong ? 1 - cur : 0);
      Acc<TM, TN, Pair> R;
      if (active) {
        if (zs >= 0) {
          acc_load<P, TM, TN, Pair>(team + zs * C::SLOT, i0, j0, R);
        } else {
          acc_zero(R);
        }
        team_product<P, TM, TN, Pair>(team + xs * C::SLOT, team + ys * C::SLOT, i0, j0, R);
      }
      if (!kPingPong || is_poly) team_sync<T>(tic);
      if (active) {
        if constexpr (feed_product<P, TM, TN, Pair>()) {
          if (is_poly) {
            team_epilogue<P, TM, TN, Pair>(prog + st, team, t, i0, j0, R);
          } else {
            acc_store<P, TM, TN, Pair>(team + rs * C::SLOT, i0, j0, R);
          }
        } else {
          acc_store<P, TM, TN, Pair>(team + rs * C::SLOT, i0, j0, R);
          if (is_poly && step->nout > 0) {
            if constexpr (rowmap_elementwise<P, TM, TN, Pair>()) team_sync<T>(tic);  // other threads' tiles
            team_epilogue<P, TM, TN, Pair>(prog + st, team, t, i0, j0, R);
          }
        }
      }
      team_sync<T>(tic);
      if (!is_poly) cur = rs;
    }

    // ---- the n x n result, 16-byte chunks spread over the team ----
    if (valid) {
      const float* res = team + cur * C::SLOT + (Pair ? C::PLANE : 0);
      const float nanv = __int_as_float(0x7fc00000);
      if (T >= 32 && out_vec && n == P) {
        // Full-size tile: every chunk exists; all shared loads issue before the stores.
        constexpr int RES_PER_THREAD = (P * P / 4 + T - 1) / T;
        float4 v[RES_PER_THREAD];
#pragma unroll
        for (int k = 0; k < RES_PER_THREAD; ++k) {
          const int idx = t + k * T;
          if (idx < P * P / 4) v[k] = *reinterpret_cast<const float4*>(res + pidx<P, TM>(idx / (P / 4), 4 * (idx % (P / 4))));
        }
#pragma unroll
        for (int k = 0; k < RES_PER_THREAD; ++k) {
          const int idx = t + k * T;
          if (idx < P * P / 4) {
            if (team_bad) v[k] = make_float4(nanv, nanv, nanv, nanv);
            store_chunk(out, dtype, b * (P * P) + 4 * idx, v[k]);
          }
        }
      } else {
        store_plane<P, TM, T>(res, out, dtype, b, n, t, out_vec, false, team_bad);
      }
      if (Pair && out2 != nullptr)
        store_plane<P, TM, T>(team + cur * C::SLOT, out2, dtype, b, n, t, (flags & kOut2Vec) != 0,
                              (flags & kOut2T) != 0, team_bad);
    }
    if (t == 0) scratch[3] = 0;  // non-finite flag: every thread read it before the steps
    team_sync<T>(tic);  // the result slot is read before the next matrix is written
  }
}

}  // namespace fhx
