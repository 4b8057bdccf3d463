// Degree classification and grouping for the team kernel whose teams share a warp (5 <= n <= 8:
// eight 4-thread or four 8-thread teams per warp).
//
// Teams in one warp run in lockstep, so a warp costs as much as its most expensive matrix.  On a
// batch of mixed norms (config 3: degrees 4/8/12/18 in about equal shares, 0-4 squarings) that
// is 7.4 product steps per 8 x 8 matrix where the matrices themselves need 4.0.  Before the main
// kernel, two small passes group the batch by cost:
//
//   classify   one thread per matrix: nu = min(||A||_1, ||A||_inf) in float64 (rows and columns
//              each summed in ascending order, so A and A^T give the same bits), (m, s) by
//              choose_degree, a 16-bit key per matrix, and a histogram of key bins;
//   scatter    the bin starts (every CTA scans the histogram itself) and every matrix's index
//              into its bin's range of a permutation.
//
// The main kernel then takes its matrices in permutation order and each team runs its matrix's
// own (m, s) from the key: a matrix's result depends on that matrix alone (no degree shared with
// neighbours), and the Frechet backward on A^T repeats the forward's (m, s) exactly.  The order
// inside a bin (from shared-memory atomics) varies from run to run; it only decides which team
// computes which matrix, never a result.
//
// Workspace (caller-allocated, fhx_workspace_bytes): keys (2 B per matrix), permutation (4 B per
// matrix), histogram and bin cursors (kSortBins words each, adjacent: zeroed by one memset before
// the classify pass).
#pragma once

#include "expm_common.cuh"

namespace fhx {

constexpr int kSortThreads = 256;
constexpr int kKeySMax = 31;                       // squarings beyond this share one bin
constexpr int kSortBins = 6 * (kKeySMax + 1) + 1;  // (degree, s) bins + one for non-finite
constexpr unsigned short kKeyBad = 0xffffu;        // a non-finite entry

// key: bits 0-2 degree index, bits 3-15 squarings (s <= 8191 covers every float32 input)
__host__ __device__ __forceinline__ unsigned short make_key(int m, int s) {
  return static_cast<unsigned short>(degree_index(m) | (s << 3));
}
__device__ __forceinline__ int key_bin(unsigned short key) {
  if (key == kKeyBad) return kSortBins - 1;
  const int s = key >> 3;
  return (key & 7) * (kKeySMax + 1) + (s < kKeySMax ? s : kKeySMax);
}

struct SortWorkspace {
  unsigned short* keys;
  int* perm;
  unsigned* hist;
  unsigned* cursor;
};

__host__ __device__ constexpr size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

__host__ __device__ constexpr size_t sort_workspace_bytes(int64_t batch) {
  return align256(size_t(batch) * 2) + align256(size_t(batch) * 4) + 2 * align256(kSortBins * 4);
}

__host__ __forceinline__ SortWorkspace sort_workspace(void* base, int64_t batch) {
  char* p = static_cast<char*>(base);
  SortWorkspace w;
  w.keys = reinterpret_cast<unsigned short*>(p);
  p += align256(size_t(batch) * 2);
  w.perm = reinterpret_cast<int*>(p);
  p += align256(size_t(batch) * 4);
  w.hist = reinterpret_cast<unsigned*>(p);
  p += align256(kSortBins * 4);
  w.cursor = reinterpret_cast<unsigned*>(p);
  return w;
}

// Block-level histogram of the bins in `bin` (-1: no matrix), added to the global one.
__device__ __forceinline__ void add_block_histogram(int bin, unsigned* __restrict__ hist, unsigned* s_cnt) {
  for (int i = threadIdx.x; i < kSortBins; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  if (bin >= 0) atomicAdd(&s_cnt[bin], 1u);
  __syncthreads();
  for (int i = threadIdx.x; i < kSortBins; i += blockDim.x)
    if (s_cnt[i]) atomicAdd(&hist[i], s_cnt[i]);
}

// Four consecutive elements of a matrix along its contiguous dimension, as floats.
__device__ __forceinline__ float4 load_vec4(const View& v, int dtype, int64_t off) {
  if (dtype == kF32) return ld_f32x4(static_cast<const float*>(v.data) + off);
  const uint2 h = ld_u32x2(reinterpret_cast<const unsigned*>(static_cast<const unsigned short*>(v.data) + off));
  auto dec = [&](unsigned w) {
    const unsigned short u = static_cast<unsigned short>(w);
    return dtype == kBF16 ? __bfloat162float(__ushort_as_bfloat16(u)) : __half2float(__ushort_as_half(u));
  };
  return make_float4(dec(h.x & 0xffffu), dec(h.x >> 16), dec(h.y & 0xffffu), dec(h.y >> 16));
}

// Classification flags: bit 0 = rows are the contiguous dimension (else columns), bit 1 = the
// contiguous dimension moves in aligned 4-element vectors (n % 4 == 0).
enum : unsigned { kClsRows = 1u, kClsVec = 2u };

// The key of a matrix from its float64 line sums |a| (rows[i], columns[j]) and whether an entry
// was non-finite.
template <int P>
__device__ __forceinline__ unsigned short key_of_sums(const double (&row)[P], const double (&col)[P], bool bad) {
  double nrow = 0.0, ncol = 0.0;
#pragma unroll
  for (int t = 0; t < P; ++t) {
    nrow = fmax(nrow, row[t]);
    ncol = fmax(ncol, col[t]);
  }
  if (bad) return kKeyBad;
  int m, s;
  choose_degree(fmin(nrow, ncol), &m, &s);
  return make_key(m, s);
}

// The key of a full P x P matrix given as its 16-byte chunks along the contiguous dimension:
// x[o][q / 4] = elements q..q+3 of line o (a row if `rows`, else a column).  Row sums accumulate
// over ascending columns and column sums over ascending rows.
template <int P>
__device__ __forceinline__ unsigned short key_of_matrix(const float4 (&x)[P][P / 4], bool rows) {
  double row[P], col[P];
#pragma unroll
  for (int t = 0; t < P; ++t) row[t] = col[t] = 0.0;
  bool bad = false;
#pragma unroll
  for (int o = 0; o < P; ++o) {
#pragma unroll
    for (int q = 0; q < P; q += 4) {
      const float xs[4] = {x[o][q / 4].x, x[o][q / 4].y, x[o][q / 4].z, x[o][q / 4].w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = rows ? o : q + u, j = rows ? q + u : o;
        bad |= !isfinite(xs[u]);
        const double av = fabs(double(xs[u]));
        row[i] += av;
        col[j] += av;
      }
    }
  }
  return key_of_sums<P>(row, col, bad);
}

// One thread per matrix of a strided [batch, n, n] view (P bounds n).  Row sums
// accumulate over ascending columns and column sums over ascending rows whatever the loop
// order, so the float64 norms of A and A^T are bit-identical.
template <int P>
__global__ void __launch_bounds__(kSortThreads) classify_kernel(View a, int64_t batch, int n, int dtype,
                                                                unsigned flags, SortWorkspace ws) {
  __shared__ unsigned s_cnt[kSortBins];
  const int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  int bin = -1;
  if (b < batch) {
    const int64_t base = b * a.s0;
    const bool rows = flags & kClsRows;
    unsigned short key;
    if ((flags & kClsVec) && n == P) {
      // whole matrix: every vector load issued before the first sum
      float4 x[P][P / 4];
#pragma unroll
      for (int o = 0; o < P; ++o)
#pragma unroll
        for (int q = 0; q < P; q += 4)
          x[o][q / 4] = load_vec4(a, dtype, rows ? base + o * a.s1 + q * a.s2 : base + q * a.s1 + o * a.s2);
      key = key_of_matrix<P>(x, rows);
    } else {
      double row[P], col[P];
#pragma unroll
      for (int t = 0; t < P; ++t) row[t] = col[t] = 0.0;
      bool bad = false;
      auto add = [&](int i, int j, float v) {
        bad |= !isfinite(v);
        const double av = fabs(double(v));
        row[i] += av;
        col[j] += av;
      };
      if (flags & kClsVec) {
        // along the contiguous dimension in 4-element vectors (n % 4 == 0)
#pragma unroll
        for (int o = 0; o < P; ++o) {
#pragma unroll
          for (int q = 0; q < P; q += 4) {
            if (o < n && q < n) {
              const int64_t off = rows ? base + o * a.s1 + q * a.s2 : base + q * a.s1 + o * a.s2;
              const float4 x = load_vec4(a, dtype, off);
              const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                if (rows) add(o, q + u, xs[u]);
                else add(q + u, o, xs[u]);
              }
            }
          }
        }
      } else {
#pragma unroll
        for (int o = 0; o < P; ++o)
#pragma unroll
          for (int q = 0; q < P; ++q)
            if (o < n && q < n) {
              // (the sign of a negated view does not change |a|)
              if (rows) add(o, q, load_elem(a.data, dtype, base + o * a.s1 + q * a.s2));
              else add(q, o, load_elem(a.data, dtype, base + q * a.s1 + o * a.s2));
            }
      }
      key = key_of_sums<P>(row, col, bad);
    }
    ws.keys[b] = key;
    bin = key_bin(key);
  }
  add_block_histogram(bin, ws.hist, s_cnt);
}

// classify_kernel<8> for a dense float32 batch: matrix b is the 64 floats at a + 64 b, rows or
// columns contiguous (flags).  One thread per matrix reading its own 256 bytes makes every warp
// load touch 32 cache lines, which left the general kernel waiting on L1 (about 2.7 TB/s).  Here
// each warp first copies its 32 matrices (8 KB) into shared memory with fully coalesced 16-byte
// loads, each matrix padded by 16 bytes so that the 32 threads then read their own matrices
// without bank conflicts; the sums and keys are those of classify_kernel's whole-matrix path.
constexpr int kDenseThreads = 128;
constexpr int kDenseStride = 68;  // floats per matrix in shared memory (64 + 4 of padding)

__global__ void __launch_bounds__(kDenseThreads, 5) classify_dense8_kernel(const float* __restrict__ a, int64_t batch,
                                                                        unsigned flags, SortWorkspace ws) {
  __shared__ __align__(16) float s_m[kDenseThreads * kDenseStride];
  __shared__ unsigned s_cnt[kSortBins];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kSortBins; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  float* sw = s_m + warp * 32 * kDenseStride;
  // Tiles of kDenseThreads matrices, grid-strided: one histogram flush per CTA, not per tile.
  for (int64_t tile = blockIdx.x; tile * kDenseThreads < batch; tile += gridDim.x) {
    const int64_t first = tile * kDenseThreads + warp * 32;  // the warp's first matrix
    float4 v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int g = k * 32 + lane;  // chunk g of the warp's 512: matrix g / 16, chunk g % 16
      v[k] = first + (g >> 4) < batch ? ld_f32x4(a + (first + (g >> 4)) * 64 + 4 * (g & 15))
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncwarp();  // the previous tile's reads of this warp's region are done
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int g = k * 32 + lane;
      *reinterpret_cast<float4*>(sw + (g >> 4) * kDenseStride + 4 * (g & 15)) = v[k];
    }
    __syncwarp();
    const int64_t b = first + lane;
    if (b < batch) {
      float4 x[8][2];
#pragma unroll
      for (int o = 0; o < 8; ++o)
#pragma unroll
        for (int q = 0; q < 2; ++q)
          x[o][q] = *reinterpret_cast<const float4*>(sw + lane * kDenseStride + 8 * o + 4 * q);
      const unsigned short key = key_of_matrix<8>(x, (flags & kClsRows) != 0);
      ws.keys[b] = key;
      atomicAdd(&s_cnt[key_bin(key)], 1u);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kSortBins; i += blockDim.x)
    if (s_cnt[i]) atomicAdd(&ws.hist[i], s_cnt[i]);
}

// Exclusive prefix sum of the kSortBins histogram counts into s_start, by every CTA of the scatter
// pass for itself (a few hundred words; warp-shuffle scans, then the warp totals).
__device__ __forceinline__ void bin_starts(const unsigned* __restrict__ hist, unsigned* s_start, unsigned* s_warp) {
  static_assert(kSortBins <= kSortThreads, "one bin per thread");
  const int i = threadIdx.x, lane = i & 31, warp = i >> 5;
  const unsigned c = i < kSortBins ? hist[i] : 0u;
  unsigned v = c;  // inclusive scan within the warp
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const unsigned o = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += o;
  }
  if (lane == 31) s_warp[warp] = v;
  __syncthreads();
  if (warp == 0) {
    unsigned w = lane < kSortThreads / 32 ? s_warp[lane] : 0u;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const unsigned o = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += o;
    }
    if (lane < kSortThreads / 32) s_warp[lane] = w;  // inclusive totals of warps 0..lane
  }
  __syncthreads();
  if (i < kSortBins) s_start[i] = v - c + (warp > 0 ? s_warp[warp - 1] : 0u);
}

// perm[start(bin) + rank] = b: a CTA reserves one range per bin with a global atomic on the bin's
// cursor (zero on entry) and hands out ranks inside it with shared-memory atomics.
__global__ void __launch_bounds__(kSortThreads) scatter_kernel(int64_t batch, SortWorkspace ws) {
  __shared__ unsigned s_cnt[kSortBins];
  __shared__ unsigned s_base[kSortBins];
  __shared__ unsigned s_warp[kSortThreads / 32];
  const int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int i = threadIdx.x; i < kSortBins; i += blockDim.x) s_cnt[i] = 0;
  bin_starts(ws.hist, s_base, s_warp);  // (its barriers also order the zeroing above)
  int bin = -1;
  unsigned local = 0;
  if (b < batch) {
    bin = key_bin(ws.keys[b]);
    local = atomicAdd(&s_cnt[bin], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kSortBins; i += blockDim.x)
    if (s_cnt[i]) s_base[i] += atomicAdd(&ws.cursor[i], s_cnt[i]);
  __syncthreads();
  if (bin >= 0) ws.perm[s_base[bin] + local] = int(b);
}

}  // namespace fhx
