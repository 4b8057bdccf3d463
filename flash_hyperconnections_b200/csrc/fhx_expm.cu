// C ABI of the batched small-matrix exponential: argument checks, kernel selection and
// launch geometry.  Declarations and status codes: include/fhx.h.
//
// Reference counterpart: the host launcher small_matrix_exp_cuda (csrc/matrix_exp.cu:51-78)
// with launch_small_matrix_exp (:13-33).  There, every call first materialises a
// contiguous FP32 copy of the input (and of the direction), zero-padded to 4/8/16/32, and
// un-pads the output with another copy; here the kernels read any strided view in the I/O
// dtype directly and write the n x n output once.
#include <cstdint>
#include <atomic>
#include <mutex>

#include "expm_common.cuh"
#include "expm_reg.cuh"
#include "expm_team.cuh"
#include "fhx.h"

#ifndef FHX_FRECHET32_TILE
#define FHX_FRECHET32_TILE 2
#endif
#ifndef FHX_FORWARD32_TILE
#define FHX_FORWARD32_TILE 44
#endif
#ifndef FHX_DENSE_CTAS_PER_SM
#define FHX_DENSE_CTAS_PER_SM 5
#endif
#ifndef FHX_FRECHET8_TILE
#define FHX_FRECHET8_TILE 24
#endif

namespace fhx {

thread_local cudaError_t g_last_cuda_error = cudaSuccess;

std::atomic<unsigned long long> g_launches{0};

void note_launches(int count) { g_launches.fetch_add(static_cast<unsigned long long>(count), std::memory_order_relaxed); }

int cuda_status(cudaError_t err) {
  if (err == cudaSuccess) return FHX_OK;
  g_last_cuda_error = err;
  return FHX_ERR_CUDA;
}

namespace {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  bool ready = false;
  int sms = 0;
};

std::mutex g_mutex;
DeviceInfo g_devices[kMaxDevices];


// Per-(kernel, device) launch geometry: resident CTAs per SM at the kernel's smem size.
struct LaunchShape {
  bool ready[kMaxDevices] = {};
  int blocks_per_sm[kMaxDevices] = {};
};

int device_sms(int dev) {
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceInfo& d = g_devices[dev];
  if (!d.ready) {
    if (cuda_status(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != FHX_OK) return -1;
    d.ready = true;
  }
  return d.sms;
}

template <typename Kernel>
int resident_blocks(Kernel kernel, LaunchShape& shape, int dev, int threads, size_t smem) {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!shape.ready[dev]) {
    if (smem > 48 * 1024 &&
        cuda_status(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem))) != FHX_OK)
      return -1;
    int blocks = 0;
    if (cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, threads, smem)) != FHX_OK)
      return -1;
    shape.blocks_per_sm[dev] = blocks > 0 ? blocks : 1;
    shape.ready[dev] = true;
  }
  return shape.blocks_per_sm[dev];
}

bool aligned(const void* p, size_t bytes) { return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0; }

template <int N, bool Pair>
int launch_reg(const View& a, const View& e, void* out, void* out2, bool out2_t, int64_t batch, int dtype,
               cudaStream_t stream) {
  constexpr int threads = kRegThreads;
  const int64_t blocks = (batch + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return FHX_ERR_SIZE;
  // 4 x 4: rows with unit inner stride, 4-element-aligned row and matrix strides and an aligned
  // base are read as one vector each; the contiguous output is written the same way.
  const size_t row_bytes = dtype == kF32 ? 16 : 8;
  auto rows = [&](const View& v) {
    return N == 4 && v.s2 == 1 && v.s1 % 4 == 0 && v.s0 % 4 == 0 && aligned(v.data, row_bytes);
  };
  unsigned flags = 0;
  if (rows(a)) flags |= 1u;
  if (Pair && rows(e)) flags |= 2u;
  if (N == 4 && aligned(out, row_bytes)) flags |= 4u;
  if (out2_t) flags |= 8u;
  if (N == 4 && out2 != nullptr && aligned(out2, row_bytes)) flags |= 16u;
  expm_reg_kernel<N, Pair><<<unsigned(blocks), threads, 0, stream>>>(a, e, out, out2, batch, dtype, flags);
  note_launches(1);
  return cuda_status(cudaGetLastError());
}

// Load/store layout flags of the team kernel (see the enum in expm_team.cuh).
template <int P>
unsigned layout_flags(const View& a, const View& e, const void* out, const void* out2, bool out2_t, int n, int dtype,
                      bool pair) {
  unsigned f = 0;
  // Row chunks when the elements of a row are closest in memory, else column chunks; a chunk
  // is one 128-bit (float32) or 64-bit (half types) load when it is contiguous, aligned and
  // n == P.
  auto rows = [](const View& v) { return v.s2 <= v.s1; };
  auto vec = [&](const View& v) {
    const int64_t inner = rows(v) ? v.s2 : v.s1;
    const int64_t outer = rows(v) ? v.s1 : v.s2;
    return n == P && inner == 1 && outer % 4 == 0 && v.s0 % 4 == 0 && aligned(v.data, dtype == kF32 ? 16 : 8);
  };
  if (rows(a)) f |= kARows;
  if (vec(a)) f |= kAVec;
  if (pair) {
    if (rows(e)) f |= kERows;
    if (vec(e)) f |= kEVec;
  }
  const size_t esz = dtype == kF32 ? 4 : 2;
  if (n % 4 == 0 && aligned(out, 4 * esz)) f |= kOutVec;
  if (out2 != nullptr && n % 4 == 0 && aligned(out2, 4 * esz)) f |= kOut2Vec;
  if (out2_t) f |= kOut2T;
  return f;
}

// TM x TN: a thread's register tile; WARPS: warps per CTA.  A team is (P/TM) * (P/TN)
// threads; one CTA holds WARPS * 32 / team-size teams.
template <int P, int TM, int TN, bool Pair, int WARPS, bool Grouped, bool KeysOut = false>
int launch_team_kernel(const View& a, const View& e, void* out, void* out2, bool out2_t, int64_t batch, int n,
                       int dtype, cudaStream_t stream, const int* perm, const unsigned short* keys,
                       unsigned short* keys_out) {
  using C = TeamCfg<P, TM, TN, Pair>;
  constexpr int threads = WARPS * 32;
  constexpr int teams = threads / C::T;
  constexpr size_t smem = size_t(teams) * C::TEAM_FLOATS * sizeof(float);
  static LaunchShape shape;
  auto kernel = expm_team_kernel<P, TM, TN, Pair, WARPS, Grouped, KeysOut>;
  int dev = 0;
  const int st = cuda_status(cudaGetDevice(&dev));
  if (st != FHX_OK) return st;
  if (dev < 0 || dev >= kMaxDevices) return FHX_ERR_CUDA;
  const int sms = device_sms(dev);
  const int per_sm = resident_blocks(kernel, shape, dev, threads, smem);
  if (sms <= 0 || per_sm <= 0) return FHX_ERR_CUDA;
  const int64_t items = (batch + teams - 1) / teams;
  const int64_t resident = int64_t(sms) * per_sm;
  const int blocks = int(items < resident ? items : resident);
  kernel<<<blocks, threads, smem, stream>>>(a, e, out, out2, perm, keys, keys_out, batch, n, dtype,
                                            layout_flags<P>(a, e, out, out2, out2_t, n, dtype, Pair));
  note_launches(1);
  return cuda_status(cudaGetLastError());
}

// grouped (may be null): the keys of every matrix, with the permutation of group_by_degree
// (P = 8) or without one (the 16 x 16 Frechet kernel: keyed mode, the keys a forward launch
// stored); keys_out (may be null; the 16 x 16 forward only): store every matrix's key there.
template <int P, int TM, int TN, bool Pair, int WARPS>
int launch_team(const View& a, const View& e, void* out, void* out2, bool out2_t, int64_t batch, int n, int dtype,
                cudaStream_t stream, const SortWorkspace* grouped = nullptr, unsigned short* keys_out = nullptr) {
  if constexpr (P == 8 || (P == 16 && Pair)) {
    if (grouped != nullptr)
      return launch_team_kernel<P, TM, TN, Pair, WARPS, true>(a, e, out, out2, out2_t, batch, n, dtype, stream,
                                                              grouped->perm, grouped->keys, nullptr);
  }
  if constexpr (P == 16 && !Pair) {
    if (keys_out != nullptr)
      return launch_team_kernel<P, TM, TN, Pair, WARPS, false, true>(a, e, out, out2, out2_t, batch, n, dtype, stream,
                                                                     nullptr, nullptr, keys_out);
  }
  return launch_team_kernel<P, TM, TN, Pair, WARPS, false>(a, e, out, out2, out2_t, batch, n, dtype, stream, nullptr,
                                                           nullptr, nullptr);
}

// Grouping passes of expm_sort.cuh on the view `a` (5 <= n <= 8): keys, histogram and permutation in
// the caller's workspace.
template <int P>
int group_by_degree(const View& a, int64_t batch, int n, int dtype, void* workspace, cudaStream_t stream,
                    SortWorkspace* out) {
  const SortWorkspace w = sort_workspace(workspace, batch);
  // histogram and bin cursors (adjacent) to zero
  int st = cuda_status(cudaMemsetAsync(w.hist, 0, 2 * align256(kSortBins * sizeof(unsigned)), stream));
  if (st != FHX_OK) return st;
  // the contiguous dimension of the view, and whether it moves in aligned 4-element vectors
  const bool rows = a.s2 == 1 || (a.s1 != 1 && a.s2 <= a.s1);
  const int64_t outer = rows ? a.s1 : a.s2;
  const int64_t inner = rows ? a.s2 : a.s1;
  unsigned flags = rows ? kClsRows : 0u;
  if (n % 4 == 0 && inner == 1 && outer % 4 == 0 && a.s0 % 4 == 0 && aligned(a.data, dtype == kF32 ? 16 : 8))
    flags |= kClsVec;
  const int64_t blocks = (batch + kSortThreads - 1) / kSortThreads;
  if (blocks > 0x7fffffffLL) return FHX_ERR_SIZE;
  // dense float32 8 x 8 batch (rows or columns contiguous): the coalesced classification
  const bool dense8 = P == 8 && n == 8 && dtype == kF32 && a.s0 == 64 &&
                      ((a.s1 == 8 && a.s2 == 1) || (a.s1 == 1 && a.s2 == 8)) && aligned(a.data, 16);
  if (dense8) {
    // at most FHX_DENSE_CTAS_PER_SM resident CTAs per SM, each looping over tiles
    int dev = 0;
    st = cuda_status(cudaGetDevice(&dev));
    if (st != FHX_OK) return st;
    if (dev < 0 || dev >= kMaxDevices) return FHX_ERR_CUDA;
    const int64_t tiles = (batch + kDenseThreads - 1) / kDenseThreads;
    const int64_t cap = int64_t(device_sms(dev)) * FHX_DENSE_CTAS_PER_SM;
    if (cap <= 0) return FHX_ERR_CUDA;
    const int64_t dblocks = tiles < cap ? tiles : cap;
    classify_dense8_kernel<<<unsigned(dblocks), kDenseThreads, 0, stream>>>(static_cast<const float*>(a.data), batch,
                                                                             flags, w);
  } else {
    classify_kernel<P><<<unsigned(blocks), kSortThreads, 0, stream>>>(a, batch, n, dtype, flags, w);
  }
  scatter_kernel<<<unsigned(blocks), kSortThreads, 0, stream>>>(batch, w);
  note_launches(2);
  st = cuda_status(cudaGetLastError());
  if (st != FHX_OK) return st;
  *out = w;
  return FHX_OK;
}

// Sizes whose teams share a warp with a shared degree unless grouped: the 8 x 8 kernels.
bool grouped_size(int n) { return n >= 5 && n <= 8; }

// out2 (Frechet launches only, may be null): also write exp(A) there, transposed if out2_t.
// workspace (may be null): for 5 <= n <= 8, group the batch by degree first (expm_sort.cuh);
// with reuse_grouping, the workspace already holds that grouping (from a launch on the same
// matrices or their transposes) and the grouping passes are skipped.
template <bool Pair>
int dispatch(const View& a, const View& e, void* out, int64_t batch, int n, int dtype, cudaStream_t stream,
             void* out2 = nullptr, bool out2_t = false, void* workspace = nullptr, bool reuse_grouping = false) {
  switch (n) {
    case 2: return launch_reg<2, Pair>(a, e, out, out2, out2_t, batch, dtype, stream);
    case 3: return launch_reg<3, Pair>(a, e, out, out2, out2_t, batch, dtype, stream);
    case 4: return launch_reg<4, Pair>(a, e, out, out2, out2_t, batch, dtype, stream);
    default: break;
  }
  // Tile shapes (TM x TN per thread) and warps per team, chosen by measurement on B200:
  // more warps per SM beat larger per-thread tiles as long as the shared-memory wavefront
  // budget holds.  32 x 32: forward 4 x 4 tiles in two-warp teams (16 warps per SM at 128
  // registers), Frechet 2 x 4 tiles in four-warp teams (20 warps per SM at 40 KB of shared
  // state per matrix).  8 x 8: 4 x 4 tiles, eight teams per warp; the grouped Frechet (with a
  // workspace) 2 x 4 tiles, four teams per warp (128 registers and 16 warps per SM, 12 % faster
  // than 4 x 4 tiles at 228 registers and 8 warps; without a workspace the eight matrices of a
  // warp share one degree, so that kernel keeps the forward's eight teams).  16 x 16: forward 4 x 4 tiles,
  // two teams per warp; Frechet 2 x 4 tiles, one team per warp (20 % faster than 4 x 4 tiles,
  // whose 254 registers left 8 warps per SM).
  SortWorkspace ws{};
  const SortWorkspace* grouped = nullptr;
  unsigned short* keys_out = nullptr;
  if (workspace != nullptr && grouped_size(n)) {
    if (reuse_grouping) {
      ws = sort_workspace(workspace, batch);
    } else {
      const int st = group_by_degree<8>(a, batch, n, dtype, workspace, stream, &ws);
      if (st != FHX_OK) return st;
    }
    grouped = &ws;
  } else if (workspace != nullptr && n > 8 && n <= 16) {
    // 9 <= n <= 16: the workspace holds one key per matrix; the forward stores them and the
    // Frechet launch of fhx_frechet_grouped reads them (keyed mode, no norm phase: measured
    // 5.6 % off the 16 x 16 Frechet kernel, against 3.7 % more for the forward that stores them;
    // at 32 x 32 the keyed kernel measured no faster, so 17 <= n <= 32 keeps its norm phase)
    if (Pair && reuse_grouping) {
      ws.keys = static_cast<unsigned short*>(workspace);
      ws.perm = nullptr;
      grouped = &ws;
    } else if (!Pair) {
      keys_out = static_cast<unsigned short*>(workspace);
    }
  }
#if FHX_FRECHET8_TILE == 24
  if constexpr (Pair) {
    if (n <= 8 && grouped != nullptr)
      return launch_team<8, 2, 4, true, 1>(a, e, out, out2, out2_t, batch, n, dtype, stream, grouped);
  }
#endif
  if (n <= 8) return launch_team<8, 4, 4, Pair, 1>(a, e, out, out2, out2_t, batch, n, dtype, stream, grouped);
  if (n <= 16) {
    if constexpr (Pair) {
      return launch_team<16, 2, 4, true, 1>(a, e, out, out2, out2_t, batch, n, dtype, stream, grouped);
    } else {
      return launch_team<16, 4, 4, false, 1>(a, e, out, out2, out2_t, batch, n, dtype, stream, nullptr, keys_out);
    }
  }
  if constexpr (Pair) {
#if FHX_FRECHET32_TILE == 4
    return launch_team<32, 4, 4, true, 2>(a, e, out, out2, out2_t, batch, n, dtype, stream, grouped);
#elif FHX_FRECHET32_TILE == 28
    return launch_team<32, 2, 8, true, 2>(a, e, out, out2, out2_t, batch, n, dtype, stream, grouped);
#else
    return launch_team<32, 2, 4, true, 4>(a, e, out, out2, out2_t, batch, n, dtype, stream, grouped);
#endif
  } else {
#if FHX_FORWARD32_TILE == 48
    return launch_team<32, 4, 8, false, 1>(a, e, out, out2, out2_t, batch, n, dtype, stream, nullptr, keys_out);
#elif FHX_FORWARD32_TILE == 84
    return launch_team<32, 8, 4, false, 1>(a, e, out, out2, out2_t, batch, n, dtype, stream, nullptr, keys_out);
#else
    return launch_team<32, 4, 4, false, 2>(a, e, out, out2, out2_t, batch, n, dtype, stream, nullptr, keys_out);
#endif
  }
}

int check_common(int64_t batch, int32_t n, int32_t dtype, const void* out) {
  if (n < 2 || n > FHX_MAX_N || batch < 0) return FHX_ERR_SIZE;
  if (dtype != FHX_DTYPE_F32 && dtype != FHX_DTYPE_BF16 && dtype != FHX_DTYPE_F16) return FHX_ERR_DTYPE;
  if (batch > 0 && out == nullptr) return FHX_ERR_POINTER;
  return FHX_OK;
}

int check_view(const void* p, int64_t s0, int64_t s1, int64_t s2, int64_t batch) {
  if (batch > 0 && p == nullptr) return FHX_ERR_POINTER;
  if (s0 < 0 || s1 < 0 || s2 < 0) return FHX_ERR_STRIDE;
  return FHX_OK;
}

// ---- scratch of fhx_matrix_exp_noalloc ----
// Some callers cannot allocate device memory at all (see include/fhx.h); for them the grouping
// workspace of the 5 <= n <= 8 path lives in this file-scope array, sized for
// FHX_NOALLOC_MAX_BATCH matrices (about 6 MiB, held by every GPU that loads the library until
// the process exits).  In host code the name is only a host-side stand-in for the symbol; the
// device address comes from cudaGetSymbolAddress, once per device, with that device current.
constexpr size_t kNoAllocScratchBytes = sort_workspace_bytes(FHX_NOALLOC_MAX_BATCH);

struct NoAllocScratch {
  bool ready[kMaxDevices] = {};
  void* ptr[kMaxDevices] = {};
};
NoAllocScratch g_noalloc;

}  // namespace
}  // namespace fhx

static __device__ __align__(256) unsigned char g_noalloc_scratch[fhx::kNoAllocScratchBytes];

namespace fhx {
namespace {

// Device address of g_noalloc_scratch on the current device (looked up on the first call there).
int noalloc_scratch(void** out) {
  int dev = 0;
  int st = cuda_status(cudaGetDevice(&dev));
  if (st != FHX_OK) return st;
  if (dev < 0 || dev >= kMaxDevices) return FHX_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_noalloc.ready[dev]) {
    void* p = nullptr;
    st = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    if (st != FHX_OK) return st;
    g_noalloc.ptr[dev] = p;
    g_noalloc.ready[dev] = true;
  }
  *out = g_noalloc.ptr[dev];
  return FHX_OK;
}

}  // namespace
}  // namespace fhx

extern "C" {

int32_t fhx_matrix_exp(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                       void* output, int64_t batch, int32_t n, int32_t dtype, void* stream) {
  using namespace fhx;
  int st = check_common(batch, n, dtype, output);
  if (st != FHX_OK) return st;
  st = check_view(input, in_s0, in_s1, in_s2, batch);
  if (st != FHX_OK) return st;
  if (batch == 0) return FHX_OK;
  const View a{input, in_s0, in_s1, in_s2, in_negate ? -1.f : 1.f};
  const View none{nullptr, 0, 0, 0, 1.f};
  return dispatch<false>(a, none, output, batch, n, dtype, static_cast<cudaStream_t>(stream));
}

int32_t fhx_frechet(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                    const void* direction, int64_t dir_s0, int64_t dir_s1, int64_t dir_s2, int32_t dir_negate,
                    void* output, int64_t batch, int32_t n, int32_t dtype, void* stream) {
  using namespace fhx;
  int st = check_common(batch, n, dtype, output);
  if (st != FHX_OK) return st;
  st = check_view(input, in_s0, in_s1, in_s2, batch);
  if (st != FHX_OK) return st;
  st = check_view(direction, dir_s0, dir_s1, dir_s2, batch);
  if (st != FHX_OK) return st;
  if (batch == 0) return FHX_OK;
  const View a{input, in_s0, in_s1, in_s2, in_negate ? -1.f : 1.f};
  const View e{direction, dir_s0, dir_s1, dir_s2, dir_negate ? -1.f : 1.f};
  return dispatch<true>(a, e, output, batch, n, dtype, static_cast<cudaStream_t>(stream));
}

size_t fhx_workspace_bytes(int64_t batch, int32_t n) {
  if (batch <= 0 || n < 5 || n > 16) return 0;
  if (fhx::grouped_size(n)) return fhx::sort_workspace_bytes(batch);
  return fhx::align256(size_t(batch) * sizeof(unsigned short));  // one key per matrix
}

int32_t fhx_matrix_exp_ws(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                          void* output, int64_t batch, int32_t n, int32_t dtype, void* workspace,
                          size_t workspace_bytes, void* stream) {
  using namespace fhx;
  int st = check_common(batch, n, dtype, output);
  if (st != FHX_OK) return st;
  st = check_view(input, in_s0, in_s1, in_s2, batch);
  if (st != FHX_OK) return st;
  if (batch == 0) return FHX_OK;
  if (workspace_bytes < fhx_workspace_bytes(batch, n) || (workspace == nullptr && workspace_bytes > 0))
    return FHX_ERR_WORKSPACE;
  const View a{input, in_s0, in_s1, in_s2, in_negate ? -1.f : 1.f};
  const View none{nullptr, 0, 0, 0, 1.f};
  return dispatch<false>(a, none, output, batch, n, dtype, static_cast<cudaStream_t>(stream), nullptr, false,
                         fhx_workspace_bytes(batch, n) ? workspace : nullptr);
}

int32_t fhx_frechet_ws(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                       const void* direction, int64_t dir_s0, int64_t dir_s1, int64_t dir_s2, int32_t dir_negate,
                       void* output, int64_t batch, int32_t n, int32_t dtype, void* workspace, size_t workspace_bytes,
                       void* stream) {
  using namespace fhx;
  int st = check_common(batch, n, dtype, output);
  if (st != FHX_OK) return st;
  st = check_view(input, in_s0, in_s1, in_s2, batch);
  if (st != FHX_OK) return st;
  st = check_view(direction, dir_s0, dir_s1, dir_s2, batch);
  if (st != FHX_OK) return st;
  if (batch == 0) return FHX_OK;
  if (workspace_bytes < fhx_workspace_bytes(batch, n) || (workspace == nullptr && workspace_bytes > 0))
    return FHX_ERR_WORKSPACE;
  const View a{input, in_s0, in_s1, in_s2, in_negate ? -1.f : 1.f};
  const View e{direction, dir_s0, dir_s1, dir_s2, dir_negate ? -1.f : 1.f};
  return dispatch<true>(a, e, output, batch, n, dtype, static_cast<cudaStream_t>(stream), nullptr, false,
                        fhx_workspace_bytes(batch, n) ? workspace : nullptr);
}

int32_t fhx_frechet_grouped(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                            const void* direction, int64_t dir_s0, int64_t dir_s1, int64_t dir_s2,
                            int32_t dir_negate, void* output, int64_t batch, int32_t n, int32_t dtype,
                            const void* workspace, size_t workspace_bytes, void* stream) {
  using namespace fhx;
  int st = check_common(batch, n, dtype, output);
  if (st != FHX_OK) return st;
  st = check_view(input, in_s0, in_s1, in_s2, batch);
  if (st != FHX_OK) return st;
  st = check_view(direction, dir_s0, dir_s1, dir_s2, batch);
  if (st != FHX_OK) return st;
  if (batch == 0) return FHX_OK;
  if (workspace_bytes < fhx_workspace_bytes(batch, n) || (workspace == nullptr && workspace_bytes > 0))
    return FHX_ERR_WORKSPACE;
  const View a{input, in_s0, in_s1, in_s2, in_negate ? -1.f : 1.f};
  const View e{direction, dir_s0, dir_s1, dir_s2, dir_negate ? -1.f : 1.f};
  // the kernels only read the grouping (keys and permutation) of a reused workspace
  return dispatch<true>(a, e, output, batch, n, dtype, static_cast<cudaStream_t>(stream), nullptr, false,
                        fhx_workspace_bytes(batch, n) ? const_cast<void*>(workspace) : nullptr, true);
}

int32_t fhx_matrix_exp_frechet(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                               const void* direction, int64_t dir_s0, int64_t dir_s1, int64_t dir_s2,
                               int32_t dir_negate, void* exp_output, int32_t exp_transposed, void* frechet_output,
                               int64_t batch, int32_t n, int32_t dtype, void* workspace, size_t workspace_bytes,
                               void* stream) {
  using namespace fhx;
  int st = check_common(batch, n, dtype, frechet_output);
  if (st != FHX_OK) return st;
  if (batch > 0 && exp_output == nullptr) return FHX_ERR_POINTER;
  st = check_view(input, in_s0, in_s1, in_s2, batch);
  if (st != FHX_OK) return st;
  st = check_view(direction, dir_s0, dir_s1, dir_s2, batch);
  if (st != FHX_OK) return st;
  if (batch == 0) return FHX_OK;
  if (workspace != nullptr && workspace_bytes < fhx_workspace_bytes(batch, n)) return FHX_ERR_WORKSPACE;
  const View a{input, in_s0, in_s1, in_s2, in_negate ? -1.f : 1.f};
  const View e{direction, dir_s0, dir_s1, dir_s2, dir_negate ? -1.f : 1.f};
  return dispatch<true>(a, e, frechet_output, batch, n, dtype, static_cast<cudaStream_t>(stream), exp_output,
                        exp_transposed != 0, fhx_workspace_bytes(batch, n) ? workspace : nullptr);
}

int32_t fhx_matrix_exp_noalloc(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                               void* output, int64_t batch, int32_t n, int32_t dtype, void* stream) {
  using namespace fhx;
  int st = check_common(batch, n, dtype, output);
  if (st != FHX_OK) return st;
  st = check_view(input, in_s0, in_s1, in_s2, batch);
  if (st != FHX_OK) return st;
  if (batch == 0) return FHX_OK;
  if (batch > FHX_NOALLOC_MAX_BATCH) return FHX_ERR_NOALLOC_LIMIT;
  const View a{input, in_s0, in_s1, in_s2, in_negate ? -1.f : 1.f};
  const View none{nullptr, 0, 0, 0, 1.f};
  void* scratch = nullptr;
  if (grouped_size(n)) {
    st = noalloc_scratch(&scratch);
    if (st != FHX_OK) return st;
  }
  return dispatch<false>(a, none, output, batch, n, dtype, static_cast<cudaStream_t>(stream), nullptr, false,
                         scratch);
}

const char* fhx_status_string(int32_t status) {
  switch (status) {
    case FHX_OK: return "ok";
    case FHX_ERR_SIZE: return "expected 2 <= n <= 32 and batch >= 0";
    case FHX_ERR_DTYPE: return "dtype must be float32, bfloat16 or float16";
    case FHX_ERR_POINTER: return "null data pointer for a non-empty batch";
    case FHX_ERR_STRIDE: return "negative stride";
    case FHX_ERR_CUDA: return "a CUDA runtime call or kernel launch failed (see fhx_last_cuda_error)";
    case FHX_ERR_WORKSPACE: return "workspace smaller than fhx_workspace_bytes(batch, n)";
    case FHX_ERR_NOALLOC_LIMIT: return "batch larger than FHX_NOALLOC_MAX_BATCH, the limit of fhx_matrix_exp_noalloc";
    default: return "unknown status";
  }
}

int32_t fhx_last_cuda_error(void) { return static_cast<int32_t>(fhx::g_last_cuda_error); }

const char* fhx_last_cuda_error_string(void) { return cudaGetErrorString(fhx::g_last_cuda_error); }

int32_t fhx_abi_version(void) { return 106; }

uint64_t fhx_launch_count(void) { return fhx::g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
