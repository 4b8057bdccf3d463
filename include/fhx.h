/*
 * fhx.h -- C ABI of the B200 batched small-matrix exponential (libfhx.so).
 *
 * Plain pointers, element strides and sizes; no framework types.  Every entry point
 * launches asynchronously on the given CUDA stream of the *current* device and returns a
 * status code (FHX_OK on success).  Inputs are read-only, the output is written in full,
 * nothing is retained between calls and no device memory is allocated.
 *
 * Reference interfaces these replace (nickjeliopoulos/flash-hyperconnections):
 *   fhx_matrix_exp  <- op schema  flash_hypercons::_matrix_exp(Tensor input) -> Tensor
 *                      (csrc/register.cpp:11, CUDA impl csrc/register.cpp:16,
 *                       host launcher csrc/matrix_exp.cu:80-82 -> :51-78)
 *   fhx_frechet     <- op schema  flash_hypercons::_frechet(Tensor input, Tensor direction) -> Tensor
 *                      (csrc/register.cpp:12, CUDA impl csrc/register.cpp:17,
 *                       host launcher csrc/matrix_exp.cu:84-86 -> :51-78)
 * The argument checks of csrc/matrix_exp.cu:52-58 map to FHX_ERR_* codes below; the
 * reference's pre-copies (dtype cast, contiguous, resolve_neg, zero padding,
 * csrc/matrix_exp.cu:35-44,77) are replaced by the strides/negate arguments, which the
 * kernels honour in their load path.
 */
#ifndef FHX_H_
#define FHX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element type of input, direction and output (all three share it). */
#define FHX_DTYPE_F32 0
#define FHX_DTYPE_BF16 1
#define FHX_DTYPE_F16 2

/* Status codes. */
#define FHX_OK 0
#define FHX_ERR_SIZE 1       /* n outside [2, 32] or batch < 0                          */
#define FHX_ERR_DTYPE 2      /* dtype not one of FHX_DTYPE_*                            */
#define FHX_ERR_POINTER 3    /* null data pointer with batch > 0                        */
#define FHX_ERR_STRIDE 4     /* negative stride                                         */
#define FHX_ERR_CUDA 5       /* a CUDA runtime call or the kernel launch failed; the
                                cudaError_t is kept for fhx_last_cuda_error()            */
#define FHX_ERR_WORKSPACE 6  /* workspace smaller than fhx_workspace_bytes(batch, n)   */
#define FHX_ERR_NOALLOC_LIMIT 7 /* batch > FHX_NOALLOC_MAX_BATCH in fhx_matrix_exp_noalloc */

#define FHX_MAX_N 32
#define FHX_NOALLOC_MAX_BATCH (1 << 20) /* matrices per call of fhx_matrix_exp_noalloc      */
#define FHX_MIX_MAX_N 4      /* streams per token of the fused stream mixing            */

/*
 * Y = exp(A) for a batch of n x n matrices, 2 <= n <= 32.
 *   input            A, element (b, i, j) at input[b*in_s0 + i*in_s1 + j*in_s2]
 *   in_negate        non-zero: use -A (a lazily negated view)
 *   output           contiguous [batch, n, n], same dtype
 *   stream           a cudaStream_t (NULL = legacy default stream)
 * Any non-finite entry of a matrix makes that matrix's whole output NaN.
 */
int32_t fhx_matrix_exp(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                       void* output, int64_t batch, int32_t n, int32_t dtype, void* stream);

/*
 * Frechet derivative L(A, E) = d/dt exp(A + tE) at t = 0 (the upper-right block of
 * exp([[A, E], [0, A]])).  The autograd backward of Y = exp(X) is
 * fhx_frechet(X^T, dY), obtained by passing X's strides with in_s1/in_s2 swapped.
 * The degree and number of squarings depend on A only and are identical for A and A^T,
 * except for 5 <= n <= 8 without a workspace (fhx_matrix_exp / fhx_frechet): there the eight
 * matrices that share a warp run the largest degree chosen among them, which is at least as
 * accurate; a matrix's output bits can then depend on its aligned group of 8 neighbours (within
 * the tolerance).  Results are bit-stable for batch prefixes made of whole aligned groups and
 * for re-runs of the same batch.  The _ws entry points make those sizes per-matrix too.
 * Any non-finite entry of A or E makes that matrix's whole output NaN.
 */
int32_t fhx_frechet(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                    const void* direction, int64_t dir_s0, int64_t dir_s1, int64_t dir_s2, int32_t dir_negate,
                    void* output, int64_t batch, int32_t n, int32_t dtype, void* stream);

/*
 * Device workspace (bytes) that fhx_matrix_exp_ws / fhx_frechet_ws / fhx_frechet_grouped /
 * fhx_matrix_exp_frechet need for a batch of n x n matrices: 6 bytes per matrix plus 2 KB for
 * 5 <= n <= 8 (the degree grouping), 2 bytes per matrix rounded up to 256 for 9 <= n <= 16 (one
 * key per matrix), 0 otherwise.
 */
size_t fhx_workspace_bytes(int64_t batch, int32_t n);

/*
 * fhx_matrix_exp and fhx_frechet with a caller-allocated device workspace of at least
 * fhx_workspace_bytes(batch, n) bytes (16-byte aligned; contents on entry do not matter, and
 * the workspace must not be used by another call in flight on the GPU at the same time).  For
 * 5 <= n <= 8, where eight matrices share a warp, the batch is first grouped by (degree,
 * squarings) -- two small passes that classify every matrix in float64 and build a
 * permutation -- so that the matrices of a warp run the same program, and every matrix runs its
 * own degree: its result depends on that matrix alone (bit-stable under any batching), and
 * fhx_frechet_ws on A^T repeats the (m, s) of fhx_matrix_exp_ws on A exactly.  Other n are
 * per-matrix already; for 9 <= n <= 16 fhx_matrix_exp_ws stores each matrix's key -- its
 * (m, s) -- in the workspace for a later fhx_frechet_grouped, and fhx_frechet_ws does not use it.
 * n <= 4 and n >= 17 need no workspace (workspace_bytes may be 0).
 * Reference interfaces: as fhx_matrix_exp / fhx_frechet (the workspace replaces the
 * reference's per-call pre-copies, csrc/matrix_exp.cu:35-44, which the caching allocator
 * provides there).
 */
int32_t fhx_matrix_exp_ws(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                          void* output, int64_t batch, int32_t n, int32_t dtype, void* workspace,
                          size_t workspace_bytes, void* stream);
int32_t fhx_frechet_ws(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                       const void* direction, int64_t dir_s0, int64_t dir_s1, int64_t dir_s2, int32_t dir_negate,
                       void* output, int64_t batch, int32_t n, int32_t dtype, void* workspace, size_t workspace_bytes,
                       void* stream);

/*
 * fhx_frechet_ws that reuses the grouping of an earlier fhx_matrix_exp_ws on the same matrices
 * (or their transposes: the classification of A and A^T is identical), same batch and n.  An
 * extension without reference counterpart, for the autograd backward: exp(X) on X, then
 * L(X^T, dY) on X^T, with the forward's workspace kept until the backward.  For 5 <= n <= 8 the
 * grouping passes are skipped, and for 9 <= n <= 16 the kernel's norm phase: every matrix runs
 * the forward's (m, s) from the stored keys; the kernels only read the workspace.  Results
 * equal fhx_frechet_ws's bit for bit.  The caller guarantees that the workspace holds those
 * keys and that the matrices were not changed in between: a workspace of other matrices gives
 * wrong results (permutation entries outside [0, batch) are skipped, so nothing is read or
 * written out of bounds).  n <= 4 and n >= 17 ignore the workspace (their backward recomputes
 * the same (m, s) from A^T).
 */
int32_t fhx_frechet_grouped(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                            const void* direction, int64_t dir_s0, int64_t dir_s1, int64_t dir_s2,
                            int32_t dir_negate, void* output, int64_t batch, int32_t n, int32_t dtype,
                            const void* workspace, size_t workspace_bytes, void* stream);

/*
 * fhx_matrix_exp_ws for callers that cannot allocate device memory.  No counterpart in the
 * reference (whose operator allocates through PyTorch's caching allocator).  Some callers have
 * no allocator to call: a plugin inside a host engine that owns all device memory and hands the
 * plugin only its input and output buffers, or a latency-critical path that must never enter
 * cudaMalloc (which can synchronize the device and take unbounded time).  This entry point
 * takes inputs and outputs like fhx_matrix_exp and allocates nothing: for 5 <= n <= 8 its
 * grouping workspace is a static device array of the library, sized for at most
 * FHX_NOALLOC_MAX_BATCH matrices (about 6 MiB, held by every GPU that loads the library until
 * the process exits); other n need no workspace.  Results equal fhx_matrix_exp_ws's.
 *   - A batch larger than FHX_NOALLOC_MAX_BATCH returns FHX_ERR_NOALLOC_LIMIT (nothing runs).
 *   - The first call on a device looks up the array's device address there
 *     (cudaGetSymbolAddress, with that device current); make that first call before any
 *     stream capture.
 *   - Every call shares the one array and each call fully rewrites what it reads from it.
 *     Calls that overlap on the GPU -- on different streams, or from different host threads --
 *     race on it: issue them in one stream order.
 */
int32_t fhx_matrix_exp_noalloc(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                               void* output, int64_t batch, int32_t n, int32_t dtype, void* stream);

/*
 * exp(A) and L(A, E) from ONE launch: the Frechet kernel carries the pair (exp, derivative)
 * through its program anyway, and this entry point stores both parts.
 *   exp_output       contiguous [batch, n, n]: exp(A), or exp(A)^T = exp(A^T) when
 *                    exp_transposed is non-zero
 *   frechet_output   contiguous [batch, n, n]: L(A, E)
 * Two uses:
 *   - forward-mode AD (JVP) of exp at A with tangent E: primal exp(A) and tangent L(A, E);
 *   - forward and backward of Y = exp(X) together, when the upstream gradient G is known:
 *     pass A = X^T (in_s1/in_s2 swapped), E = G, exp_transposed = 1; then
 *     exp_output = exp(X) = Y and frechet_output = L(X^T, G) = dL/dX.
 * workspace (may be null, else at least fhx_workspace_bytes(batch, n) bytes): as in
 * fhx_frechet_ws.  The pair's degree and scaling are those of fhx_frechet (with a workspace:
 * fhx_frechet_ws) on the same A, so frechet_output equals that call's output bit for bit;
 * without a workspace, exp_output can differ from fhx_matrix_exp's in the last bits where the
 * forward kernel shares a degree between neighbouring matrices.
 * Reference counterpart: none as one call.  It fuses the forward-AD rule of the reference
 * (native, flash_hypercons/ops/matrix_exp/__init__.py:89-94) and the forward + backward pair
 * _matrix_exp / _frechet (csrc/register.cpp:11-12) into one launch.
 */
int32_t fhx_matrix_exp_frechet(const void* input, int64_t in_s0, int64_t in_s1, int64_t in_s2, int32_t in_negate,
                               const void* direction, int64_t dir_s0, int64_t dir_s1, int64_t dir_s2,
                               int32_t dir_negate, void* exp_output, int32_t exp_transposed, void* frechet_output,
                               int64_t batch, int32_t n, int32_t dtype, void* workspace, size_t workspace_bytes,
                               void* stream);

/*
 * Hyper-connection stream mixing fused with the exponential, one warp per token:
 *   Y[t] = exp(H[t]) X[t]
 * for tokens t < `tokens`, H[t] an n x n mixing matrix (2 <= n <= FHX_MIX_MAX_N) and X[t] the
 * token's n residual streams of width d.
 *   h               H, element (t, i, j) at h[t*h_s0 + i*h_s1 + j*h_s2] in h_dtype;
 *                   h_negate non-zero: use -H
 *   x               X, element (t, j, c) at x[t*x_s0 + j*x_s1 + c] in x_dtype (unit column stride)
 *   y               contiguous [tokens, n, d] in x_dtype
 * exp(H[t]) is computed in registers with the arithmetic of fhx_matrix_exp's n <= 4 kernel and
 * never written to memory; a non-finite entry of H[t] makes Y[t] NaN.  Rows move in 16-byte
 * chunks when d and the row strides allow it.
 * Reference counterpart: none (the reference computes exp only; its name refers to
 * hyper-connections, README.md:1-5).  Unfused, this is fhx_matrix_exp followed by a batched
 * [n x n] x [n x d] product reading exp(H) back from memory.
 */
int32_t fhx_stream_mix(const void* h, int64_t h_s0, int64_t h_s1, int64_t h_s2, int32_t h_negate, int32_t h_dtype,
                       const void* x, int64_t x_s0, int64_t x_s1, int32_t x_dtype, void* y, int64_t tokens, int32_t n,
                       int64_t d, void* stream);

/*
 * Device workspace (bytes) of fhx_stream_mix_backward: tokens * n * n float32 values.
 */
size_t fhx_stream_mix_workspace_bytes(int64_t tokens, int32_t n);

/*
 * Backward of fhx_stream_mix for the upstream gradient dY (x_dtype, element (t, i, c) at
 * dy[t*dy_s0 + i*dy_s1 + c]):
 *   dX[t] = exp(H[t])^T dY[t]                 dx: contiguous [tokens, n, d] in x_dtype
 *   dH[t] = L(H[t]^T, dY[t] X[t]^T)           dh: contiguous [tokens, n, n] in h_dtype
 * Two launches: a warp per token streams X and dY once, writing dX (exp(H[t]) recomputed in
 * registers) and G[t] = dY[t] X[t]^T, reduced over d in float32 in a fixed order
 * (deterministic), into the workspace; then one thread per token computes dH[t] from H[t]^T and
 * G[t] with the arithmetic of fhx_frechet's n <= 4 kernel.
 *   workspace        at least fhx_stream_mix_workspace_bytes(tokens, n) bytes, 4-byte aligned
 *                    (contents on entry do not matter; not shared with a call in flight)
 */
int32_t fhx_stream_mix_backward(const void* h, int64_t h_s0, int64_t h_s1, int64_t h_s2, int32_t h_negate,
                                int32_t h_dtype, const void* x, int64_t x_s0, int64_t x_s1, int32_t x_dtype,
                                const void* dy, int64_t dy_s0, int64_t dy_s1, void* dx, void* dh, int64_t tokens,
                                int32_t n, int64_t d, void* workspace, size_t workspace_bytes, void* stream);

/* Static description of a status code. */
const char* fhx_status_string(int32_t status);

/*
 * The cudaError_t behind the calling thread's most recent FHX_ERR_CUDA (cudaSuccess = 0 if
 * none), and its cudaGetErrorString text.  The launch check reads cudaGetLastError(), so an
 * earlier asynchronous fault still pending on the device is reported by the next call, as
 * with any CUDA launch check.  (The reference's C10_CUDA_KERNEL_LAUNCH_CHECK,
 * csrc/matrix_exp.cu:32, reports the same cudaGetErrorString text in its exception.)
 */
int32_t fhx_last_cuda_error(void);
const char* fhx_last_cuda_error_string(void);

/* ABI version of this library (major * 100 + minor). */
int32_t fhx_abi_version(void);

/*
 * Kernels this library has launched in this process (all devices and threads), counted on the
 * host at each launch.  No reference counterpart: tests and benchmarks read it around a call to
 * count its launches without the CUDA profiler.
 */
uint64_t fhx_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* FHX_H_ */
