// Allocation-free split-K GEMM entry point (C ABI).
//
// This entry point has no counterpart in the reference; it is an addition of this
// framework. It exists for callers that cannot call cudaMalloc at the point where
// they need a product: a serving process whose memory pool has already reserved the
// device's HBM (a cudaMalloc there fails or forces the pool to give memory back),
// and C/C++ hosts that do not run torch's caching allocator and must not have a
// library allocate device memory behind their own allocator (cudaMalloc and
// cudaFree can also synchronise the device, which such a host schedules itself).
//
// It runs the same tcgen05 GEMM kernel as the torch binding `gemm_test`
//   out[M, N] (bf16, row-major, row stride out_ld) = A * B^T
// with a forced split-K count, but keeps the split-K partials and the per-tile
// arrival counters in one file-scope device array of NSB_GEMM_NOALLOC_SCRATCH_BYTES
// (4 MiB) instead of allocating them. It calls no cudaMalloc, cudaFree or any
// allocating library routine (torch's included).
//
// Operands: `a` is A with rows x cols elements and row stride a_ld; a_mn_major = 0
// means A is [M, K] (K-major), 1 means A is stored [K, M] (MN-major). The same for
// `b` with N in place of M. All three pointers 16-byte aligned; the strides of A and
// B a multiple of 8 elements (TMA rules) and at least their row lengths
// (a_ld >= a_cols, b_ld >= b_cols); out_ld >= N.
//
// Limits: splits in [1, 16]; splits * M * N * 4 bytes of partials must fit in the
// partial area (NSB_GEMM_NOALLOC_PARTIAL_FLOATS floats); a launch that splits K
// (more than one effective split) has at most NSB_GEMM_NOALLOC_MAX_TILES output
// tiles (128 x BN, BN = 64..256 by N), one arrival counter each. An unsplit launch
// uses no scratch and has no tile limit. Larger problems are rejected with an
// error code and a message; they are not truncated.
//
// State that must start at zero: the per-tile arrival counters. Static device
// storage starts zeroed and every completed launch leaves the counters it used at
// zero again. After a launch that reported a device-side timeout (status word
// nonzero), call nsb_gemm_noalloc_reset before the next launch. The partial area
// needs no initial value.
//
// Concurrency: the scratch is one array per device. Two calls on the same device
// whose kernels can overlap (different streams without ordering, or different host
// threads) race on the partials and the counters and produce wrong results. Order
// all calls on a device, e.g. issue them on one stream.
//
// Set-up: nsb_gemm_noalloc_setup(device) looks up the scratch address on `device`
// (made current for the call; the previous current device is restored). The entry
// point performs that set-up itself on its first call for the current device;
// when relying on that, make the first call before any stream capture begins.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

#define NSB_GEMM_NOALLOC_SCRATCH_BYTES (4u << 20)
#define NSB_GEMM_NOALLOC_MAX_TILES 4096u
#define NSB_GEMM_NOALLOC_PARTIAL_FLOATS ((NSB_GEMM_NOALLOC_SCRATCH_BYTES - 4u * NSB_GEMM_NOALLOC_MAX_TILES - 256u) / 4u)

// 0 on success; otherwise a nonzero code, and nsb_gemm_noalloc_error() describes it.
int nsb_gemm_noalloc_setup(int device);

// Enqueue out = A * B^T on `stream` (a cudaStream_t; null = legacy default stream).
// Return codes: 0 ok, 1 invalid argument, 2 over the scratch limits, 3 CUDA error.
int nsb_gemm_bf16_splitk_noalloc(const void* a, int a_mn_major, long long a_rows, long long a_cols,
                                 long long a_ld, const void* b, int b_mn_major, long long b_rows,
                                 long long b_cols, long long b_ld, void* out, long long out_ld, int M,
                                 int N, int K, int splits, void* stream);

// Device-side status word of the current device (nonzero after a bounded wait in the
// kernel timed out). Synchronous read; no allocation. 0 on success.
int nsb_gemm_noalloc_status(int* status);

// Zero the counters and the status word of the current device on `stream`.
int nsb_gemm_noalloc_reset(void* stream);

// Message of the calling thread's last failed call ("" if none).
const char* nsb_gemm_noalloc_error(void);

#ifdef __cplusplus
}
#endif
