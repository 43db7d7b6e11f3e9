// Allocation-free GEMM entry point.
//
// This entry point has no counterpart in the reference: it is an addition of
// this library for callers that must not allocate device memory themselves or
// have it allocated for them -- for example a host application that hands
// out every byte of device memory from its own pre-sized pool and forbids
// other allocations, or a latency-critical caller that cannot afford
// cudaMalloc/cudaFree, which may synchronize the whole device.  The ordinary
// op (torch.ops.b200.gemm_bf16_out) takes its split-K scratch from PyTorch's
// allocator; this one uses a fixed scratch area compiled into the library.
//
// Contract
//   * C[M, N] = X[M, K] . W[N, K]^T in bf16 with fp32 accumulation, the same
//     kernel as the ordinary op.  The caller passes and owns X, W and C
//     (row-major, row strides in elements, 16-byte-aligned base addresses and
//     row strides, K a multiple of 8).
//   * No cudaMalloc, cudaFree or allocating library call is made.  Split-K
//     partial sums and the kernel's status word live in file-scope
//     `static __device__` arrays: B200_NOALLOC_SCRATCH_FLOATS fp32 values
//     (4 MiB) plus one small status block.  Every GPU that loads the library
//     holds this memory until the process exits.  Shapes of at most 128 rows
//     split at most 8 ways reduce their partial sums on chip (a thread-block
//     cluster) and leave the scratch untouched.
//   * The first call on a device looks up the device address of that scratch
//     (cudaGetSymbolAddress, with that device current).  Make the first call
//     on each device before any stream capture.
//   * All calls share the same scratch, which keeps the last call's contents.
//     Calls that overlap on the GPU (different streams, or several host
//     threads without ordering) race on it: serialise them on one stream.
//   * Return value: 0 when the work was enqueued on `stream` (it has not run
//     yet); B200_NOALLOC_TOO_LARGE (-1) when the chosen split-K needs more
//     than B200_NOALLOC_SCRATCH_FLOATS partial values (splits * M * N);
//     B200_NOALLOC_BAD_ARGS (-2) for invalid arguments; otherwise the
//     cudaError_t of the CUDA call that failed.
//   * Errors found while the kernel runs (a pipeline wait that gave up, bit
//     0x1; an index out of range, 0x4; a tensor-memory allocation that did not
//     return, 0x8) do not show in the return value: the kernel ORs them into
//     the status word of the fixed area, which each call clears before its
//     kernel.  b200_gemm_bf16_noalloc_status() waits for `stream` and copies
//     that word out; when it is not 0, C holds partial results.  Like the
//     scratch, the word is shared by every call on the device: read it after
//     the call it should describe and before the next one.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define B200_NOALLOC_SCRATCH_FLOATS (1u << 20)
#define B200_NOALLOC_TOO_LARGE (-1)
#define B200_NOALLOC_BAD_ARGS (-2)

#ifdef __cplusplus
extern "C" {
#endif

// splits: 0 lets the library choose (as the ordinary op does), > 0 forces it.
int b200_gemm_bf16_noalloc(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int M,
                           int N, int K, int splits, cudaStream_t stream);

// Waits until all work queued on `stream` so far has finished, then stores
// the current device's status word in *out (0: the last call's kernel ran
// without error).  Allocates nothing.  Returns 0, B200_NOALLOC_BAD_ARGS for a
// null `out`, or the cudaError_t of the failed copy or wait.
int b200_gemm_bf16_noalloc_status(uint32_t* out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
