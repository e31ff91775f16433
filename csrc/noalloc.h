// Allocation-free entry point for the fused embedding sparse update.
//
// This entry point has no counterpart in the Primus-DLRM reference: the
// reference only reaches its embedding optimizer through TorchRec/FBGEMM.
//
// Who it is for: callers that must not allocate device memory while they
// run. Examples are a host runtime that gives this library a fixed memory
// budget it may not grow, and code on a latency-critical thread that cannot
// afford the device-wide synchronisation cudaMalloc/cudaFree may imply. The
// regular entry point (the torch binding emb_reduce_update) allocates its
// scratch lazily through PyTorch's allocator. This one takes its scratch from
// a fixed array compiled into the library and allocates nothing.
//
// What it does: applies one step of SGD / Adagrad / row-wise Adagrad / Adam
// to the rows of ONE fp32 embedding table [rows, dim]. The gradients
// arrive as n rows of `grads` (fp32 or bf16, row stride `grad_stride`
// elements). `sorted_keys[q]` is the table row of sorted position q, in
// ascending order; `perm[q]` says which grad row it is. Rows that occur
// several times are summed before the update, as in the regular path.
//
// Limits: n <= PD_NOALLOC_MAX_IDS, dim <= PD_NOALLOC_MAX_DIM, dim % 4 == 0.
// The scratch array is PD_NOALLOC_MAX_IDS / 32 * PD_NOALLOC_MAX_DIM floats
// (8 MiB) plus one int per 32 ids (32 KiB). Every GPU that loads the library
// holds it until the process exits.
//
// Shared state: every call on a device uses the same scratch array, and the
// array keeps the last call's contents. The entry point clears the part it
// uses (on `stream`) before its kernel runs. Calls whose work overlaps on
// the GPU (for example on two streams without ordering) race on the array
// and give wrong results. Order them on one stream or with events.
//
// Set-up: the first call on each device looks up the device address of the
// scratch array (cudaGetSymbolAddress) with that device current. Make that
// first call before any stream capture begins on the device.
//
// Alignment: the kernel reads gradient rows as 4-element vectors and table /
// state rows as float4, so grads must be 16-byte aligned (8 bytes for bf16),
// weight and the per-element state arrays 16-byte aligned, and grad_stride a
// multiple of 4 elements with grad_stride >= dim.
//
// Return value: 0 on success; PD_NOALLOC_TOO_LARGE if n or dim exceed the
// limits above; PD_NOALLOC_BAD_ARG for null pointers, dim % 4 != 0, a
// grad_stride below dim or not a multiple of 4, a misaligned pointer, or an
// unknown optimizer / dtype; otherwise a cudaError_t value (> 0) from the
// set-up or the launch. On error nothing is launched. Table ids outside
// [0, rows) and perm values outside [0, n) are skipped and recorded as 1 in
// *err (err may be null; the rest of the call still runs).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define PD_NOALLOC_MAX_IDS (1 << 18)
#define PD_NOALLOC_MAX_DIM 256
#define PD_NOALLOC_TOO_LARGE (-1)
#define PD_NOALLOC_BAD_ARG (-2)

#ifdef __cplusplus
extern "C" {
#endif

// opt_kind: 0 sgd, 1 adagrad, 2 row-wise adagrad (state1 [rows]), 3 adam
// (state1 = m, state2 = v, both [rows, dim]); bc1/bc2: Adam bias corrections
// 1 - beta^t. grad_dtype: 0 fp32, 1 bf16.
__attribute__((visibility("default"))) int pd_emb_sparse_update_noalloc(
    const int64_t* sorted_keys, const int64_t* perm, int64_t n, const void* grads, int grad_dtype,
    int64_t grad_stride, float* weight, int64_t rows, int dim, float* state1, float* state2, int opt_kind,
    float lr, float eps, float weight_decay, float beta1, float beta2, float bc1, float bc2, int* err,
    cudaStream_t stream);

#ifdef __cplusplus
}
#endif
