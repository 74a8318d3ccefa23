// Allocation-free C entry point of the dion_b200 extension.
//
// This entry point has no counterpart in the reference project; it exists
// for callers of this library that cannot allocate device memory at the time
// they need the result, for example:
//   * host runtimes that reserve a fixed device-memory budget at start-up and
//     forbid any further cudaMalloc (and any allocator that would call it);
//   * code that runs inside an allocator or out-of-memory callback, where
//     asking an allocator for memory again would recurse or deadlock;
//   * plain C / C++ callers that link this library without PyTorch and have
//     no caching allocator to hand it.
// Such callers pass their own input and output buffers; the only scratch
// memory the computation needs lives in a fixed-size array inside this
// library (see the limits below), so the call itself allocates nothing.
#pragma once
#include <cstdint>

#ifdef __cplusplus
extern "C" {
#endif

// Scratch capacity: 65536 fp32 block partial sums (256 KiB per GPU that
// loads the library, held until the process exits). A call needs
// batch * ceil(numel / 16384) partials, i.e. at most 2^30 input elements.
#define BDION_NOALLOC_MAX_PARTIALS 65536

// Return codes.
#define BDION_NOALLOC_OK 0
#define BDION_NOALLOC_BAD_ARGUMENT (-1)
#define BDION_NOALLOC_TOO_LARGE (-2)
#define BDION_NOALLOC_SETUP_FAILED (-3)
#define BDION_NOALLOC_LAUNCH_FAILED (-4)
#define BDION_NOALLOC_PENDING_ERROR (-5)

// Per-matrix sum of squares of a batch of equally sized tensors:
//   out[b] = sum_i x[b * stride + i]^2   for b < batch, i < numel
// x: device pointer to fp32 (dtype 0) or bf16 (dtype 1) data;
// stride: elements between consecutive tensors (>= numel);
// out: device pointer to `batch` fp32 results;
// stream: the cudaStream_t to launch on (NULL = the legacy default stream).
// The work is queued on `stream`; the function does not synchronise.
//
// Errors: a CUDA error that is already pending when the call starts (left by
// earlier, unrelated work) is not this call's failure: the call then launches
// nothing, returns BDION_NOALLOC_PENDING_ERROR and leaves that error set for
// the caller's own check. A launch that fails returns
// BDION_NOALLOC_LAUNCH_FAILED, also leaving the CUDA error set.
//
// Same kernels and summation order as the extension's multi_sumsq op, so the
// results match it bit for bit.
//
// Set-up: the first call on each device looks up that device's address of
// the scratch array (cudaGetSymbolAddress) while that device is current, and
// caches it. Make that first call before any stream capture on the device.
//
// Sharing: every call on a device uses the same scratch array and leaves its
// last contents in it; every scratch slot a call reads is written earlier in
// the same call, so nothing has to be cleared between calls. Calls that can
// run at the same time on the GPU (different streams without ordering between
// them) race on the scratch array: serialise them on one stream or with events.
int bdion_batched_sumsq_noalloc(const void* x, int dtype, int64_t batch, int64_t numel, int64_t stride, float* out,
                                void* stream);

#ifdef __cplusplus
}
#endif
