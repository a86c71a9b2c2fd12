// Allocation-free entry point of the per-head GroupNorm forward.
//
// This entry point has no counterpart in the reference framework; it exists for callers that
// cannot allocate device memory while they run this op: code running inside a custom memory
// arena or allocator hook (where a nested cudaMalloc would re-enter the allocator), real-time
// or embedded hosts that forbid allocation after start-up, and foreign runtimes that hand over
// pre-allocated buffers and a stream but no allocator.  It performs the same computation as
// the regular GroupNorm forward of this library, but keeps its intermediate statistics in a
// fixed device array compiled into the library instead of allocating them.
//
// Contract:
//   * Scratch: a file-scope device array of MAMF_NOALLOC_SCRATCH_FLOATS floats (4 MiB).  Every
//     GPU that loads the library holds it until the process exits.  A call needs
//     B*H*ceil(S/64)*3 floats of it, plus 2*B*H more when mean_rstd_out is NULL; larger problems
//     are rejected with return code 2.
//   * Set-up: the first call on each device looks up the array's device address with
//     cudaGetSymbolAddress while that device is current.  Make that first call outside any
//     stream capture.
//   * Sharing: all calls use the same array and nothing in it needs to start at zero (every
//     value read is written earlier in the same call).  Calls whose work overlaps on the GPU
//     (different streams, or different host threads without ordering) race on the array; order
//     them on one stream.
//   * No cudaMalloc, cudaFree or allocating library routine is called.
//   * Errors: a launch error that earlier work left pending on the calling thread is reported
//     as rc 3 with its own message, before anything is launched.  After a failed launch the
//     cached address of the current device is dropped, so a context that was reset in the
//     meantime (cudaDeviceReset) gets a fresh lookup on the next call.
//   * Limits: B and H <= 65535; S, hd and H*hd < 2^31; B*S*H*hd < 2^63 (rc 1 otherwise).
//
// Arguments: x and y are (B, S, H*hd) contiguous, dtype 0 = float32, 1 = bfloat16; w and b are
// (H*hd,) float32; mean_rstd_out is (B*H, 2) float32 or NULL; stream is a cudaStream_t (NULL =
// legacy default stream).  Returns 0 on success, 1 for invalid arguments, 2 when the problem
// needs more scratch than the array holds, 3 for a CUDA error; mamf_noalloc_last_error() gives
// a message for the last failure on the calling thread.
#pragma once

#include <stdint.h>

#define MAMF_NOALLOC_SCRATCH_FLOATS (1 << 20)

#ifdef __cplusplus
extern "C" {
#endif

int mamf_head_groupnorm_fwd_noalloc(const void* x, const float* w, const float* b, void* y,
                                    float* mean_rstd_out, int64_t B, int64_t S, int64_t H, int64_t hd,
                                    float eps, int dtype, void* stream);

const char* mamf_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
