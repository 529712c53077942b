// Allocation-free DMD generator loss: one exported C entry point.
//
// This entry point has no counterpart in the reference; it is an addition of
// this library.
//
// Who it is for: callers that are not allowed to allocate device memory,
// for example a host application or plugin that has reserved its whole
// device-memory budget up front and forbids any further cudaMalloc, or code
// driven from a foreign runtime whose allocator this library cannot reach.
// The regular entry point (h3_a100._C.dmd_forward) allocates its reduction
// scratch and its outputs through PyTorch, so those callers cannot use it.
//
// What it computes (same definition as dmd_forward, per sample s):
//   d_s   = mean_i |generated[s,i] - x0_real[s,i]|          (floor 1e-12)
//   grad  = (x0_fake - x0_real) / d_s                       (non-finite -> 0)
//   loss  = 0.5 * mean over all samples and elements of grad^2
// All pointers are device fp32 arrays of samples * per_sample elements, except
// `loss`, one float.  The caller passes inputs and outputs; nothing is
// allocated.
//
// Scratch: a file-scope device array of 2 * H3_DMD_NOALLOC_MAX_SAMPLES floats
// (8 KiB; every GPU that loads this library holds it until the process exits).
// Calls with samples > H3_DMD_NOALLOC_MAX_SAMPLES are rejected.
//
// Set-up: the first call on a device looks up the device address of that
// array (cudaGetSymbolAddress, with the device current).  Make that first call
// on each device before any stream capture.
//
// Concurrency: every call shares the one scratch array, which keeps the last
// call's contents (each call clears the part it uses before accumulating).
// Calls that overlap on the GPU (different streams, or different host
// threads on one device) race on it and give wrong results; serialise them.
//
// Returns 0 on success, otherwise one of the H3_NOALLOC_E* codes below (a
// one-line reason is also printed to stderr).
#pragma once

#include <cuda_runtime.h>

#define H3_DMD_NOALLOC_MAX_SAMPLES 1024

#define H3_NOALLOC_OK 0
#define H3_NOALLOC_EINVAL (-1)      // null pointer or non-positive size
#define H3_NOALLOC_ETOOBIG (-2)     // samples > H3_DMD_NOALLOC_MAX_SAMPLES
#define H3_NOALLOC_ESYMBOL (-3)     // device address of the scratch array not available
#define H3_NOALLOC_ELAUNCH (-4)     // a kernel launch failed
#define H3_NOALLOC_EDEVICE (-5)     // no current CUDA device

#ifdef __cplusplus
extern "C" {
#endif

int h3_dmd_loss_noalloc(const float* generated, const float* x0_fake, const float* x0_real, long long samples,
                        long long per_sample, float* loss, float* grad, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
