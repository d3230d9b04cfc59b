// Allocation-free C entry point of the RMSNorm backward kernel.
//
// This entry point has no counterpart in the reference (ElasticMegatron ships no native code).  It exists for
// callers that cannot allocate device memory: code running inside a host framework that owns every device
// allocation through its own pool, code embedded where linking the CUDA allocator (or torch's) is not allowed,
// and callers that must not let the first call of a step grow the memory footprint.  The caller passes only
// its inputs and outputs; the per-CTA partial sums that the regular entry point (rmsnorm_bwd in
// csrc/ops/norm_act.cu) allocates per call live instead in one fixed, file-scope device array of
// EMB_NOALLOC_SCRATCH_FLOATS floats (16 MiB), which every GPU that loads this library holds until the
// process exits.
//
// Contract:
//   * dy, x: [T, H] bf16 row-major; w: [H] bf16; rstd: [T] fp32 (from the forward pass);
//     dx: [T, H] bf16 output; dw: [H] fp32 output, overwritten (accumulate == 0) or added to (!= 0).
//   * T must be at most INT_MAX (2^31 - 1) rows; H must be a multiple of 8 and at most 32768; the scratch holds grid * H floats with
//     grid = min(T, 2 * SMs, EMB_NOALLOC_SCRATCH_FLOATS / H), so every supported size fits.
//   * The first call on a device looks up the device address of the scratch array (cudaGetSymbolAddress)
//     with that device current; make that first call before any stream capture on the device.
//   * All calls on a device share the one scratch array and each call overwrites the part it uses (nothing
//     in it has to start at zero).  Calls that can overlap on the GPU - on different streams without
//     ordering between them - race on it; serialize them.
//   * No device or host memory is allocated, by this code or by any library it calls.
// Returns 0 on success, EMB_NOALLOC_EBADSIZE for a rejected shape (a message is printed to stderr), or the
// CUDA error code of a failed symbol lookup or launch.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define EMB_NOALLOC_SCRATCH_FLOATS (4 * 1024 * 1024)
#define EMB_NOALLOC_EBADSIZE (-22)

#ifdef __cplusplus
extern "C" {
#endif

int emb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw,
                            int64_t T, int64_t H, int accumulate, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
