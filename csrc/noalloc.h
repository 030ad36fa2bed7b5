// No-allocation entry point of the fused RMSNorm + adaLN-modulation backward.
//
// This entry point has no counterpart in the reference (wenhaochai/nano-gpic); it is an addition of this library.
//
// Who needs it: callers that cannot allocate device memory at the moment they call. For example: embedders that hand
// the GPU's memory to their own fixed pool and forbid any allocation behind their back, real-time loops that must not
// pay for an allocation, and hosts that call from a plain C runtime with no PyTorch caching allocator. The
// regular entry point (rms_mod_bwd in csrc/norm.cu) gets its scratch from PyTorch's allocator. This one takes the same
// inputs and outputs but keeps its scratch, the per-chunk partial column sums, in a fixed device array inside the
// library, so it calls no cudaMalloc, cudaFree or any other allocating routine.
//
// The scratch array is NG_NOALLOC_RMS_SCRATCH_FLOATS fp32 values (8 MiB). Every GPU that loads the library holds it
// until the process exits. A call needs ceil(rows_per_group / 64) * groups * 3 * C + groups * C values of it (the
// per-chunk partials, then one row of weight-gradient partials per group). For example, 128 samples x 256 tokens at
// C = 1024 need 1.70M values. Larger calls are rejected with NG_NOALLOC_ERR_TOO_LARGE and nothing is launched. The
// groups are a grid dimension, so at most 65535 groups are accepted (NG_NOALLOC_ERR_ARGS beyond).
//
// Errors: a CUDA error that earlier work left pending on the calling thread is not consumed. The call returns
// NG_NOALLOC_ERR_PENDING without launching anything, and the error stays for its owner to read.
//
// Set-up: the first call on each device looks up the array's device address (cudaGetSymbolAddress) with that device
// current. Make that first call before any stream capture begins. Later calls do no set-up.
//
// Sharing: every call on a device uses the same array, and the array keeps the last call's contents. Each call
// overwrites every value it reads, so nothing has to start at zero. Calls that overlap on the GPU (on different
// streams without ordering, or from several threads at once) race on the array and give wrong results. Order them on
// one stream, or serialise them.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define NG_NOALLOC_RMS_SCRATCH_FLOATS (2 * 1024 * 1024)

#define NG_NOALLOC_OK 0
#define NG_NOALLOC_ERR_TOO_LARGE 1  // the call needs more scratch than NG_NOALLOC_RMS_SCRATCH_FLOATS
#define NG_NOALLOC_ERR_ARGS 2       // a null pointer, C % 8 != 0, C > 2048, a non-positive size, > 65535 groups
#define NG_NOALLOC_ERR_SETUP 3      // cudaGetSymbolAddress failed (no device, or the library's module did not load)
#define NG_NOALLOC_ERR_LAUNCH 4     // a kernel launch failed (cudaGetLastError after the launch)
#define NG_NOALLOC_ERR_PENDING 5    // an earlier CUDA error was pending on this thread; left in place, nothing launched

#ifdef __cplusplus
extern "C" {
#endif

// Backward of h = bf16(w * x * rstd * (1 + scale[g]) + shift[g]), g = row / rows_per_group (see csrc/norm.cu).
//   dh, x, dres, dx: bf16 [M, C] contiguous (dres may be null); rstd: fp32 [M]; w: fp32 [C].
//   scale: bf16 rows of `ld_scale` elements (a column slice of the adaLN output), or null for a plain RMSNorm.
//   dw: fp32 [C], the weight gradient is ADDED into it (may be null).
//   dshift / dscale: fp32 rows of ld_dshift / ld_dscale elements, overwritten (ignored when scale is null; may be null).
// Launches three kernels (two when dw is null) on `stream` and returns at once. Returns NG_NOALLOC_OK or one of the
// error codes above.
int ng_rms_mod_bwd_noalloc(const void* dh, const void* x, const float* rstd, const float* w, const void* scale,
                           int64_t ld_scale, const void* dres, void* dx, float* dw, float* dshift, int64_t ld_dshift,
                           float* dscale, int64_t ld_dscale, int M, int C, int rows_per_group, cudaStream_t stream);

// Human-readable text of an error code of ng_rms_mod_bwd_noalloc.
const char* ng_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
