// Entry points of libminidist_cuda.so that allocate no device memory.
//
// This interface has no counterpart in the reference framework; it exists for
// callers of this library that cannot allocate device memory themselves.
//
// md_colsum_noalloc — column sums of a bf16 matrix into fp32, identical in
// result to md_colsum (same kernels, same fixed summation order), but its
// scratch space is a static device array inside the library instead of a
// caller-provided buffer.  Defined in csrc/embedding.cu.
//
//   x          bf16 [M, ldx] row-major input (device pointer, 4-byte aligned,
//              ldx even)
//   out        fp32 [N] output (device pointer); out[n] = sum_m x[m, n], or
//              out[n] += that sum when accumulate != 0
//   stream     CUDA stream the two kernels are queued on
//
// Returns 0 on success, MD_NOALLOC_TOO_LARGE when the job needs more scratch
// than MD_NOALLOC_SCRATCH_FLOATS, a negative value for other bad arguments, and
// a positive cudaError_t if the set-up or a launch fails.
//
// The first call on each device looks up that device's address of the static
// array (cudaGetSymbolAddress, with the device current) and caches it; make
// that first call before any stream capture.  After a cudaDeviceReset, call
// md_colsum_noalloc_reset() so the next call looks the address up again.
// All calls on a device share the one array, so calls that may overlap on the
// GPU (different streams without ordering between them) race on it; serialise
// them.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Capacity of the static scratch array: 1 Mi floats (4 MiB) per device.
#define MD_NOALLOC_SCRATCH_FLOATS (1 << 20)
#define MD_NOALLOC_TOO_LARGE (-100)

int md_colsum_noalloc(const void* x, long long ldx, int M, int N, float* out, int accumulate, cudaStream_t stream);

// Scratch floats md_colsum / md_colsum_noalloc need for an [M, N] input
// (64-bit: the product exceeds INT_MAX for N beyond about 14.5 million).
long long md_colsum_scratch_floats(int M, int N);

// Forget the cached device addresses of the scratch array (after cudaDeviceReset).
void md_colsum_noalloc_reset(void);

#ifdef __cplusplus
}
#endif
