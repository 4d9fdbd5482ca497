// C entry point of the tcgen05 bf16 GEMM that allocates no device memory.
//
// This interface has no counterpart in the reference; it exists for callers that must not allocate:
// code running inside another framework's memory pool or arena, a custom allocator's own bring-up,
// or an embedding host that owns every byte of device memory and forbids hidden cudaMalloc calls.
// The torch op `r9k::gemm_bf16` computes the same product but takes its split-K workspace as a
// caller-allocated tensor; this entry point instead keeps its split-K scratch in one fixed-size
// array of device memory that is part of the library image.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Result codes (0 = the kernel was launched).
enum {
  R9K_NOALLOC_OK = 0,
  R9K_NOALLOC_EINVAL = -1,     // bad pointer, shape, stride or alignment
  R9K_NOALLOC_ETOOLARGE = -2,  // M > 64, or the split-K scratch this shape needs exceeds the fixed array
  R9K_NOALLOC_ESETUP = -3,     // the per-device set-up failed (scratch address, kernel attributes, TMA encoder)
  R9K_NOALLOC_ELAUNCH = -4,    // the kernel launch itself failed
};

// Size of the fixed scratch array, in bytes, per device: 4 KiB of split-K tile counters, then the
// fp32 split-K partials.
#define R9K_NOALLOC_SCRATCH_BYTES (10u << 20)

// out[M, N] (bf16, row stride ldo elements) = alpha * x[M, K] @ w[N, K]^T, x and w bf16 row-major
// with row strides ldx, ldw (elements). A skinny (decode-sized) GEMM: 1 <= M <= 64, K a multiple of
// 64, every base pointer (w, x, out) 16-byte aligned and every row stride (ldw, ldx, ldo) a multiple
// of 8 elements; anything else returns R9K_NOALLOC_EINVAL. The launch goes on `stream` in ordinary
// stream order (the kernel starts after all earlier work on `stream` has finished, so w and x may be
// written by the kernel just before it) and the call returns without synchronising.
//
// status: optional device pointer to 4 ints; a kernel whose bounded wait runs out writes
// {code, kernel id, block, detail} there (first error wins) and returns. NULL records nothing.
//
// Scratch: all calls on one device share the library's single scratch array. Its tile counters
// must be zero when a kernel starts: they are zero when the library loads and every kernel that
// completes leaves them at zero, but a kernel that gave up on a timeout (nonzero status) may leave
// them dirty, after which further calls in the process are not reliable. Calls that can overlap
// in time (different streams, or host threads without ordering) race on the array and give wrong
// results; order them on one stream.
//
// Set-up: the first call on each device (with that device current) looks up the scratch address,
// sets the kernels' shared-memory limits and resolves the TMA encoder; make that first call
// before any stream capture begins. Later calls make no CUDA runtime calls besides the launch.
int r9k_gemm_bf16_noalloc(const void* w, int64_t ldw, const void* x, int64_t ldx, void* out, int64_t ldo,
                          int N, int M, int K, float alpha, int* status, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
