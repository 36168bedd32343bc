// Allocation-free entry point for the Gated DeltaNet forward.
//
// This entry point has no counterpart in the reference project; it is an
// addition of this library.
//
// rt_gdn_forward (gdn.cu) needs a caller-provided scratch workspace (the
// L2-normalised q/k and the per-chunk Gram matrices). Some callers cannot
// allocate device memory when they run the layer: an inference engine whose
// memory is owned by its own fixed pool, a latency-critical decode loop that
// cannot afford cudaMalloc's implicit device synchronisation, or a plain C
// caller (ctypes, another runtime) that has no access to PyTorch's caching
// allocator. rt_gdn_forward_noalloc serves them: the scratch lives in a
// file-scope device array, so the call allocates nothing. The caller still
// passes every input and output buffer.
//
// Preconditions (checked; a call that breaks one returns cudaErrorInvalidValue
// and launches nothing):
//   * qkv is 16-byte aligned, row_stride is a multiple of 8 elements and at
//     least (2 * Hk + Hv) * D (q | k | v of one token);
//   * Hv is a multiple of Hk, ab_stride >= Hv;
//   * a, b, out are bf16-aligned and state is float-aligned; no pointer is null.
//
// Limits and behaviour:
//   * the scratch holds RT_GDN_NOALLOC_MAX_FLOATS floats (4 MiB); calls whose
//     workspace (rt_gdn_serial_workspace_floats(B, T, Hk, D)) exceeds it return
//     cudaErrorInvalidValue before launching anything. For the 27B geometry
//     (Hk = 16, D = 128) and B = 1 that allows T <= 226 tokens per call;
//   * every GPU that loads this library keeps the 4 MiB array until the
//     process exits;
//   * the first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it; make
//     that first call before any stream capture. cudaDeviceReset invalidates
//     the cached address: after a reset, do not call this entry point again in
//     the same process;
//   * all calls share the one array and it keeps the previous call's
//     contents: every scratch value the kernels read is written earlier in the
//     same call, so nothing needs clearing, but calls that overlap on the GPU
//     (different streams without ordering) race on the scratch and must be
//     serialised by the caller.
#pragma once
#include <cuda_runtime.h>

#define RT_GDN_NOALLOC_MAX_FLOATS (1L << 20)

#ifdef __cplusplus
extern "C" {
#endif

// Capacity of the built-in scratch, in floats.
long rt_gdn_noalloc_capacity_floats();

// Same contract as rt_gdn_forward (gdn.cu) without the `work` argument.
cudaError_t rt_gdn_forward_noalloc(const void* qkv, long row_stride, const void* a, const void* b, long ab_stride,
                                   const float* A_log, const float* dt_bias, float* state, void* out, int B, int T,
                                   int Hk, int Hv, int D, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
