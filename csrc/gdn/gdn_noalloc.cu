// Allocation-free Gated DeltaNet forward: the serial path of rt_gdn_forward
// (rt_gdn_forward_serial, the one with the smallest scratch) with its scratch in
// a file-scope device array. See gdn_noalloc.h for who needs it, the size
// limit and the sharing rules. This entry point has no counterpart in the
// reference project.
#include "gdn_noalloc.h"
#include "../api.h"

#include <atomic>
#include <stdint.h>

namespace {

// The scratch itself. In host code this name is only a stand-in for the
// device symbol: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_gdn_scratch[RT_GDN_NOALLOC_MAX_FLOATS];

constexpr int kMaxDevices = 64;
// Per-device cache of the resolved address. Atomic so that first calls from several host threads are not a data
// race: two threads may both resolve the address, and they store the same value.
std::atomic<float*> g_scratch_ptr[kMaxDevices];

// Resolves (once per device, with that device current) the scratch's device address.
cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  float* cached = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (!cached) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_gdn_scratch);
    if (err != cudaSuccess) return err;
    cached = static_cast<float*>(ptr);
    g_scratch_ptr[dev].store(cached, std::memory_order_release);
  }
  *out = cached;
  return cudaSuccess;
}

bool aligned(const void* p, uintptr_t bytes) { return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0; }

}  // namespace

extern "C" long rt_gdn_noalloc_capacity_floats() { return RT_GDN_NOALLOC_MAX_FLOATS; }

extern "C" cudaError_t rt_gdn_forward_noalloc(const void* qkv, long row_stride, const void* a, const void* b,
                                              long ab_stride, const float* A_log, const float* dt_bias,
                                              float* state, void* out, int B, int T, int Hk, int Hv, int D,
                                              cudaStream_t stream) {
  if (B <= 0 || T <= 0 || Hk <= 0 || Hv <= 0 || D <= 0) return cudaErrorInvalidValue;
  if (!qkv || !a || !b || !A_log || !dt_bias || !state || !out) return cudaErrorInvalidValue;
  // The kernels copy v rows of qkv 16 bytes at a time and read a / b as bf16 scalars.
  if (Hv % Hk != 0 || row_stride % 8 != 0 || row_stride < (long)(2 * Hk + Hv) * D || ab_stride < Hv)
    return cudaErrorInvalidValue;
  if (!aligned(qkv, 16) || !aligned(a, 2) || !aligned(b, 2) || !aligned(state, 4) || !aligned(out, 2))
    return cudaErrorInvalidValue;
  if (rt_gdn_serial_workspace_floats(B, T, Hk, D) > RT_GDN_NOALLOC_MAX_FLOATS) return cudaErrorInvalidValue;
  float* work = nullptr;
  cudaError_t err = scratch_for_current_device(&work);
  if (err != cudaSuccess) return err;
  return rt_gdn_forward_serial(qkv, row_stride, a, b, ab_stride, A_log, dt_bias, state, out, work, B, T, Hk, Hv, D,
                               stream);
}
