// Shared device helpers for the sm_100a kernels of this package.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define RT_DEVICE __device__ __forceinline__

namespace rt {

enum class DType : int { F32 = 0, BF16 = 1 };

template <typename T> RT_DEVICE float to_f(T v);
template <> RT_DEVICE float to_f<float>(float v) { return v; }
template <> RT_DEVICE float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> RT_DEVICE T from_f(float v);
template <> RT_DEVICE float from_f<float>(float v) { return v; }
template <> RT_DEVICE __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

RT_DEVICE float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }
RT_DEVICE float siluf_(float x) { return x / (1.f + expf(-x)); }

// 8 bf16 values in one 16-byte word <-> 8 floats
RT_DEVICE void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(p[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}
RT_DEVICE uint4 pack8(const float* f) {
  uint4 u;
  __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

RT_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024). `scratch` holds >= 32 floats.
RT_DEVICE float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  const int warps = (blockDim.x + 31) >> 5;
  v = (threadIdx.x < warps) ? scratch[threadIdx.x] : 0.f;
  if (warp == 0) v = warp_sum(v);
  if (threadIdx.x == 0) scratch[0] = v;
  __syncthreads();
  v = scratch[0];
  __syncthreads();
  return v;
}

// Asynchronous 16-byte global->shared copy (zero-filled when !pred; gmem must still be a valid address).
RT_DEVICE void cp_async16(void* smem, const void* gmem, bool pred) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
RT_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
RT_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

}  // namespace rt

// Host-side status helpers.
#define RT_CUDA_CHECK(expr)                                                                   \
  do {                                                                                        \
    cudaError_t err__ = (expr);                                                               \
    if (err__ != cudaSuccess) return err__;                                                   \
  } while (0)
