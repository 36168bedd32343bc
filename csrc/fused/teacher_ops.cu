// Memory-bound teacher-block kernels for sm_100a (bf16 activations, fp32 math):
//   * Qwen RMSNorm with (1 + w) scaling, optionally fused with the residual add
//     that precedes it (sum rounded to bf16 first, as the model does);
//   * causal depthwise conv1d (kernel K <= 8) + SiLU with the convolution
//     window carried across chunks;
//   * GDN output norm: w * RMSNorm(x) (bf16) times SiLU(z);
//   * attention pre-processing: per-head RMSNorm of q/k, partial RoPE, and the
//     write of k/v into the KV cache at the chunk's positions.
// Each kernel streams its operands once (vectorised 16-byte accesses where
// the row length allows) and keeps intermediate values in registers or
// shared memory.
#include "../common/common.cuh"

namespace {

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------- RMSNorm (1 + w)
template <bool ADD>
__global__ void rmsnorm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ h, const float* __restrict__ w,
                               bf16* __restrict__ sum_out, bf16* __restrict__ out, int C, float eps) {
  extern __shared__ float srow[];
  __shared__ float scratch[32];
  const long row = blockIdx.x;
  const bf16* xr = x + row * C;
  float acc = 0.f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float v = rt::to_f(xr[c]);
    if (ADD) {
      v = __bfloat162float(__float2bfloat16_rn(v + rt::to_f(h[row * C + c])));
      sum_out[row * C + c] = __float2bfloat16_rn(v);
    }
    srow[c] = v;
    acc += v * v;
  }
  const float total = rt::block_sum(acc, scratch);
  const float inv = rsqrtf(total / C + eps);
  for (int c = threadIdx.x; c < C; c += blockDim.x) out[row * C + c] = __float2bfloat16_rn(srow[c] * inv * (1.f + w[c]));
}

// ---------------------------------------------------------------- conv1d + SiLU
// x: [B, T, C] bf16; state: [B, K-1, C] bf16 (oldest first); weight: [C, K] fp32 (tap K-1 = newest).
// Each thread owns one channel and a segment of SEG time steps.
constexpr int SEG = 64;
__global__ void conv1d_silu_kernel(const bf16* __restrict__ x, const bf16* __restrict__ state,
                                   const float* __restrict__ weight, bf16* __restrict__ y, bf16* __restrict__ new_state,
                                   int T, int C, int K) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int t0 = blockIdx.y * SEG;
  const int b = blockIdx.z;
  if (c >= C) return;
  float win[8];
  float wt[8];
  for (int j = 0; j < K; ++j) wt[j] = weight[c * K + j];
  // Window holds inputs t0-(K-1) .. t0-1.
  for (int j = 0; j < K - 1; ++j) {
    const int t = t0 - (K - 1) + j;
    win[j] = t >= 0 ? rt::to_f(x[((long)b * T + t) * C + c]) : rt::to_f(state[((long)b * (K - 1) + (t + K - 1)) * C + c]);
  }
  const int t1 = min(T, t0 + SEG);
  for (int t = t0; t < t1; ++t) {
    const float cur = rt::to_f(x[((long)b * T + t) * C + c]);
    float acc = cur * wt[K - 1];
    for (int j = 0; j < K - 1; ++j) acc += win[j] * wt[j];
    for (int j = 0; j + 1 < K - 1; ++j) win[j] = win[j + 1];
    if (K > 1) win[K - 2] = cur;
    y[((long)b * T + t) * C + c] = __float2bfloat16_rn(rt::siluf_(acc));
  }
  if (t1 == T) {  // the segment holding the last K-1 inputs writes the carried window
    for (int j = 0; j < K - 1; ++j) {
      const int t = T - (K - 1) + j;
      const float v = t >= 0 ? rt::to_f(x[((long)b * T + t) * C + c])
                             : rt::to_f(state[((long)b * (K - 1) + (t + K - 1)) * C + c]);
      new_state[((long)b * (K - 1) + j) * C + c] = __float2bfloat16_rn(v);
    }
  }
}

// ---------------------------------------------------------------- gated RMSNorm (GDN output)
// rows of D (<= 256) values; one warp per row.
__global__ void gated_rmsnorm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ z, const float* __restrict__ w,
                                     bf16* __restrict__ out, long rows, int D, float eps) {
  const long row = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[8];
  float acc = 0.f;
  for (int j = 0; j < 8; ++j) {
    const int c = lane + 32 * j;
    v[j] = c < D ? rt::to_f(x[row * D + c]) : 0.f;
    acc += v[j] * v[j];
  }
  acc = rt::warp_sum(acc);
  const float inv = rsqrtf(acc / D + eps);
  for (int j = 0; j < 8; ++j) {
    const int c = lane + 32 * j;
    if (c < D) {
      const float n = __bfloat162float(__float2bfloat16_rn(v[j] * inv));
      const float p = __bfloat162float(__float2bfloat16_rn(w[c] * n));
      out[row * D + c] = __float2bfloat16_rn(p * rt::siluf_(rt::to_f(z[row * D + c])));
    }
  }
}

// ---------------------------------------------------------------- q/k norm + RoPE + cache write
// One warp per (token, head) row of D <= 256 values. src rows have stride `src_stride` elements;
// rotate_half RoPE on the first `rot` dims with angle pos * inv_freq[i mod rot/2].
__global__ void norm_rope_kernel(const bf16* __restrict__ src, long src_stride, const float* __restrict__ w,
                                 const float* __restrict__ inv_freq, bf16* __restrict__ dst, int heads, int T,
                                 long dst_batch_stride, int pos0, int D, int rot, float eps, long rows) {
  extern __shared__ float buf[];
  const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * (blockDim.x >> 5) + wib;
  if (row >= rows) return;
  float* s = buf + wib * D;
  const int head = row % heads;
  const long bt = row / heads;
  const int t = bt % T;
  const long b = bt / T;
  const bf16* in = src + bt * src_stride + (long)head * (src_stride / heads);
  float acc = 0.f;
  for (int c = lane; c < D; c += 32) {
    const float v = rt::to_f(in[c]);
    s[c] = v;
    acc += v * v;
  }
  acc = rt::warp_sum(acc);
  const float inv = rsqrtf(acc / D + eps);
  __syncwarp();
  for (int c = lane; c < D; c += 32) s[c] = s[c] * inv * (1.f + w[c]);
  __syncwarp();
  const int half = rot / 2;
  const float pos = (float)(pos0 + t);
  bf16* out = dst + b * dst_batch_stride + ((long)t * heads + head) * D;
  for (int c = lane; c < D; c += 32) {
    float o = s[c];
    if (c < rot) {
      const int i = c < half ? c : c - half;
      float sn, cs;
      sincosf(pos * inv_freq[i], &sn, &cs);
      const float partner = c < half ? -s[c + half] : s[c - half];
      o = s[c] * cs + partner * sn;
    }
    out[c] = __float2bfloat16_rn(o);
  }
}

// v rows [B*T, heads*D] (row stride src_stride) into cache [B, cap, heads, D] at pos0.
__global__ void copy_rows_kernel(const bf16* __restrict__ src, long src_stride, bf16* __restrict__ dst, int T,
                                 long dst_batch_stride, int width, long rows) {
  const long row = blockIdx.x;
  if (row >= rows) return;
  const long b = row / T;
  const int t = row % T;
  const uint4* in = reinterpret_cast<const uint4*>(src + row * src_stride);
  uint4* out = reinterpret_cast<uint4*>(dst + b * dst_batch_stride + (long)t * width);
  for (int c = threadIdx.x; c < width / 8; c += blockDim.x) out[c] = in[c];
}

}  // namespace

extern "C" cudaError_t rt_rmsnorm_1p(const void* x, const void* h, const float* w, void* sum_out, void* out, long rows,
                                     int C, float eps, cudaStream_t stream) {
  const size_t smem = (size_t)C * sizeof(float);
  if (smem > 48 * 1024) {  // only rows wider than 12288 need the opt-in (set once per width class)
    RT_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    RT_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  if (h) {
    rmsnorm_kernel<true><<<rows, 256, smem, stream>>>((const bf16*)x, (const bf16*)h, w, (bf16*)sum_out, (bf16*)out, C, eps);
  } else {
    rmsnorm_kernel<false><<<rows, 256, smem, stream>>>((const bf16*)x, nullptr, w, nullptr, (bf16*)out, C, eps);
  }
  return cudaGetLastError();
}

extern "C" cudaError_t rt_conv1d_silu(const void* x, const void* state, const float* weight, void* y, void* new_state,
                                      int B, int T, int C, int K, cudaStream_t stream) {
  if (K < 1 || K > 8) return cudaErrorInvalidValue;
  dim3 grid((C + 127) / 128, (T + SEG - 1) / SEG, B);
  conv1d_silu_kernel<<<grid, 128, 0, stream>>>((const bf16*)x, (const bf16*)state, weight, (bf16*)y, (bf16*)new_state,
                                               T, C, K);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_gated_rmsnorm(const void* x, const void* z, const float* w, void* out, long rows, int D,
                                        float eps, cudaStream_t stream) {
  if (D > 256) return cudaErrorInvalidValue;
  const int warps = 8;
  gated_rmsnorm_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, stream>>>((const bf16*)x, (const bf16*)z, w,
                                                                               (bf16*)out, rows, D, eps);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_norm_rope(const void* src, long src_stride, const float* w, const float* inv_freq, void* dst,
                                    int B, int T, int heads, long dst_batch_stride, int pos0, int D, int rot, float eps,
                                    cudaStream_t stream) {
  if (D > 256 || (rot & 1)) return cudaErrorInvalidValue;
  const long rows = (long)B * T * heads;
  const int warps = 4;
  norm_rope_kernel<<<(rows + warps - 1) / warps, warps * 32, warps * D * sizeof(float), stream>>>(
      (const bf16*)src, src_stride, w, inv_freq, (bf16*)dst, heads, T, dst_batch_stride, pos0, D, rot, eps, rows);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_copy_rows(const void* src, long src_stride, void* dst, int B, int T, long dst_batch_stride,
                                    int width, cudaStream_t stream) {
  if (width % 8 || src_stride % 8) return cudaErrorInvalidValue;
  const long rows = (long)B * T;
  copy_rows_kernel<<<rows, 128, 0, stream>>>((const bf16*)src, src_stride, (bf16*)dst, T, dst_batch_stride, width, rows);
  return cudaGetLastError();
}
