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
#include <type_traits>

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

// Register-resident variant: rows of C % 8 == 0 with 16-byte aligned operands; each of the 128
// threads keeps V 8-value words of the row (C <= 8192), so x and h are read once and w once per word.
template <bool ADD, int V>
__global__ void __launch_bounds__(128) rmsnorm_vec_kernel(const uint4* __restrict__ x, const uint4* __restrict__ h,
                                                          const float4* __restrict__ w, uint4* __restrict__ sum_out,
                                                          uint4* __restrict__ out, int C8, float eps) {
  __shared__ float scratch[32];
  const long row = blockIdx.x;
  float v[V][8];
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int c = threadIdx.x + 128 * j;
    if (c < C8) {
      rt::unpack8(x[row * C8 + c], v[j]);
      if (ADD) {
        float a[8];
        rt::unpack8(h[row * C8 + c], a);
#pragma unroll
        for (int u = 0; u < 8; ++u) v[j][u] = __bfloat162float(__float2bfloat16_rn(v[j][u] + a[u]));
        sum_out[row * C8 + c] = rt::pack8(v[j]);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) acc += v[j][u] * v[j][u];
    }
  }
  const float inv = rsqrtf(rt::block_sum(acc, scratch) / (8 * C8) + eps);
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int c = threadIdx.x + 128 * j;
    if (c < C8) {
      const float4 w0 = w[2 * c], w1 = w[2 * c + 1];
      const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      float o[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) o[u] = v[j][u] * inv * (1.f + ww[u]);
      out[row * C8 + c] = rt::pack8(o);
    }
  }
}

// ---------------------------------------------------------------- conv1d + SiLU
// x: [B, T, C] bf16; state: [B, K-1, C] bf16 (oldest first); weight: [C, K] fp32 (tap K-1 = newest).
// Each thread owns one channel and a segment of SEG time steps.
constexpr int SEG = 64;
__global__ void conv1d_silu_kernel(const bf16* __restrict__ x, long xs, const bf16* __restrict__ state,
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
    win[j] = t >= 0 ? rt::to_f(x[((long)b * T + t) * xs + c]) : rt::to_f(state[((long)b * (K - 1) + (t + K - 1)) * C + c]);
  }
  const int t1 = min(T, t0 + SEG);
  for (int t = t0; t < t1; ++t) {
    const float cur = rt::to_f(x[((long)b * T + t) * xs + c]);
    float acc = cur * wt[K - 1];
    for (int j = 0; j < K - 1; ++j) acc += win[j] * wt[j];
    for (int j = 0; j + 1 < K - 1; ++j) win[j] = win[j + 1];
    if (K > 1) win[K - 2] = cur;
    y[((long)b * T + t) * C + c] = __float2bfloat16_rn(rt::siluf_(acc));
  }
  if (t1 == T) {  // the segment holding the last K-1 inputs writes the carried window
    for (int j = 0; j < K - 1; ++j) {
      const int t = T - (K - 1) + j;
      const float v = t >= 0 ? rt::to_f(x[((long)b * T + t) * xs + c])
                             : rt::to_f(state[((long)b * (K - 1) + (t + K - 1)) * C + c]);
      new_state[((long)b * (K - 1) + j) * C + c] = __float2bfloat16_rn(v);
    }
  }
}

// Vectorised variant (C % 8 == 0, 16-byte aligned rows): a thread owns 8 channels and CSEG steps. All
// K-1+CSEG input words of the segment are loaded up front (CSEG+K-1 16-byte loads in flight per
// thread), then the taps run from registers; K is a template parameter so nothing spills.
constexpr int CSEG = 16;
template <int K>
__global__ void __launch_bounds__(128) conv1d_silu_vec_kernel(const uint4* __restrict__ x, long xs8,
                                                              const uint4* __restrict__ state,
                                                              const float* __restrict__ weight, uint4* __restrict__ y,
                                                              uint4* __restrict__ new_state, int T, int C8) {
  constexpr int H = K - 1;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int t0 = blockIdx.y * CSEG, b = blockIdx.z;
  if (c >= C8) return;
  uint4 raw[H + CSEG];
#pragma unroll
  for (int j = 0; j < H + CSEG; ++j) {
    const int t = t0 - H + j;
    raw[j] = t < 0 ? state[((long)b * H + (t + H)) * C8 + c]
                   : (t < T ? x[((long)b * T + t) * xs8 + c] : make_uint4(0u, 0u, 0u, 0u));
  }
  float wt[K][8];
#pragma unroll
  for (int u = 0; u < 8; ++u)
#pragma unroll
    for (int j = 0; j < K; ++j) wt[j][u] = weight[(8 * c + u) * K + j];
#pragma unroll
  for (int i = 0; i < CSEG; ++i) {
    if (t0 + i < T) {
      float o[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) o[u] = 0.f;
#pragma unroll
      for (int j = 0; j < K; ++j) {
        float v[8];
        rt::unpack8(raw[i + j], v);
#pragma unroll
        for (int u = 0; u < 8; ++u) o[u] += v[u] * wt[j][u];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) o[u] = rt::siluf_(o[u]);
      y[((long)b * T + t0 + i) * C8 + c] = rt::pack8(o);
    }
  }
  if (t0 + CSEG >= T) {  // the segment holding step T-1 writes the carried window: inputs T-H .. T-1,
                         // all inside this segment's loaded range t0-H .. t0+CSEG-1
#pragma unroll
    for (int k = 0; k < H + CSEG; ++k) {
      const int t = t0 - H + k;
      if (t >= T - H && t < T) new_state[((long)b * H + (t - (T - H))) * C8 + c] = raw[k];
    }
  }
}

// ---------------------------------------------------------------- gated RMSNorm (GDN output)
// rows of D (<= 256) values; one warp per row.
__global__ void gated_rmsnorm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ z, const float* __restrict__ w,
                                     bf16* __restrict__ out, long rows, int D, int heads, long zs, float eps) {
  const long row = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const bf16* zr = z + (row / heads) * zs + (row % heads) * D;  // z rows: one token of `heads` heads, stride zs
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
      out[row * D + c] = __float2bfloat16_rn(p * rt::siluf_(rt::to_f(zr[c])));
    }
  }
}

// ---------------------------------------------------------------- q/k norm + RoPE + cache write
// One warp per (token, head) row of D <= 256 values. src rows have stride `src_stride` elements;
// rotate_half RoPE on the first `rot` dims with angle pos * inv_freq[i mod rot/2].
__global__ void norm_rope_kernel(const bf16* __restrict__ src, long src_stride, long head_stride,
                                 const float* __restrict__ w, const float* __restrict__ inv_freq, bf16* __restrict__ dst,
                                 int heads, int T, long dst_batch_stride, int pos0, int D, int rot, float eps,
                                 long rows) {
  extern __shared__ float buf[];
  const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * (blockDim.x >> 5) + wib;
  if (row >= rows) return;
  float* s = buf + wib * D;
  const int head = row % heads;
  const long bt = row / heads;
  const int t = bt % T;
  const long b = bt / T;
  const bf16* in = src + bt * src_stride + (long)head * head_stride;
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

// out[row] = table[ids[row]] (bf16 rows of `width`, 16-byte moves); ids outside [0, vocab) give a zero row.
__global__ void embed_rows_kernel(const long* __restrict__ ids, const bf16* __restrict__ table, long vocab,
                                  bf16* __restrict__ out, int width, long rows) {
  const long row = blockIdx.x;
  if (row >= rows) return;
  const long id = ids[row];
  uint4* o = reinterpret_cast<uint4*>(out + row * (long)width);
  if (id < 0 || id >= vocab) {
    for (int c = threadIdx.x; c < width / 8; c += blockDim.x) o[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* in = reinterpret_cast<const uint4*>(table + id * (long)width);
  for (int c = threadIdx.x; c < width / 8; c += blockDim.x) o[c] = __ldg(in + c);
}

}  // namespace

extern "C" cudaError_t rt_rmsnorm_1p(const void* x, const void* h, const float* w, void* sum_out, void* out, long rows,
                                     int C, float eps, cudaStream_t stream) {
  const bool vec = C % 8 == 0 && C <= 8192 && ((uintptr_t)x | (uintptr_t)h | (uintptr_t)w | (uintptr_t)sum_out |
                                                (uintptr_t)out) % 16 == 0;
  if (vec) {
    const int C8 = C / 8, V = (C8 + 127) / 128;
    auto go = [&](auto add, auto v) {
      rmsnorm_vec_kernel<decltype(add)::value, decltype(v)::value><<<rows, 128, 0, stream>>>(
          (const uint4*)x, (const uint4*)h, (const float4*)w, (uint4*)sum_out, (uint4*)out, C8, eps);
    };
#define RT_RMS_V(n)                                                                      \
  case n:                                                                                \
    h ? go(std::true_type{}, std::integral_constant<int, n>{})                           \
      : go(std::false_type{}, std::integral_constant<int, n>{});                         \
    break;
    switch (V) { RT_RMS_V(1) RT_RMS_V(2) RT_RMS_V(3) RT_RMS_V(4) RT_RMS_V(5) RT_RMS_V(6) RT_RMS_V(7) RT_RMS_V(8) }
#undef RT_RMS_V
    return cudaGetLastError();
  }
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

extern "C" cudaError_t rt_conv1d_silu(const void* x, long xs, const void* state, const float* weight, void* y,
                                      void* new_state, int B, int T, int C, int K, cudaStream_t stream) {
  if (K < 1 || K > 8 || xs < C) return cudaErrorInvalidValue;
  if (C % 8 == 0 && xs % 8 == 0 && (K == 4 || K == 2 || K == 3) &&
      ((uintptr_t)x | (uintptr_t)state | (uintptr_t)y | (uintptr_t)new_state) % 16 == 0) {
    const int C8 = C / 8;
    const dim3 g((C8 + 127) / 128, (T + CSEG - 1) / CSEG, B);
    auto go = [&](auto k) {
      conv1d_silu_vec_kernel<decltype(k)::value><<<g, 128, 0, stream>>>(
          (const uint4*)x, xs / 8, (const uint4*)state, weight, (uint4*)y, (uint4*)new_state, T, C8);
    };
    if (K == 4) go(std::integral_constant<int, 4>{});
    else if (K == 3) go(std::integral_constant<int, 3>{});
    else go(std::integral_constant<int, 2>{});
    return cudaGetLastError();
  }
  dim3 grid((C + 127) / 128, (T + SEG - 1) / SEG, B);
  conv1d_silu_kernel<<<grid, 128, 0, stream>>>((const bf16*)x, xs, (const bf16*)state, weight, (bf16*)y,
                                               (bf16*)new_state, T, C, K);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_gated_rmsnorm(const void* x, const void* z, const float* w, void* out, long rows, int D,
                                        int heads, long zs, float eps, cudaStream_t stream) {
  if (D > 256 || heads < 1) return cudaErrorInvalidValue;
  const int warps = 8;
  gated_rmsnorm_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, stream>>>((const bf16*)x, (const bf16*)z, w,
                                                                               (bf16*)out, rows, D, heads, zs, eps);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_norm_rope(const void* src, long src_stride, long head_stride, const float* w,
                                    const float* inv_freq, void* dst, int B, int T, int heads, long dst_batch_stride,
                                    int pos0, int D, int rot, float eps, cudaStream_t stream) {
  if (D > 256 || (rot & 1)) return cudaErrorInvalidValue;
  const long rows = (long)B * T * heads;
  const int warps = 4;
  norm_rope_kernel<<<(rows + warps - 1) / warps, warps * 32, warps * D * sizeof(float), stream>>>(
      (const bf16*)src, src_stride, head_stride, w, inv_freq, (bf16*)dst, heads, T, dst_batch_stride, pos0, D, rot, eps,
      rows);
  return cudaGetLastError();
}

// Embedding lookup: out [rows, width] bf16 = table [vocab, width] rows at ids (int64).
extern "C" cudaError_t rt_embed_rows(const long* ids, const void* table, long vocab, void* out, int width, long rows,
                                     cudaStream_t stream) {
  if (width % 8 || (reinterpret_cast<uintptr_t>(table) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return cudaErrorInvalidValue;
  if (rows <= 0) return cudaSuccess;
  embed_rows_kernel<<<rows, 128, 0, stream>>>(ids, (const bf16*)table, vocab, (bf16*)out, width, rows);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_copy_rows(const void* src, long src_stride, void* dst, int B, int T, long dst_batch_stride,
                                    int width, cudaStream_t stream) {
  if (width % 8 || src_stride % 8) return cudaErrorInvalidValue;
  const long rows = (long)B * T;
  copy_rows_kernel<<<rows, 128, 0, stream>>>((const bf16*)src, src_stride, (bf16*)dst, T, dst_batch_stride, width, rows);
  return cudaGetLastError();
}
