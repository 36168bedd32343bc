// WKV7 token-by-token update for decoding (T small, no checkpoints), sm_100a.
// The recurrence is RWKV7's (RWKV-LM, Apache-2.0; see NOTICE at the project root); this code is our own.
//
// Per (batch, head) one CTA of N threads; thread i owns value row i of the fp32 state S[i][:] in registers:
//   sa = S[i] . a_t,   S[i][j] = S[i][j] d_t[j] + sa b_t[j] + v_t[i] k_t[j],   y_t[i] = S[i] . r_t,
// d = exp(-e^{-1/2} sigmoid(w)) (same decay parameterisation as the chunked kernel and the reference's
// kernels/wkv7_state.cu:12-40). The per-token vectors (r, d, k, a, b) are staged in shared memory once per
// step and read as broadcasts. State traffic is one read and one write of the state per call, so a decode
// step is bandwidth-bound on the state (B*H*N*N*8 bytes).
#include "../common/common.cuh"

namespace {

constexpr float DECAY_SCALE = 0.6065306597126334f;

template <typename T, int N>
__global__ void __launch_bounds__(N)
wkv7_step_kernel(int T_, int H, const T* __restrict__ r, const T* __restrict__ w, const T* __restrict__ k,
                 const T* __restrict__ v, const T* __restrict__ a, const T* __restrict__ b,
                 const float* __restrict__ s0, T* __restrict__ y, float* __restrict__ s_end) {
  __shared__ float vec[5][N];  // r, d, k, a, b
  const int bh = blockIdx.x, bi = bh / H, h = bh % H, i = threadIdx.x;
  const float* src = s0 + (long)bh * N * N + (long)i * N;
  float s[N];
#pragma unroll
  for (int j = 0; j < N; j += 4) {
    const float4 q = *reinterpret_cast<const float4*>(src + j);
    s[j] = q.x; s[j + 1] = q.y; s[j + 2] = q.z; s[j + 3] = q.w;
  }
  for (int t = 0; t < T_; ++t) {
    const long off = (((long)bi * T_ + t) * H + h) * N;
    __syncthreads();  // previous step's vectors consumed
    vec[0][i] = rt::to_f(r[off + i]);
    vec[1][i] = expf(-DECAY_SCALE * rt::sigmoidf_(rt::to_f(w[off + i])));
    vec[2][i] = rt::to_f(k[off + i]);
    vec[3][i] = rt::to_f(a[off + i]);
    vec[4][i] = rt::to_f(b[off + i]);
    const float vi = rt::to_f(v[off + i]);
    __syncthreads();
    float sa = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) sa += s[j] * vec[3][j];
    float out = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      s[j] = s[j] * vec[1][j] + sa * vec[4][j] + vi * vec[2][j];
      out += s[j] * vec[0][j];
    }
    y[off + i] = rt::from_f<T>(out);
  }
  float* dst = s_end + (long)bh * N * N + (long)i * N;
#pragma unroll
  for (int j = 0; j < N; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(s[j], s[j + 1], s[j + 2], s[j + 3]);
}

template <typename T, int N>
cudaError_t launch(int B, int T_, int H, const void* r, const void* w, const void* k, const void* v, const void* a,
                   const void* b, const float* s0, void* y, float* s_end, cudaStream_t stream) {
  wkv7_step_kernel<T, N><<<B * H, N, 0, stream>>>(T_, H, (const T*)r, (const T*)w, (const T*)k, (const T*)v,
                                                   (const T*)a, (const T*)b, s0, (T*)y, s_end);
  return cudaGetLastError();
}

}  // namespace

// Head sizes 32, 64 and 128; returns cudaErrorInvalidValue for others (callers use the chunked kernel).
extern "C" cudaError_t rt_wkv7_step(int dtype, int B, int T_, int H, int N, const void* r, const void* w,
                                    const void* k, const void* v, const void* a, const void* b, const float* s0,
                                    void* y, float* s_end, cudaStream_t stream) {
#define RT_STEP(TYPE)                                                                                    \
  switch (N) {                                                                                           \
    case 32: return launch<TYPE, 32>(B, T_, H, r, w, k, v, a, b, s0, y, s_end, stream);                 \
    case 64: return launch<TYPE, 64>(B, T_, H, r, w, k, v, a, b, s0, y, s_end, stream);                 \
    case 128: return launch<TYPE, 128>(B, T_, H, r, w, k, v, a, b, s0, y, s_end, stream);               \
    default: return cudaErrorInvalidValue;                                                               \
  }
  if (dtype == 1) { RT_STEP(__nv_bfloat16) }
  RT_STEP(float)
#undef RT_STEP
}
