// Gated DeltaNet token-by-token update for decoding (T small), sm_100a.
//
// Per (batch, value head) one CTA of D threads; thread i owns value column i of the fp32 state S[:, i]
// (the [B, Hv, Dk, Dv] cache layout, so each key row j is a coalesced 4*D-byte access):
//   kv_i = sum_j S[j][i] k_j,   Vt_i = beta (v_i - e^g kv_i),   S[j][i] = e^g S[j][i] + k_j Vt_i,
//   o_i = sum_j S[j][i] q_j,
// with q, k L2-normalised (eps 1e-6, q scaled by D^-1/2), g = -exp(A_log) softplus(a + dt_bias) and
// beta = sigmoid(b) rounded to bf16 -- the same definitions as the chunked kernels.
#include "../common/common.cuh"

namespace {

using bf16 = __nv_bfloat16;

template <int D>
__global__ void __launch_bounds__(D)
gdn_step_kernel(const bf16* __restrict__ qkv, long row_stride, const bf16* __restrict__ pa,
                const bf16* __restrict__ pb, long ab_stride, const float* __restrict__ A_log,
                const float* __restrict__ dt_bias, float* __restrict__ state, bf16* __restrict__ out, int T, int Hk,
                int Hv) {
  __shared__ float qs[D], ks[D], red[2][D / 32];
  const int b = blockIdx.x / Hv, h = blockIdx.x % Hv, i = threadIdx.x;
  const int kh = h / (Hv / Hk);
  const int lane = i & 31, warp = i >> 5;
  float* st = state + ((long)b * Hv + h) * D * D;
  float s[D];
#pragma unroll
  for (int j = 0; j < D; ++j) s[j] = st[(long)j * D + i];
  const float neg_a = -expf(A_log[h]), dtb = dt_bias[h];
  for (int t = 0; t < T; ++t) {
    const bf16* row = qkv + ((long)b * T + t) * row_stride;
    const float q = rt::to_f(row[(long)kh * D + i]);
    const float k = rt::to_f(row[(long)(Hk + kh) * D + i]);
    const float v = rt::to_f(row[2L * Hk * D + (long)h * D + i]);
    const float q2 = rt::warp_sum(q * q), k2 = rt::warp_sum(k * k);
    __syncthreads();  // previous step's qs/ks/red consumed
    if (lane == 0) {
      red[0][warp] = q2;
      red[1][warp] = k2;
    }
    __syncthreads();
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int w = 0; w < D / 32; ++w) {
      sq += red[0][w];
      sk += red[1][w];
    }
    qs[i] = q * rsqrtf(sq + 1e-6f) * rsqrtf((float)D);
    ks[i] = k * rsqrtf(sk + 1e-6f);
    const long gr = ((long)b * T + t) * ab_stride + h;
    const float av = rt::to_f(pa[gr]) + dtb;
    const float eg = expf(neg_a * (av > 20.f ? av : log1pf(expf(av))));
    const float beta = __bfloat162float(__float2bfloat16_rn(rt::sigmoidf_(rt::to_f(pb[gr]))));
    __syncthreads();
    float kv = 0.f;
#pragma unroll
    for (int j = 0; j < D; ++j) kv += s[j] * ks[j];
    const float vt = beta * (v - eg * kv);
    float o = 0.f;
#pragma unroll
    for (int j = 0; j < D; ++j) {
      s[j] = eg * s[j] + ks[j] * vt;
      o += s[j] * qs[j];
    }
    out[(((long)b * T + t) * Hv + h) * D + i] = __float2bfloat16_rn(o);
  }
#pragma unroll
  for (int j = 0; j < D; ++j) st[(long)j * D + i] = s[j];
}

}  // namespace

// Same contract as rt_gdn_forward (no workspace); D = 64 or 128, otherwise cudaErrorInvalidValue.
extern "C" cudaError_t rt_gdn_step(const void* qkv, long row_stride, const void* a, const void* b, long ab_stride,
                                   const float* A_log, const float* dt_bias, float* state, void* out, int B, int T,
                                   int Hk, int Hv, int D, cudaStream_t stream) {
  if (Hv % Hk) return cudaErrorInvalidValue;
  switch (D) {
    case 128:
      gdn_step_kernel<128><<<B * Hv, 128, 0, stream>>>((const bf16*)qkv, row_stride, (const bf16*)a, (const bf16*)b,
                                                        ab_stride, A_log, dt_bias, state, (bf16*)out, T, Hk, Hv);
      break;
    case 64:
      gdn_step_kernel<64><<<B * Hv, 64, 0, stream>>>((const bf16*)qkv, row_stride, (const bf16*)a, (const bf16*)b,
                                                      ab_stride, A_log, dt_bias, state, (bf16*)out, T, Hk, Hv);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}
