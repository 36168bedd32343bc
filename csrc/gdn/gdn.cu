// Gated DeltaNet (GDN) chunked forward for the frozen teacher, sm_100a.
//
// Per value head h (key head h / (Hv/Hk)) with state S[key j][value i]
// (the [B, Hv, Dk, Dv] layout of the model's cache) and per-step scalar gate:
//   S_t = e^{g_t} S_{t-1} + k_t (beta_t (v_t - e^{g_t} S_{t-1}^T k_t))^T,  o_t = S_t^T q_t
// with q, k L2-normalised (eps 1e-6) and q scaled by Dk^{-1/2}; g_t =
// -exp(A_log) * softplus(a_t + dt_bias), beta_t = sigmoid(b_t) (rounded to bf16
// like the model's bf16 activations).
//
// This is the DPLR recurrence of the WKV7 kernel with decay e^{g} on every
// key, a = k, b = -beta e^{g} k, v' = beta v, r = q; because the decay is a
// per-head scalar, every chunk factor is formed pairwise as e^{Lambda_x -
// Lambda_y} <= 1 (no growth), so large negative gates are safe. Chunks of
// L = 16 steps; per chunk only two Gram matrices are needed, KK = K K^T and
// QK = Q K^T, shared by the Hv/Hk value heads of a key head: a first kernel
// computes them (and the normalised q, k) once per (batch, key head, chunk),
// the recurrent kernel then runs per (batch, value head, 16 value columns).
#include "../common/common.cuh"

namespace {

constexpr int L = 16;
constexpr int R = 16;       // value columns per CTA
constexpr int THREADS = 128;
using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------- prep: normalise q/k, Gram matrices
// grid (chunks, Hk, B); qkv rows [B, T, conv_dim] with q at [0, Hk*D), k at [Hk*D, 2*Hk*D).
template <int D>
__global__ void __launch_bounds__(THREADS)
gdn_prep_kernel(const bf16* __restrict__ qkv, long row_stride, int T, int Hk, float* __restrict__ qn,
                float* __restrict__ kn, float* __restrict__ gram) {
  constexpr int SP = D + 4;
  __shared__ __align__(16) float sq[L * SP];
  __shared__ __align__(16) float sk[L * SP];
  const int ch = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int chunks = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float scale = rsqrtf((float)D);
  for (int tt = warp; tt < L; tt += THREADS / 32) {
    const int t = ch * L + tt;
    float qv[D / 32], kv[D / 32];
    float q2 = 0.f, k2 = 0.f;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
      const int c = lane + 32 * j;
      qv[j] = t < T ? rt::to_f(qkv[((long)b * T + t) * row_stride + (long)kh * D + c]) : 0.f;
      kv[j] = t < T ? rt::to_f(qkv[((long)b * T + t) * row_stride + (long)(Hk + kh) * D + c]) : 0.f;
      q2 += qv[j] * qv[j];
      k2 += kv[j] * kv[j];
    }
    q2 = rt::warp_sum(q2);
    k2 = rt::warp_sum(k2);
    const float iq = rsqrtf(q2 + 1e-6f) * scale, ik = rsqrtf(k2 + 1e-6f);
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
      const int c = lane + 32 * j;
      sq[tt * SP + c] = qv[j] * iq;
      sk[tt * SP + c] = kv[j] * ik;
      if (t < T) {
        qn[(((long)b * T + t) * Hk + kh) * D + c] = qv[j] * iq;
        kn[(((long)b * T + t) * Hk + kh) * D + c] = kv[j] * ik;
      }
    }
  }
  __syncthreads();
  // gram[b][kh][ch] = {KK[L][L], QK[L][L]}
  float* out = gram + (((long)b * Hk + kh) * chunks + ch) * 2 * L * L;
  {
    const int t = threadIdx.x >> 3, s0 = threadIdx.x & 7, s1 = s0 + 8;
    float kk0 = 0, kk1 = 0, qk0 = 0, qk1 = 0;
    const float4* kt = reinterpret_cast<const float4*>(sk + t * SP);
    const float4* qt = reinterpret_cast<const float4*>(sq + t * SP);
    const float4* a0 = reinterpret_cast<const float4*>(sk + s0 * SP);
    const float4* a1 = reinterpret_cast<const float4*>(sk + s1 * SP);
#pragma unroll 4
    for (int q = 0; q < D / 4; ++q) {
      const float4 x = kt[q], y = qt[q], u = a0[q], w = a1[q];
      kk0 += x.x * u.x + x.y * u.y + x.z * u.z + x.w * u.w;
      kk1 += x.x * w.x + x.y * w.y + x.z * w.z + x.w * w.w;
      qk0 += y.x * u.x + y.y * u.y + y.z * u.z + y.w * u.w;
      qk1 += y.x * w.x + y.y * w.y + y.z * w.z + y.w * w.w;
    }
    out[t * L + s0] = kk0;
    out[t * L + s1] = kk1;
    out[L * L + t * L + s0] = qk0;
    out[L * L + t * L + s1] = qk1;
  }
}

// ---------------------------------------------------------------- recurrent chunk kernel
// grid (D/R, Hv, B). Value columns [col0, col0+R) of value head h. The next chunk's q, k, Gram matrices
// and v columns are copied asynchronously (cp.async, double buffered) while the current chunk computes;
// the per-step gates of the next chunk are prefetched into registers.
template <int D>
struct GdnSmem {
  static constexpr int SP = D + 4;
  static constexpr int STAGE = 2 * L * SP + 2 * L * L + L * R / 2;  // q, k, gram (fp32) + v (bf16) in floats
  static constexpr int FLOATS = 2 * STAGE + D * (R + 1) + 4 * L * R + 4 * L * (L + 1) + 6 * L;
};

template <int D>
RT_DEVICE void gdn_issue(float* stage, const float* qn, const float* kn, const float* gram, const bf16* qkv,
                         long row_stride, long vbase, int b, int T, int Hk, int kh, int ch, int chunks) {
  using G = GdnSmem<D>;
  float* sq = stage;
  float* sk = sq + L * G::SP;
  float* sg = sk + L * G::SP;
  bf16* sv = reinterpret_cast<bf16*>(sg + 2 * L * L);
  constexpr int QV = D / 4;
  for (int e = threadIdx.x; e < 2 * L * QV; e += THREADS) {
    const int which = e / (L * QV), rem = e % (L * QV), tt = rem / QV, c = (rem % QV) * 4, t = ch * L + tt;
    const bool ok = t < T;
    const float* base = which ? kn : qn;
    const float* src = base + (ok ? (((long)b * T + t) * Hk + kh) * D + c : 0);
    rt::cp_async16((which ? sk : sq) + tt * G::SP + c, src, ok);
  }
  const float* gsrc = gram + (((long)b * Hk + kh) * chunks + ch) * 2 * L * L;
  for (int e = threadIdx.x; e < 2 * L * L / 4; e += THREADS) rt::cp_async16(sg + 4 * e, gsrc + 4 * e, true);
  for (int e = threadIdx.x; e < L * (R / 8); e += THREADS) {
    const int tt = e / (R / 8), i = (e % (R / 8)) * 8, t = ch * L + tt;
    const bool ok = t < T;
    const bf16* src = qkv + (ok ? ((long)b * T + t) * row_stride + vbase + i : 0);
    rt::cp_async16(sv + tt * R + i, src, ok);
  }
  rt::cp_async_commit();
}

template <int D>
__global__ void __launch_bounds__(THREADS)
gdn_chunk_kernel(const float* __restrict__ qn, const float* __restrict__ kn, const float* __restrict__ gram,
                 const bf16* __restrict__ qkv, long row_stride, const bf16* __restrict__ pa,
                 const bf16* __restrict__ pb, long ab_stride, const float* __restrict__ A_log,
                 const float* __restrict__ dt_bias, float* __restrict__ state, bf16* __restrict__ out, int T, int Hk,
                 int Hv) {
  using G = GdnSmem<D>;
  constexpr int SP = G::SP;
  extern __shared__ __align__(16) float sm[];
  float* stage[2] = {sm, sm + G::STAGE};
  float* S = sm + 2 * G::STAGE;   // [D][R+1] state block (key j, value column i)
  float* V = S + D * (R + 1);     // [L][R]  beta * v
  float* Z = V + L * R;           // [L][R]
  float* U = Z + L * R;           // [L][R]
  float* Y = U + L * R;           // [L][R]
  float* Mab = Y + L * R;         // [L][L+1]
  float* Mak = Mab + L * (L + 1);
  float* Mrb = Mak + L * (L + 1);
  float* Mrk = Mrb + L * (L + 1);
  float* lam = Mrk + L * (L + 1); // [L] cumulative log decay
  float* beta = lam + L;          // [L]
  float* e_prev = beta + L;       // [L] e^{Lambda_{t-1}}
  float* e_cur = e_prev + L;      // [L] e^{Lambda_t}
  float* c_u = e_cur + L;         // [L] -beta_s e^{Lambda_L - Lambda_{s-1}}
  float* c_v = c_u + L;           // [L] e^{Lambda_L - Lambda_s}
  const int rb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (Hv / Hk);
  const int col0 = rb * R;
  const int chunks = (T + L - 1) / L;
  const long vbase = 2L * Hk * D + (long)h * D + col0;  // v column offset inside a qkv row
  float* st = state + ((long)b * Hv + h) * D * D;       // [D key][D value]
  gdn_issue<D>(stage[0], qn, kn, gram, qkv, row_stride, vbase, b, T, Hk, kh, 0, chunks);
  for (int e = threadIdx.x; e < D * R; e += THREADS) {
    const int j = e / R, i = e % R;
    S[j * (R + 1) + i] = st[(long)j * D + col0 + i];
  }
  const float neg_a = -expf(A_log[h]);
  const float dtb = dt_bias[h];
  // Gate inputs of the current chunk held in registers by threads < L.
  float ga = 0.f, gb = 0.f;
  if (threadIdx.x < L && threadIdx.x < T) {
    ga = rt::to_f(pa[((long)b * T + threadIdx.x) * ab_stride + h]);
    gb = rt::to_f(pb[((long)b * T + threadIdx.x) * ab_stride + h]);
  }
  for (int ch = 0; ch < chunks; ++ch) {
    const int t0 = ch * L;
    if (ch + 1 < chunks) {
      gdn_issue<D>(stage[(ch + 1) & 1], qn, kn, gram, qkv, row_stride, vbase, b, T, Hk, kh, ch + 1, chunks);
      rt::cp_async_wait<1>();
    } else {
      rt::cp_async_wait<0>();
    }
    float na = 0.f, nb = 0.f;  // next chunk's gates (prefetched into registers)
    if (threadIdx.x < L) {
      const int tn = t0 + L + threadIdx.x;
      if (tn < T) {
        na = rt::to_f(pa[((long)b * T + tn) * ab_stride + h]);
        nb = rt::to_f(pb[((long)b * T + tn) * ab_stride + h]);
      }
      const int tt = threadIdx.x, t = t0 + tt;
      float g = 0.f, bt = 0.f;
      if (t < T) {
        const float av = ga + dtb;
        const float sp = av > 20.f ? av : log1pf(expf(av));
        g = neg_a * sp;
        bt = __bfloat162float(__float2bfloat16_rn(rt::sigmoidf_(gb)));
      }
      lam[tt] = g;
      beta[tt] = bt;
    }
    __syncthreads();
    const float* sq = stage[ch & 1];
    const float* sk = sq + L * SP;
    const float* gr = sk + L * SP;
    const bf16* sv = reinterpret_cast<const bf16*>(gr + 2 * L * L);
    if (threadIdx.x == 0) {
      float run = 0.f;
      for (int tt = 0; tt < L; ++tt) { run += lam[tt]; lam[tt] = run; }
    }
    __syncthreads();
    if (threadIdx.x < L) {
      const int tt = threadIdx.x;
      const float prev = tt ? lam[tt - 1] : 0.f, lL = lam[L - 1];
      e_prev[tt] = expf(prev);
      e_cur[tt] = expf(lam[tt]);
      c_u[tt] = -beta[tt] * expf(lL - prev);
      c_v[tt] = expf(lL - lam[tt]);
    }
    for (int e = threadIdx.x; e < L * R; e += THREADS) V[e] = rt::to_f(sv[e]) * beta[e / R];
    // Chunk matrices from the Gram matrices (all exponents <= 0).
    for (int e = threadIdx.x; e < L * L; e += THREADS) {
      const int t = e / L, s = e % L;
      const float kk = gr[e], qk = gr[L * L + e];
      const float lt = lam[t], lt1 = t ? lam[t - 1] : 0.f, ls = lam[s], ls1 = s ? lam[s - 1] : 0.f;
      Mab[t * (L + 1) + s] = s < t ? -beta[s] * kk * expf(lt1 - ls1) : 0.f;
      Mak[t * (L + 1) + s] = s < t ? kk * expf(lt1 - ls) : 0.f;
      Mrb[t * (L + 1) + s] = s <= t ? -beta[s] * qk * expf(lt - ls1) : 0.f;
      Mrk[t * (L + 1) + s] = s <= t ? qk * expf(lt - ls) : 0.f;
    }
    __syncthreads();
    // Z = e^{Lambda_{t-1}} S0^T k_t + Mak V ;  Yp = e^{Lambda_t} S0^T q_t + Mrk V
    for (int e = threadIdx.x; e < L * R; e += THREADS) {
      const int t = e / R, i = e % R;
      float zk = 0.f, yq = 0.f;
#pragma unroll 8
      for (int j = 0; j < D; ++j) {
        const float sv2 = S[j * (R + 1) + i];
        zk += sk[t * SP + j] * sv2;
        yq += sq[t * SP + j] * sv2;
      }
      float z = zk * e_prev[t], y = yq * e_cur[t];
      for (int s = 0; s < t; ++s) z += Mak[t * (L + 1) + s] * V[s * R + i];
      for (int s = 0; s <= t; ++s) y += Mrk[t * (L + 1) + s] * V[s * R + i];
      Z[e] = z;
      Y[e] = y;
    }
    __syncthreads();
    if (threadIdx.x < R) {
      const int i = threadIdx.x;
      for (int t = 0; t < L; ++t) {
        float u = Z[t * R + i];
        for (int s = 0; s < t; ++s) u += Mab[t * (L + 1) + s] * U[s * R + i];
        U[t * R + i] = u;
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < L * R; e += THREADS) {
      const int t = e / R, i = e % R;
      float y = Y[e];
      for (int s = 0; s <= t; ++s) y += Mrb[t * (L + 1) + s] * U[s * R + i];
      const int tg = t0 + t;
      if (tg < T) out[(((long)b * T + tg) * Hv + h) * D + col0 + i] = __float2bfloat16_rn(y);
    }
    // S_L = e^{Lambda_L} S0 + sum_s k_s (U_s c_s + V_s d_s), c_s = -beta_s e^{Lambda_L - Lambda_{s-1}},
    // d_s = e^{Lambda_L - Lambda_s}.
    const float eL = e_cur[L - 1];
    for (int e = threadIdx.x; e < D * R; e += THREADS) {
      const int j = e / R, i = e % R;
      float acc = S[j * (R + 1) + i] * eL;
#pragma unroll
      for (int s = 0; s < L; ++s) acc += sk[s * SP + j] * (U[s * R + i] * c_u[s] + V[s * R + i] * c_v[s]);
      S[j * (R + 1) + i] = acc;
    }
    ga = na;
    gb = nb;
    __syncthreads();
  }
  for (int e = threadIdx.x; e < D * R; e += THREADS) {
    const int j = e / R, i = e % R;
    st[(long)j * D + col0 + i] = S[j * (R + 1) + i];
  }
}

template <int D>
cudaError_t launch(const void* qkv, long row_stride, const void* a, const void* b, long ab_stride, const float* A_log,
                   const float* dt_bias, float* state, void* out, float* work, int B, int T, int Hk, int Hv,
                   cudaStream_t stream) {
  const int chunks = (T + L - 1) / L;
  float* qn = work;
  float* kn = qn + (long)B * T * Hk * D;
  float* gram = kn + (long)B * T * Hk * D;
  gdn_prep_kernel<D><<<dim3(chunks, Hk, B), THREADS, 0, stream>>>((const bf16*)qkv, row_stride, T, Hk, qn, kn, gram);
  RT_CUDA_CHECK(cudaGetLastError());
  const size_t smem = GdnSmem<D>::FLOATS * sizeof(float);
  RT_CUDA_CHECK(cudaFuncSetAttribute(gdn_chunk_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  gdn_chunk_kernel<D><<<dim3(D / R, Hv, B), THREADS, smem, stream>>>(
      qn, kn, gram, (const bf16*)qkv, row_stride, (const bf16*)a, (const bf16*)b, ab_stride, A_log, dt_bias, state,
      (bf16*)out, T, Hk, Hv);
  return cudaGetLastError();
}

}  // namespace

// Scratch floats needed by rt_gdn_forward: normalised q and k plus the Gram matrices.
extern "C" long rt_gdn_workspace_floats(int B, int T, int Hk, int D) {
  const long chunks = (T + L - 1) / L;
  return 2L * B * T * Hk * D + (long)B * Hk * chunks * 2 * L * L;
}

// qkv: conv+SiLU output rows [B*T, row_stride] bf16 (q | k | v); a, b: [B*T, ab_stride] bf16 gate inputs;
// state: [B, Hv, D, D] fp32, updated in place; out: [B, T, Hv, D] bf16.
extern "C" cudaError_t rt_gdn_forward(const void* qkv, long row_stride, const void* a, const void* b, long ab_stride,
                                      const float* A_log, const float* dt_bias, float* state, void* out, float* work,
                                      int B, int T, int Hk, int Hv, int D, cudaStream_t stream) {
  if (Hv % Hk) return cudaErrorInvalidValue;
  switch (D) {
    case 128: return launch<128>(qkv, row_stride, a, b, ab_stride, A_log, dt_bias, state, out, work, B, T, Hk, Hv, stream);
    case 64: return launch<64>(qkv, row_stride, a, b, ab_stride, A_log, dt_bias, state, out, work, B, T, Hk, Hv, stream);
    case 32: return launch<32>(qkv, row_stride, a, b, ab_stride, A_log, dt_bias, state, out, work, B, T, Hk, Hv, stream);
    default: return cudaErrorInvalidValue;
  }
}
