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
// grid (D/R, Hv, B), 256 threads. Value columns [col0, col0+R) of value head h; the state block is held
// value-major (S[i][j], i value column, j key) so every inner product over keys uses 128-bit shared loads.
// The next chunk's q, k, Gram matrices and v columns are copied asynchronously (cp.async, double buffered)
// while the current chunk computes; the per-step gates of the next chunk are prefetched into registers.
constexpr int CT = 256;

template <int D>
struct GdnSmem {
  static constexpr int SP = D + 4;
  static constexpr int STAGE = 2 * L * SP + 2 * L * L + L * R / 2;  // q, k, gram (fp32) + v (bf16) in floats
  static constexpr int FLOATS = 2 * STAGE + R * SP + 5 * L * R + 4 * L * (L + 1) + 6 * L;
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
  for (int e = threadIdx.x; e < 2 * L * QV; e += CT) {
    const int which = e / (L * QV), rem = e % (L * QV), tt = rem / QV, c = (rem % QV) * 4, t = ch * L + tt;
    const bool ok = t < T;
    const float* base = which ? kn : qn;
    const float* src = base + (ok ? (((long)b * T + t) * Hk + kh) * D + c : 0);
    rt::cp_async16((which ? sk : sq) + tt * G::SP + c, src, ok);
  }
  const float* gsrc = gram + (((long)b * Hk + kh) * chunks + ch) * 2 * L * L;
  for (int e = threadIdx.x; e < 2 * L * L / 4; e += CT) rt::cp_async16(sg + 4 * e, gsrc + 4 * e, true);
  for (int e = threadIdx.x; e < L * (R / 8); e += CT) {
    const int tt = e / (R / 8), i = (e % (R / 8)) * 8, t = ch * L + tt;
    const bool ok = t < T;
    const bf16* src = qkv + (ok ? ((long)b * T + t) * row_stride + vbase + i : 0);
    rt::cp_async16(sv + tt * R + i, src, ok);
  }
  rt::cp_async_commit();
}

template <int D>
__global__ void __launch_bounds__(CT)
gdn_chunk_kernel(const float* __restrict__ qn, const float* __restrict__ kn, const float* __restrict__ gram,
                 const bf16* __restrict__ qkv, long row_stride, const bf16* __restrict__ pa,
                 const bf16* __restrict__ pb, long ab_stride, const float* __restrict__ A_log,
                 const float* __restrict__ dt_bias, float* __restrict__ state, bf16* __restrict__ out, int T, int Hk,
                 int Hv) {
  using G = GdnSmem<D>;
  constexpr int SP = G::SP;
  extern __shared__ __align__(16) float sm[];
  float* stage[2] = {sm, sm + G::STAGE};
  float* S = sm + 2 * G::STAGE;   // [R][SP] state block, value-major
  float* V = S + R * SP;          // [L][R]  beta * v
  float* Z = V + L * R;           // [L][R]
  float* U = Z + L * R;           // [L][R]
  float* Y = U + L * R;           // [L][R]
  float* Q = Y + L * R;           // [L][R]  per-step state-update coefficients
  float* Mab = Q + L * R;         // [L][L+1]
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
  for (int e = threadIdx.x; e < D * R; e += CT) {
    const int j = e / R, i = e % R;
    S[i * SP + j] = st[(long)j * D + col0 + i];
  }
  const float neg_a = -expf(A_log[h]);
  const float dtb = dt_bias[h];
  float ga = 0.f, gb = 0.f;  // gate inputs of the current chunk (threads < L)
  if (threadIdx.x < L && threadIdx.x < T) {
    ga = rt::to_f(pa[((long)b * T + threadIdx.x) * ab_stride + h]);
    gb = rt::to_f(pb[((long)b * T + threadIdx.x) * ab_stride + h]);
  }
  const int ti = threadIdx.x >> 4, ii = threadIdx.x & 15;  // (t, i) owned in the L x R loops
  for (int ch = 0; ch < chunks; ++ch) {
    const int t0 = ch * L;
    if (ch + 1 < chunks) {
      gdn_issue<D>(stage[(ch + 1) & 1], qn, kn, gram, qkv, row_stride, vbase, b, T, Hk, kh, ch + 1, chunks);
      rt::cp_async_wait<1>();
    } else {
      rt::cp_async_wait<0>();
    }
    float na = 0.f, nb = 0.f;
    if (threadIdx.x < L) {
      const int tn = t0 + L + threadIdx.x;
      if (tn < T) {
        na = rt::to_f(pa[((long)b * T + tn) * ab_stride + h]);
        nb = rt::to_f(pb[((long)b * T + tn) * ab_stride + h]);
      }
      float g = 0.f, bt = 0.f;
      if (t0 + threadIdx.x < T) {
        const float av = ga + dtb;
        g = neg_a * (av > 20.f ? av : log1pf(expf(av)));
        bt = __bfloat162float(__float2bfloat16_rn(rt::sigmoidf_(gb)));
      }
      lam[threadIdx.x] = g;
      beta[threadIdx.x] = bt;
    }
    __syncthreads();
    const float* sq = stage[ch & 1];
    const float* sk = sq + L * SP;
    const float* gr = sk + L * SP;
    const bf16* sv = reinterpret_cast<const bf16*>(gr + 2 * L * L);
    if (threadIdx.x < 32) {  // inclusive scan of the 16 log-gates in one warp
      float x = threadIdx.x < L ? lam[threadIdx.x] : 0.f;
#pragma unroll
      for (int o = 1; o < L; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, o);
        if (threadIdx.x >= o) x += y;
      }
      const float lL = __shfl_sync(0xffffffffu, x, L - 1);
      const float prev = __shfl_up_sync(0xffffffffu, x, 1);
      if (threadIdx.x < L) {
        const float pv = threadIdx.x ? prev : 0.f;
        lam[threadIdx.x] = x;
        e_prev[threadIdx.x] = expf(pv);
        e_cur[threadIdx.x] = expf(x);
        c_u[threadIdx.x] = -beta[threadIdx.x] * expf(lL - pv);
        c_v[threadIdx.x] = expf(lL - x);
      }
    }
    V[threadIdx.x] = rt::to_f(sv[threadIdx.x]);  // L * R == CT
    __syncthreads();
    {  // chunk matrices from the Gram matrices (all exponents <= 0); beta-scaled V
      const int t = ti, s2 = ii;
      const float kk = gr[t * L + s2], qk = gr[L * L + t * L + s2];
      const float lt = lam[t], lt1 = t ? lam[t - 1] : 0.f, ls = lam[s2], ls1 = s2 ? lam[s2 - 1] : 0.f;
      Mab[t * (L + 1) + s2] = s2 < t ? -beta[s2] * kk * expf(lt1 - ls1) : 0.f;
      Mak[t * (L + 1) + s2] = s2 < t ? kk * expf(lt1 - ls) : 0.f;
      Mrb[t * (L + 1) + s2] = s2 <= t ? -beta[s2] * qk * expf(lt - ls1) : 0.f;
      Mrk[t * (L + 1) + s2] = s2 <= t ? qk * expf(lt - ls) : 0.f;
      V[threadIdx.x] *= beta[ti];
    }
    __syncthreads();
    {  // Z = e^{Lambda_{t-1}} S0 k_t + Mak V ;  Yp = e^{Lambda_t} S0 q_t + Mrk V
      const float4* kt = reinterpret_cast<const float4*>(sk + ti * SP);
      const float4* qt = reinterpret_cast<const float4*>(sq + ti * SP);
      const float4* si = reinterpret_cast<const float4*>(S + ii * SP);
      float zk = 0.f, yq = 0.f;
#pragma unroll 8
      for (int u = 0; u < D / 4; ++u) {
        const float4 s4 = si[u], k4 = kt[u], q4 = qt[u];
        zk += k4.x * s4.x + k4.y * s4.y + k4.z * s4.z + k4.w * s4.w;
        yq += q4.x * s4.x + q4.y * s4.y + q4.z * s4.z + q4.w * s4.w;
      }
      float z = zk * e_prev[ti], y = yq * e_cur[ti];
      for (int s2 = 0; s2 < ti; ++s2) z += Mak[ti * (L + 1) + s2] * V[s2 * R + ii];
      for (int s2 = 0; s2 <= ti; ++s2) y += Mrk[ti * (L + 1) + s2] * V[s2 * R + ii];
      Z[threadIdx.x] = z;
      Y[threadIdx.x] = y;
    }
    __syncthreads();
    if (threadIdx.x < R) {
      const int i = threadIdx.x;
      for (int t = 0; t < L; ++t) {
        float u = Z[t * R + i];
        for (int s2 = 0; s2 < t; ++s2) u += Mab[t * (L + 1) + s2] * U[s2 * R + i];
        U[t * R + i] = u;
      }
    }
    __syncthreads();
    {
      float y = Y[threadIdx.x];
      for (int s2 = 0; s2 <= ti; ++s2) y += Mrb[ti * (L + 1) + s2] * U[s2 * R + ii];
      const int tg = t0 + ti;
      if (tg < T) out[(((long)b * T + tg) * Hv + h) * D + col0 + ii] = __float2bfloat16_rn(y);
      Q[threadIdx.x] = U[threadIdx.x] * c_u[ti] + V[threadIdx.x] * c_v[ti];
    }
    __syncthreads();
    // S_L[i][j] = e^{Lambda_L} S0[i][j] + sum_s Q[s][i] k_s[j]
    const float eL = e_cur[L - 1];
    for (int e = threadIdx.x; e < R * (D / 4); e += CT) {
      const int i = e / (D / 4), j = (e % (D / 4)) * 4;
      float4 acc = *reinterpret_cast<float4*>(S + i * SP + j);
      acc.x *= eL; acc.y *= eL; acc.z *= eL; acc.w *= eL;
#pragma unroll
      for (int s2 = 0; s2 < L; ++s2) {
        const float qv = Q[s2 * R + i];
        const float4 k4 = *reinterpret_cast<const float4*>(sk + s2 * SP + j);
        acc.x += qv * k4.x; acc.y += qv * k4.y; acc.z += qv * k4.z; acc.w += qv * k4.w;
      }
      *reinterpret_cast<float4*>(S + i * SP + j) = acc;
    }
    ga = na;
    gb = nb;
    __syncthreads();
  }
  for (int e = threadIdx.x; e < D * R; e += CT) {
    const int j = e / R, i = e % R;
    st[(long)j * D + col0 + i] = S[i * SP + j];
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
  gdn_chunk_kernel<D><<<dim3(D / R, Hv, B), CT, smem, stream>>>(
      qn, kn, gram, (const bf16*)qkv, row_stride, (const bf16*)a, (const bf16*)b, ab_stride, A_log, dt_bias, state,
      (bf16*)out, T, Hk, Hv);
  return cudaGetLastError();
}

}  // namespace

// Long prefills take the WY path (csrc/gdn/gdn_wy.cu: state-free chunk algebra in parallel, a light serial state
// pass); short calls (decode steps, small chunks) the serial 16-step kernel above.
long rt_gdn_wy_workspace_floats(int B, int T, int Hk, int Hv, int D);
cudaError_t rt_gdn_wy_forward(const void* qkv, long row_stride, const void* a, const void* b, long ab_stride,
                              const float* A_log, const float* dt_bias, float* state, void* out, float* work, int B,
                              int T, int Hk, int Hv, int D, cudaStream_t stream);

extern "C" cudaError_t rt_gdn_step(const void* qkv, long row_stride, const void* a, const void* b, long ab_stride,
                                   const float* A_log, const float* dt_bias, float* state, void* out, int B, int T,
                                   int Hk, int Hv, int D, cudaStream_t stream);

namespace {
constexpr int WY_MIN_T = 128;
constexpr int STEP_MAX_T = 4;  // decode-sized calls: token-by-token kernel (gdn_step.cu), no workspace
bool use_wy(int T, long row_stride, int D) { return T >= WY_MIN_T && (D == 64 || D == 128) && row_stride % 8 == 0; }
bool use_step(int T, int D) { return T <= STEP_MAX_T && (D == 64 || D == 128); }
}  // namespace

// Scratch floats of the serial 16-step path alone.
extern "C" long rt_gdn_serial_workspace_floats(int B, int T, int Hk, int D) {
  const long chunks = (T + L - 1) / L;
  return 2L * B * T * Hk * D + (long)B * Hk * chunks * 2 * L * L;
}

// Scratch floats needed by rt_gdn_forward for these sizes (row_stride decides the path only through alignment).
extern "C" long rt_gdn_workspace_floats(int B, int T, int Hk, int Hv, int D, long row_stride) {
  if (use_step(T, D)) return 0;
  if (use_wy(T, row_stride, D)) return rt_gdn_wy_workspace_floats(B, T, Hk, Hv, D);
  return rt_gdn_serial_workspace_floats(B, T, Hk, D);
}

// The serial 16-step path for any T (its scratch is rt_gdn_serial_workspace_floats).
extern "C" cudaError_t rt_gdn_forward_serial(const void* qkv, long row_stride, const void* a, const void* b,
                                             long ab_stride, const float* A_log, const float* dt_bias, float* state,
                                             void* out, float* work, int B, int T, int Hk, int Hv, int D,
                                             cudaStream_t stream) {
  if (Hv % Hk) return cudaErrorInvalidValue;
  switch (D) {
    case 128: return launch<128>(qkv, row_stride, a, b, ab_stride, A_log, dt_bias, state, out, work, B, T, Hk, Hv, stream);
    case 64: return launch<64>(qkv, row_stride, a, b, ab_stride, A_log, dt_bias, state, out, work, B, T, Hk, Hv, stream);
    case 32: return launch<32>(qkv, row_stride, a, b, ab_stride, A_log, dt_bias, state, out, work, B, T, Hk, Hv, stream);
    default: return cudaErrorInvalidValue;
  }
}

// qkv: conv+SiLU output rows [B*T, row_stride] bf16 (q | k | v); a, b: [B*T, ab_stride] bf16 gate inputs;
// state: [B, Hv, D, D] fp32, updated in place; out: [B, T, Hv, D] bf16.
extern "C" cudaError_t rt_gdn_forward(const void* qkv, long row_stride, const void* a, const void* b, long ab_stride,
                                      const float* A_log, const float* dt_bias, float* state, void* out, float* work,
                                      int B, int T, int Hk, int Hv, int D, cudaStream_t stream) {
  if (Hv % Hk) return cudaErrorInvalidValue;
  if (use_step(T, D))
    return rt_gdn_step(qkv, row_stride, a, b, ab_stride, A_log, dt_bias, state, out, B, T, Hk, Hv, D, stream);
  if (use_wy(T, row_stride, D))
    return rt_gdn_wy_forward(qkv, row_stride, a, b, ab_stride, A_log, dt_bias, state, out, work, B, T, Hk, Hv, D,
                             stream);
  return rt_gdn_forward_serial(qkv, row_stride, a, b, ab_stride, A_log, dt_bias, state, out, work, B, T, Hk, Hv, D,
                               stream);
}
