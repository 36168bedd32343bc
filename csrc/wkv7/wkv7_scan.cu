// WKV7 forward as a parallel per-chunk pass plus a light serial scan, sm_100a (head sizes 32, 64, 128).
// The recurrence is RWKV7's (RWKV-LM, Apache-2.0; see NOTICE at the project root); this code is our own.
//
// Same chunk algebra as wkv7.cu (chunks of L = 16, decayed vectors a~ = a e^{Lambda_{t-1}}, r~ = r e^{Lambda_t},
// b~ = b e^{-Lambda_s}, k~ = k e^{-Lambda_s}, chunk matrices Mab, Mak (s < t), Mrb, Mrk (s <= t)), with every
// term that does not depend on the chunk-start state S0 moved out of the sequential loop. With
// T = (I - Mab)^{-1}:
//   U  = W S0^T + U0,       W  = T A~,                U0 = T (Mak V)
//   Y  = Q S0^T + Y0,       Q  = R~ + Mrb W,          Y0 = Mrk V + Mrb U0
//   S_L[i][j] = S0[i][j] D_L[j] + sum_t U[t][i] B^[t][j] + sum_t V[t][i] K^[t][j],   B^ = B~ D_L, K^ = K~ D_L.
// Kernel 1 (grid chunks x B*H, parallel) forms W, Q, B^, K^, U0, Y0 and D_L per chunk; kernel 2 (grid
// N/16 row blocks x B*H) walks the chunks: two 16 x 16 x N products for U and Y (y is written directly),
// the checkpoint store, and the state update -- a fraction of the work of the fused serial kernel, with the
// next chunk's record prefetched by cp.async.
#include "../common/common.cuh"

namespace {

constexpr int L = 16;
constexpr int R = 8;           // value rows per CTA in the scan (one U/Y output and one state quad per thread)
constexpr int THREADS = 128;
constexpr float DECAY_SCALE = 0.6065306597126334f;

// Per-chunk record in the workspace: W, Q, B^, K^ [L][N]; U0, Y0 [L][N] (value columns); D_L [N].
template <int N>
struct Rec {
  static constexpr int W = 0, Q = L * N, BH = 2 * L * N, KH = 3 * L * N, U0 = 4 * L * N, Y0 = 5 * L * N,
                       DL = 6 * L * N, FLOATS = 6 * L * N + N;
};

// ---------------------------------------------------------------- kernel 1: per-chunk terms
template <typename T, int N>
__global__ void __launch_bounds__(THREADS)
wkv7_chunk_kernel(int T_, int H, const T* __restrict__ pr, const T* __restrict__ pw, const T* __restrict__ pk,
                  const T* __restrict__ pv, const T* __restrict__ pa, const T* __restrict__ pb,
                  float* __restrict__ work) {
  constexpr int SP = N + 4, MP = L + 1;
  extern __shared__ __align__(16) float sm[];
  float* r = sm;
  float* a = r + L * SP;
  float* b = a + L * SP;
  float* k = b + L * SP;
  float* v = k + L * SP;
  float* lam = v + L * SP;
  float (*M)[L * MP] = reinterpret_cast<float (*)[L * MP]>(lam + L * SP);
  float* Ti = lam + L * SP + 4 * L * MP;
  float* dl = Ti + L * MP;
  const int ch = blockIdx.x, bh = blockIdx.y, batch = bh / H, head = bh % H, chunks = gridDim.x;
  const int t0 = ch * L, tid = threadIdx.x;
  for (int e = tid; e < L * N; e += THREADS) {
    const int tt = e / N, j = e % N, t = t0 + tt, o = tt * SP + j;
    const bool ok = t < T_;
    const long src = (((long)batch * T_ + (ok ? t : 0)) * H + head) * N + j;
    r[o] = ok ? rt::to_f(pr[src]) : 0.f;
    k[o] = ok ? rt::to_f(pk[src]) : 0.f;
    a[o] = ok ? rt::to_f(pa[src]) : 0.f;
    b[o] = ok ? rt::to_f(pb[src]) : 0.f;
    v[o] = ok ? rt::to_f(pv[src]) : 0.f;
    lam[o] = ok ? -DECAY_SCALE * rt::sigmoidf_(rt::to_f(pw[src])) : 0.f;
  }
  __syncthreads();
  if (tid < N) {
    float run = 0.f;
#pragma unroll
    for (int tt = 0; tt < L; ++tt) {
      run += lam[tt * SP + tid];
      lam[tt * SP + tid] = run;
    }
    dl[tid] = expf(run);
  }
  __syncthreads();
  for (int e = tid; e < L * N; e += THREADS) {
    const int tt = e / N, j = e % N, o = tt * SP + j;
    const float cur = lam[o], prev = tt ? lam[o - SP] : 0.f;
    const float inv = expf(-cur);
    r[o] *= expf(cur);
    a[o] *= expf(prev);
    b[o] *= inv;
    k[o] *= inv;
  }
  __syncthreads();
  {  // chunk matrices; thread: row t = tid >> 3, columns s0 = tid & 7 and s0 + 8
    const int t = tid >> 3, s0 = tid & 7, s1 = s0 + 8;
    float ab0 = 0, ak0 = 0, rb0 = 0, rk0 = 0, ab1 = 0, ak1 = 0, rb1 = 0, rk1 = 0;
#pragma unroll 4
    for (int j = 0; j < N; j += 4) {
      const float4 x = *reinterpret_cast<const float4*>(a + t * SP + j);
      const float4 y = *reinterpret_cast<const float4*>(r + t * SP + j);
      const float4 p0 = *reinterpret_cast<const float4*>(b + s0 * SP + j);
      const float4 u0 = *reinterpret_cast<const float4*>(k + s0 * SP + j);
      const float4 p1 = *reinterpret_cast<const float4*>(b + s1 * SP + j);
      const float4 u1 = *reinterpret_cast<const float4*>(k + s1 * SP + j);
      ab0 += x.x * p0.x + x.y * p0.y + x.z * p0.z + x.w * p0.w;
      ak0 += x.x * u0.x + x.y * u0.y + x.z * u0.z + x.w * u0.w;
      rb0 += y.x * p0.x + y.y * p0.y + y.z * p0.z + y.w * p0.w;
      rk0 += y.x * u0.x + y.y * u0.y + y.z * u0.z + y.w * u0.w;
      ab1 += x.x * p1.x + x.y * p1.y + x.z * p1.z + x.w * p1.w;
      ak1 += x.x * u1.x + x.y * u1.y + x.z * u1.z + x.w * u1.w;
      rb1 += y.x * p1.x + y.y * p1.y + y.z * p1.z + y.w * p1.w;
      rk1 += y.x * u1.x + y.y * u1.y + y.z * u1.z + y.w * u1.w;
    }
    M[0][t * MP + s0] = s0 < t ? ab0 : 0.f;
    M[1][t * MP + s0] = s0 < t ? ak0 : 0.f;
    M[2][t * MP + s0] = s0 <= t ? rb0 : 0.f;
    M[3][t * MP + s0] = s0 <= t ? rk0 : 0.f;
    M[0][t * MP + s1] = s1 < t ? ab1 : 0.f;
    M[1][t * MP + s1] = s1 < t ? ak1 : 0.f;
    M[2][t * MP + s1] = s1 <= t ? rb1 : 0.f;
    M[3][t * MP + s1] = s1 <= t ? rk1 : 0.f;
  }
  __syncthreads();
  if (tid < L) {  // T = (I - Mab)^{-1}, one column per thread
    const int s = tid;
    for (int t = 0; t < L; ++t) {
      float x = t == s ? 1.f : 0.f;
      if (t > s)
        for (int q = s; q < t; ++q) x += M[0][t * MP + q] * Ti[q * MP + s];
      Ti[t * MP + s] = x;
    }
  }
  __syncthreads();
  float* rec = work + ((long)bh * chunks + ch) * Rec<N>::FLOATS;
  // W = T A~ (in registers per thread, then Q = R~ + Mrb W needs W of all rows: stage W in shared `a`'s slot
  // after use) and X = Mak V staged the same way; thread e covers (t, j) pairs.
  float Wv[L * N / THREADS], Xv[L * N / THREADS];
#pragma unroll
  for (int q = 0; q < L * N / THREADS; ++q) {
    const int e = tid + q * THREADS, t = e / N, j = e % N;
    float w = 0.f, x = 0.f;
    for (int s = 0; s <= t; ++s) w += Ti[t * MP + s] * a[s * SP + j];
    for (int s = 0; s < t; ++s) x += M[1][t * MP + s] * v[s * SP + j];
    Wv[q] = w;
    Xv[q] = x;
  }
  __syncthreads();  // all reads of a~ done: reuse a for W, lam for X
#pragma unroll
  for (int q = 0; q < L * N / THREADS; ++q) {
    const int e = tid + q * THREADS, t = e / N, j = e % N;
    a[t * SP + j] = Wv[q];
    lam[t * SP + j] = Xv[q];
    rec[Rec<N>::W + e] = Wv[q];
  }
  __syncthreads();
  // U0 = T X; then Q = R~ + Mrb W; B^, K^
#pragma unroll
  for (int q = 0; q < L * N / THREADS; ++q) {
    const int e = tid + q * THREADS, t = e / N, j = e % N;
    float u = 0.f, qq = r[t * SP + j];
    for (int s = 0; s <= t; ++s) {
      u += Ti[t * MP + s] * lam[s * SP + j];
      qq += M[2][t * MP + s] * a[s * SP + j];
    }
    Xv[q] = u;
    rec[Rec<N>::Q + e] = qq;
    rec[Rec<N>::BH + e] = b[t * SP + j] * dl[j];
    rec[Rec<N>::KH + e] = k[t * SP + j] * dl[j];
  }
  __syncthreads();  // reads of X (in lam) done: stage U0 there
#pragma unroll
  for (int q = 0; q < L * N / THREADS; ++q) {
    const int e = tid + q * THREADS, t = e / N, j = e % N;
    lam[t * SP + j] = Xv[q];
    rec[Rec<N>::U0 + e] = Xv[q];
  }
  __syncthreads();
  // Y0 = Mrk V + Mrb U0
#pragma unroll
  for (int q = 0; q < L * N / THREADS; ++q) {
    const int e = tid + q * THREADS, t = e / N, j = e % N;
    float y = 0.f;
    for (int s = 0; s <= t; ++s) y += M[3][t * MP + s] * v[s * SP + j] + M[2][t * MP + s] * lam[s * SP + j];
    rec[Rec<N>::Y0 + e] = y;
  }
  if (tid < N) rec[Rec<N>::DL + tid] = dl[tid];
}

// ---------------------------------------------------------------- kernel 2: serial scan over chunks
template <int N>
struct ScanSmem {
  static constexpr int SP = N + 4;
  // per stage: W, Q, B^, K^ [L][SP]; U0, Y0, V [L][R]; D_L [N]
  static constexpr int STAGE = 4 * L * SP + 3 * L * R + N;
  static constexpr int FLOATS = 2 * STAGE + R * SP + 2 * L * R;
};

template <typename T, int N>
RT_DEVICE void scan_issue(float* st, const float* rec, const T* pv, int T_, int H, int batch, int head, int t0,
                          int row0, const T* zero) {
  constexpr int SP = N + 4;
  for (int e = threadIdx.x; e < 4 * L * (N / 4); e += THREADS) {
    const int which = e / (L * N / 4), rem = e % (L * N / 4), tt = rem / (N / 4), j = (rem % (N / 4)) * 4;
    rt::cp_async16(st + which * L * SP + tt * SP + j, rec + which * L * N + tt * N + j, true);
  }
  float* u0 = st + 4 * L * SP;
  for (int e = threadIdx.x; e < 2 * L * (R / 4); e += THREADS) {
    const int which = e / (L * R / 4), rem = e % (L * R / 4), tt = rem / (R / 4), i = (rem % (R / 4)) * 4;
    rt::cp_async16(u0 + which * L * R + tt * R + i, rec + (4 + which) * L * N + tt * N + row0 + i, true);
  }
  float* dl = u0 + 3 * L * R;
  for (int e = threadIdx.x; e < N / 4; e += THREADS) rt::cp_async16(dl + 4 * e, rec + 6 * L * N + 4 * e, true);
  // V rows of this block in the input dtype (R * sizeof(T) = 16 or 32 bytes per step), zero-filled past T
  T* vv = reinterpret_cast<T*>(u0 + 2 * L * R);
  constexpr int VPR = R * sizeof(T) / 16;  // 16-byte copies per step
  for (int e = threadIdx.x; e < L * VPR; e += THREADS) {
    const int tt = e / VPR, part = e % VPR, t = t0 + tt;
    const bool ok = t < T_;
    const T* src = ok ? pv + (((long)batch * T_ + t) * H + head) * N + row0 + part * (16 / sizeof(T)) : zero;
    rt::cp_async16(vv + tt * R + part * (16 / sizeof(T)), src, ok);
  }
  rt::cp_async_commit();
}

template <typename T, int N>
__global__ void __launch_bounds__(THREADS)
wkv7_scan_kernel(int T_, int H, const T* __restrict__ pv, const float* __restrict__ s0, const float* __restrict__ work,
                 T* __restrict__ py, float* __restrict__ s_end, float* __restrict__ checkpoints) {
  using SM = ScanSmem<N>;
  constexpr int SP = SM::SP;
  extern __shared__ __align__(16) float sm[];
  float* stage[2] = {sm, sm + SM::STAGE};
  float* S = sm + 2 * SM::STAGE;   // [R][SP]
  float* U = S + R * SP;           // [L][R]
  float* Yb = U + L * R;           // [L][R]
  const int rb = blockIdx.x, bh = blockIdx.y, batch = bh / H, head = bh % H, row0 = rb * R;
  const int chunks = (T_ + L - 1) / L;
  const long NN = (long)N * N;
  const float* recs = work + (long)bh * chunks * Rec<N>::FLOATS;
  scan_issue<T, N>(stage[0], recs, pv, T_, H, batch, head, 0, row0, pv);
  for (int e = threadIdx.x; e < R * N; e += THREADS) {
    const int i = e / N, j = e % N;
    S[i * SP + j] = s0[bh * NN + (long)(row0 + i) * N + j];
  }
  for (int ch = 0; ch < chunks; ++ch) {
    const int t0 = ch * L;
    float* cur = stage[ch & 1];
    if (ch + 1 < chunks) {
      scan_issue<T, N>(stage[(ch + 1) & 1], recs + (long)(ch + 1) * Rec<N>::FLOATS, pv, T_, H, batch, head, t0 + L,
                       row0, pv);
      rt::cp_async_wait<1>();
    } else {
      rt::cp_async_wait<0>();
    }
    __syncthreads();
    const float* W = cur;
    const float* Q = cur + L * SP;
    const float* BH = cur + 2 * L * SP;
    const float* KH = cur + 3 * L * SP;
    const float* U0 = cur + 4 * L * SP;
    const float* Y0 = U0 + L * R;
    const T* V = reinterpret_cast<const T*>(U0 + 2 * L * R);
    const float* DL = U0 + 3 * L * R;
    if (checkpoints) {
      float* dst = checkpoints + ((long)bh * (chunks + 1) + ch) * NN;
      for (int e = threadIdx.x; e < R * (N / 4); e += THREADS) {
        const int i = e / (N / 4), j = (e % (N / 4)) * 4;
        *reinterpret_cast<float4*>(dst + (long)(row0 + i) * N + j) = *reinterpret_cast<const float4*>(S + i * SP + j);
      }
    }
    // U[t][i] = U0 + W[t] . S[i];  Y[t][i] = Y0 + Q[t] . S[i]  (two outputs of each kind per thread)
    for (int e = threadIdx.x; e < L * R; e += THREADS) {
      const int t = e / R, i = e % R;
      const float4* wt = reinterpret_cast<const float4*>(W + t * SP);
      const float4* qt = reinterpret_cast<const float4*>(Q + t * SP);
      const float4* si = reinterpret_cast<const float4*>(S + i * SP);
      float u = U0[e], y = Y0[e];
#pragma unroll 8
      for (int q = 0; q < N / 4; ++q) {
        const float4 s4 = si[q], w4 = wt[q], q4 = qt[q];
        u += w4.x * s4.x + w4.y * s4.y + w4.z * s4.z + w4.w * s4.w;
        y += q4.x * s4.x + q4.y * s4.y + q4.z * s4.z + q4.w * s4.w;
      }
      U[e] = u;
      const int tg = t0 + t;
      if (tg < T_) py[(((long)batch * T_ + tg) * H + head) * N + row0 + i] = rt::from_f<T>(y);
    }
    __syncthreads();
    // S[i][j] = S[i][j] D_L[j] + sum_t U[t][i] B^[t][j] + V[t][i] K^[t][j]; thread: 4 consecutive j, R*N/512 rows
    for (int e = threadIdx.x; e < R * (N / 4); e += THREADS) {
      const int i = e / (N / 4), j = (e % (N / 4)) * 4;
      float4 acc = *reinterpret_cast<const float4*>(S + i * SP + j);
      const float4 d = *reinterpret_cast<const float4*>(DL + j);
      acc.x *= d.x; acc.y *= d.y; acc.z *= d.z; acc.w *= d.w;
#pragma unroll
      for (int t = 0; t < L; ++t) {
        const float u = U[t * R + i], vv = rt::to_f(V[t * R + i]);
        const float4 b4 = *reinterpret_cast<const float4*>(BH + t * SP + j);
        const float4 k4 = *reinterpret_cast<const float4*>(KH + t * SP + j);
        acc.x += u * b4.x + vv * k4.x;
        acc.y += u * b4.y + vv * k4.y;
        acc.z += u * b4.z + vv * k4.z;
        acc.w += u * b4.w + vv * k4.w;
      }
      *reinterpret_cast<float4*>(S + i * SP + j) = acc;
    }
    __syncthreads();
  }
  float* fin = checkpoints ? checkpoints + ((long)bh * (chunks + 1) + chunks) * NN : nullptr;
  for (int e = threadIdx.x; e < R * N; e += THREADS) {
    const int i = e / N, j = e % N;
    s_end[bh * NN + (long)(row0 + i) * N + j] = S[i * SP + j];
    if (fin) fin[(long)(row0 + i) * N + j] = S[i * SP + j];
  }
}

template <typename T, int N>
cudaError_t launch(int B, int T_, int H, const void* r, const void* w, const void* k, const void* v, const void* a,
                   const void* b, const float* s0, void* y, float* s_end, float* ckpt, float* work,
                   cudaStream_t stream) {
  const int chunks = (T_ + L - 1) / L;
  constexpr int chunk_smem = (6 * L * (N + 4) + 5 * L * (L + 1) + N) * 4;
  RT_CUDA_CHECK(cudaFuncSetAttribute(wkv7_chunk_kernel<T, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, chunk_smem));
  wkv7_chunk_kernel<T, N><<<dim3(chunks, B * H), THREADS, chunk_smem, stream>>>(
      T_, H, (const T*)r, (const T*)w, (const T*)k, (const T*)v, (const T*)a, (const T*)b, work);
  RT_CUDA_CHECK(cudaGetLastError());
  const int smem = ScanSmem<N>::FLOATS * 4;
  RT_CUDA_CHECK(cudaFuncSetAttribute(wkv7_scan_kernel<T, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  wkv7_scan_kernel<T, N><<<dim3(N / R, B * H), THREADS, smem, stream>>>(T_, H, (const T*)v, s0, work, (T*)y, s_end,
                                                                         ckpt);
  return cudaGetLastError();
}

}  // namespace

// Workspace floats of the two-pass forward (0 when the head size is not 32, 64 or 128).
extern "C" long rt_wkv7_scan_workspace_floats(int B, int T_, int H, int N) {
  const long chunks = (T_ + L - 1) / L;
  switch (N) {
    case 32: return (long)B * H * chunks * Rec<32>::FLOATS;
    case 64: return (long)B * H * chunks * Rec<64>::FLOATS;
    case 128: return (long)B * H * chunks * Rec<128>::FLOATS;
    default: return 0;
  }
}

extern "C" cudaError_t rt_wkv7_scan_forward(int dtype, int B, int T_, int H, int N, const void* r, const void* w,
                                            const void* k, const void* v, const void* a, const void* b,
                                            const float* s0, void* y, float* s_end, float* checkpoints, float* work,
                                            cudaStream_t stream) {
#define RT_SCAN(TYPE)                                                                                              \
  switch (N) {                                                                                                     \
    case 32: return launch<TYPE, 32>(B, T_, H, r, w, k, v, a, b, s0, y, s_end, checkpoints, work, stream);        \
    case 64: return launch<TYPE, 64>(B, T_, H, r, w, k, v, a, b, s0, y, s_end, checkpoints, work, stream);        \
    case 128: return launch<TYPE, 128>(B, T_, H, r, w, k, v, a, b, s0, y, s_end, checkpoints, work, stream);      \
    default: return cudaErrorInvalidValue;                                                                         \
  }
  if (dtype == 1) { RT_SCAN(__nv_bfloat16) }
  RT_SCAN(float)
#undef RT_SCAN
}
