// Chunked RWKV7 (WKV7) state recurrence, forward and backward, for sm_100a.
// The recurrence is RWKV7's (RWKV-LM, Apache-2.0; see NOTICE at the project root); this code is our own.
//
// Semantics match the reference kernel (kernels/wkv7_state.cu:12-79 of the
// reference project): state S[value i][key j] per (batch, head),
//   d_t = exp(-e^{-1/2} sigmoid(w_t)),  S_t = S_{t-1} diag(d_t) + (S_{t-1} a_t) b_t^T + v_t k_t^T,
//   y_t = S_t r_t,
// with an explicit initial state s0 and final state output.
//
// Algorithm (own design; this file holds the forward, wkv7_bwd.cu the backward):
// the sequence is cut into chunks of L = 16 steps.
// With Lambda_t the cumulative log decay inside a chunk and
//   a~_t = a_t e^{Lambda_{t-1}}, r~_t = r_t e^{Lambda_t}, b~_s = b_s e^{-Lambda_s}, k~_s = k_s e^{-Lambda_s},
// the per-chunk update of every value row is
//   U = (I - Mab)^{-1} (A~ S0^T + Mak V)             (u_t = S_{t-1} a_t)
//   Y = R~ S0^T + Mrb U + Mrk V
//   S_L = S0 diag(D_L) + U^T (B~ D_L) + V^T (K~ D_L)
// where Mxy[t][s] = x~_t . y~_s (strictly lower for a-rows, inclusive for
// r-rows). Value rows are independent, so each CTA owns R = 16 rows of one
// head and the head's rows are spread over N/16 CTAs. The forward pass keeps
// S in shared memory, prefetches the next chunk's inputs with cp.async while
// the current chunk computes, and stores only chunk-start states
// ("checkpoints") when a backward is needed. Padded tail steps use zero
// inputs and zero log-decay.
#include <initializer_list>
#include "../common/common.cuh"


namespace {

constexpr int L = 16;        // chunk length
constexpr int R = 16;        // value rows per CTA
constexpr int THREADS = 128;
constexpr float DECAY_SCALE = 0.6065306597126334f;

template <int NP>
struct Smem {
  static constexpr int SP = NP + 4;         // padded row stride (float4-aligned, conflict-free)
  static constexpr int KEY = L * SP;        // one [L][SP] key-side array
  static constexpr int ROWS = L * R;        // one [L][R] row-side array
  static constexpr int MAT = L * (L + 1);   // one [L][L+1] chunk matrix
  static constexpr int STATE = R * SP;      // [R][SP]
  // Partial sums reduced across the cluster in the backward pass.
  static constexpr int PART = 4 * MAT + 4 * KEY + NP;
};

// Raw (input dtype) staging of one chunk: r, w, k, a, b [L][NP], v and dy [L][R] (dy in backward),
// filled by 16-byte cp.async copies (zero-filled outside the sequence / head) one chunk ahead.
template <typename T, int NP>
struct Raw {
  static constexpr int VEC = 16 / sizeof(T);
  static constexpr int KEYV = L * NP;
  static constexpr int ELEMS = 5 * KEYV + 2 * L * R;
  static constexpr int FLOATS = (ELEMS * (int)sizeof(T) + 15) / 16 * 4;  // size in floats, 16-byte multiple
};

// Issues the copies of chunk t0 into `raw` (one commit group per call).
template <typename T, int NP, bool ASYNC>
RT_DEVICE void issue_chunk(T* raw, const T* pr, const T* pw, const T* pk, const T* pa, const T* pb, const T* pv,
                           const T* pdy, int T_, int H, int N, int batch, int head, int t0, int row0) {
  using RW = Raw<T, NP>;
  constexpr int VEC = RW::VEC, QV = NP / VEC;
  for (int e = threadIdx.x; e < 5 * L * QV; e += THREADS) {
    const int tensor = e / (L * QV), rem = e % (L * QV), tt = rem / QV, j = (rem % QV) * VEC;
    const int t = t0 + tt;
    const bool ok = (t < T_) && (j < N);
    const T* base = tensor == 0 ? pr : tensor == 1 ? pw : tensor == 2 ? pk : tensor == 3 ? pa : pb;
    const T* src = base + (ok ? ((long)(batch * T_ + t) * H + head) * N + j : 0);
    T* dst = raw + tensor * RW::KEYV + tt * NP + j;
    if (ASYNC) {
      rt::cp_async16(dst, src, ok);
    } else {
#pragma unroll
      for (int u = 0; u < VEC; ++u) dst[u] = (ok && j + u < N) ? src[u] : rt::from_f<T>(0.f);
    }
  }
  constexpr int RV = R / VEC;
  const int rows_arrays = pdy ? 2 : 1;
  for (int e = threadIdx.x; e < rows_arrays * L * RV; e += THREADS) {
    const int which = e / (L * RV), rem = e % (L * RV), tt = rem / RV, i = (rem % RV) * VEC;
    const int t = t0 + tt, row = row0 + i;
    const bool ok = (t < T_) && (row < N);
    const T* base = which ? pdy : pv;
    const T* src = base + (ok ? ((long)(batch * T_ + t) * H + head) * N + row : 0);
    T* dst = raw + 5 * RW::KEYV + which * L * R + tt * R + i;
    if (ASYNC) {
      rt::cp_async16(dst, src, ok);
    } else {
#pragma unroll
      for (int u = 0; u < VEC; ++u) dst[u] = (ok && row + u < N) ? src[u] : rt::from_f<T>(0.f);
    }
  }
  if (ASYNC) rt::cp_async_commit();
}

// Per-chunk preparation from the raw staging: cumulative log decay, decayed vectors, D_L and the four
// chunk matrices (fp32 in shared memory).
template <typename T, int NP>
struct Chunk {
  using S = Smem<NP>;
  float *r, *a, *b, *k, *lam, *sig, *dl, *v, *M;

  RT_DEVICE void bind(float* base) {
    r = base; a = r + S::KEY; b = a + S::KEY; k = b + S::KEY; lam = k + S::KEY; sig = lam + S::KEY;
    dl = sig + S::KEY; v = dl + NP; M = v + S::ROWS;
  }
  static constexpr int FLOATS = 6 * S::KEY + NP + S::ROWS + 4 * S::MAT;

  // dy_out (optional): receives the chunk's output gradient rows as fp32 [L][R].
  RT_DEVICE void prepare(const T* raw, int T_, int N, int t0, float* dy_out) {
    using RW = Raw<T, NP>;
    const int tid = threadIdx.x;
    for (int e = tid; e < L * NP; e += THREADS) {
      const int tt = e / NP, j = e % NP;
      const bool ok = (t0 + tt < T_) && (j < N);
      const int o = tt * S::SP + j;
      r[o] = rt::to_f<T>(raw[0 * RW::KEYV + e]);
      k[o] = rt::to_f<T>(raw[2 * RW::KEYV + e]);
      a[o] = rt::to_f<T>(raw[3 * RW::KEYV + e]);
      b[o] = rt::to_f<T>(raw[4 * RW::KEYV + e]);
      const float sg = ok ? rt::sigmoidf_(rt::to_f<T>(raw[1 * RW::KEYV + e])) : 0.f;
      sig[o] = sg;
      lam[o] = -DECAY_SCALE * sg;
    }
    for (int e = tid; e < L * R; e += THREADS) {
      v[e] = rt::to_f<T>(raw[5 * RW::KEYV + e]);
      if (dy_out) dy_out[e] = rt::to_f<T>(raw[5 * RW::KEYV + L * R + e]);
    }
    __syncthreads();
    if (tid < NP) {
      float run = 0.f;
#pragma unroll
      for (int tt = 0; tt < L; ++tt) {
        run += lam[tt * S::SP + tid];
        lam[tt * S::SP + tid] = run;
      }
      dl[tid] = expf(run);
    }
    __syncthreads();
    for (int e = tid; e < L * NP; e += THREADS) {
      const int tt = e / NP, j = e % NP, o = tt * S::SP + j;
      const float cur = lam[o];
      const float prev = tt ? lam[o - S::SP] : 0.f;
      const float ec = expf(cur), inv = 1.f / ec;
      r[o] *= ec;
      a[o] *= expf(prev);
      b[o] *= inv;
      k[o] *= inv;
    }
    __syncthreads();
    // Chunk matrices: M[0]=Mab (s<t), M[1]=Mak (s<t), M[2]=Mrb (s<=t), M[3]=Mrk (s<=t).
    {
      const int t = tid >> 3, s0 = tid & 7, s1 = s0 + 8;
      float ab0 = 0, ak0 = 0, rb0 = 0, rk0 = 0, ab1 = 0, ak1 = 0, rb1 = 0, rk1 = 0;
      const float4* at = reinterpret_cast<const float4*>(a + t * S::SP);
      const float4* rt4 = reinterpret_cast<const float4*>(r + t * S::SP);
      const float4* b0 = reinterpret_cast<const float4*>(b + s0 * S::SP);
      const float4* k0 = reinterpret_cast<const float4*>(k + s0 * S::SP);
      const float4* b1 = reinterpret_cast<const float4*>(b + s1 * S::SP);
      const float4* k1 = reinterpret_cast<const float4*>(k + s1 * S::SP);
#pragma unroll 4
      for (int q = 0; q < NP / 4; ++q) {
        const float4 x = at[q], y = rt4[q], p = b0[q], u = k0[q], p1 = b1[q], u1 = k1[q];
        ab0 += x.x * p.x + x.y * p.y + x.z * p.z + x.w * p.w;
        ak0 += x.x * u.x + x.y * u.y + x.z * u.z + x.w * u.w;
        rb0 += y.x * p.x + y.y * p.y + y.z * p.z + y.w * p.w;
        rk0 += y.x * u.x + y.y * u.y + y.z * u.z + y.w * u.w;
        ab1 += x.x * p1.x + x.y * p1.y + x.z * p1.z + x.w * p1.w;
        ak1 += x.x * u1.x + x.y * u1.y + x.z * u1.z + x.w * u1.w;
        rb1 += y.x * p1.x + y.y * p1.y + y.z * p1.z + y.w * p1.w;
        rk1 += y.x * u1.x + y.y * u1.y + y.z * u1.z + y.w * u1.w;
      }
      const int o0 = t * (L + 1) + s0, o1 = t * (L + 1) + s1;
      M[0 * S::MAT + o0] = s0 < t ? ab0 : 0.f;
      M[1 * S::MAT + o0] = s0 < t ? ak0 : 0.f;
      M[2 * S::MAT + o0] = s0 <= t ? rb0 : 0.f;
      M[3 * S::MAT + o0] = s0 <= t ? rk0 : 0.f;
      M[0 * S::MAT + o1] = s1 < t ? ab1 : 0.f;
      M[1 * S::MAT + o1] = s1 < t ? ak1 : 0.f;
      M[2 * S::MAT + o1] = s1 <= t ? rb1 : 0.f;
      M[3 * S::MAT + o1] = s1 <= t ? rk1 : 0.f;
    }
    __syncthreads();
  }

  RT_DEVICE float m(int which, int t, int s) const { return M[which * S::MAT + t * (L + 1) + s]; }
};

// Issues the copy of the fp32 chunk-start state rows [R][NP] of this CTA (backward).
template <int NP, bool ASYNC>
RT_DEVICE void issue_state(float* dst, const float* src_state, int N, int row0) {
  constexpr int QV = NP / 4;
  for (int e = threadIdx.x; e < R * QV; e += THREADS) {
    const int i = e / QV, j = (e % QV) * 4, row = row0 + i;
    const bool ok = row < N && j < N;
    const float* src = src_state + (ok ? (long)row * N + j : 0);
    if (ASYNC) {
      rt::cp_async16(dst + i * NP + j, src, ok);
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u) dst[i * NP + j + u] = (ok && j + u < N) ? src[u] : 0.f;
    }
  }
  if (ASYNC) rt::cp_async_commit();
}

// Z[t][i] = a~_t . S0_i + sum_{s<t} Mak[t][s] v[s][i]; Yp = r~_t . S0_i + sum_{s<=t} Mrk[t][s] v[s][i];
// then U by forward substitution. Leaves Z, U (and Yp if requested) in shared memory.
template <typename T, int NP>
RT_DEVICE void solve_u(const Chunk<T, NP>& c, const float* S0, float* Z, float* U, float* Yp) {
  using S = Smem<NP>;
  for (int e = threadIdx.x; e < L * R; e += THREADS) {
    const int t = e / R, i = e % R;
    const float4* at = reinterpret_cast<const float4*>(c.a + t * S::SP);
    const float4* rt4 = reinterpret_cast<const float4*>(c.r + t * S::SP);
    const float4* si = reinterpret_cast<const float4*>(S0 + i * S::SP);
    float z = 0.f, y = 0.f;
#pragma unroll 4
    for (int q = 0; q < NP / 4; ++q) {
      const float4 s = si[q], x = at[q], w = rt4[q];
      z += x.x * s.x + x.y * s.y + x.z * s.z + x.w * s.w;
      y += w.x * s.x + w.y * s.y + w.z * s.z + w.w * s.w;
    }
    for (int s = 0; s < t; ++s) z += c.m(1, t, s) * c.v[s * R + i];
    for (int s = 0; s <= t; ++s) y += c.m(3, t, s) * c.v[s * R + i];
    Z[e] = z;
    if (Yp) Yp[e] = y;
  }
  __syncthreads();
  if (threadIdx.x < R) {
    const int i = threadIdx.x;
    for (int t = 0; t < L; ++t) {
      float u = Z[t * R + i];
      for (int s = 0; s < t; ++s) u += c.m(0, t, s) * U[s * R + i];
      U[t * R + i] = u;
    }
  }
  __syncthreads();
}

template <typename T, int NP, bool ASYNC>
__global__ void __launch_bounds__(THREADS)
wkv7_forward_kernel(int T_, int H, int N, const T* __restrict__ pr, const T* __restrict__ pw,
                    const T* __restrict__ pk, const T* __restrict__ pv, const T* __restrict__ pa,
                    const T* __restrict__ pb, const float* __restrict__ s0, T* __restrict__ py,
                    float* __restrict__ s_end, float* __restrict__ checkpoints) {
  using S = Smem<NP>;
  using RW = Raw<T, NP>;
  extern __shared__ __align__(16) float smem[];
  constexpr int ST = ASYNC ? 2 : 1;
  T* raw[2] = {reinterpret_cast<T*>(smem), reinterpret_cast<T*>(smem + (ST - 1) * RW::FLOATS)};
  Chunk<T, NP> c;
  c.bind(smem + ST * RW::FLOATS);
  float* St = smem + ST * RW::FLOATS + Chunk<T, NP>::FLOATS;
  float* Z = St + S::STATE;
  float* U = Z + S::ROWS;
  float* Y = U + S::ROWS;
  const int rb = blockIdx.x, bh = blockIdx.y, batch = bh / H, head = bh % H, row0 = rb * R;
  const int chunks = (T_ + L - 1) / L;
  const long NN = (long)N * N;
  if (ASYNC) issue_chunk<T, NP, ASYNC>(raw[0], pr, pw, pk, pa, pb, pv, nullptr, T_, H, N, batch, head, 0, row0);
  for (int e = threadIdx.x; e < R * NP; e += THREADS) {
    const int i = e / NP, j = e % NP, row = row0 + i;
    St[i * S::SP + j] = (row < N && j < N) ? s0[bh * NN + (long)row * N + j] : 0.f;
  }
  for (int ch = 0; ch < chunks; ++ch) {
    const int t0 = ch * L;
    if (checkpoints) {
      float* dst = checkpoints + ((long)bh * (chunks + 1) + ch) * NN;
      for (int e = threadIdx.x; e < R * NP; e += THREADS) {
        const int i = e / NP, j = e % NP, row = row0 + i;
        if (row < N && j < N) dst[(long)row * N + j] = St[i * S::SP + j];
      }
    }
    if constexpr (ASYNC) {
      if (ch + 1 < chunks) {
        issue_chunk<T, NP, ASYNC>(raw[(ch + 1) & 1], pr, pw, pk, pa, pb, pv, nullptr, T_, H, N, batch, head,
                                  t0 + L, row0);
        rt::cp_async_wait<1>();
      } else {
        rt::cp_async_wait<0>();
      }
    } else {
      issue_chunk<T, NP, ASYNC>(raw[0], pr, pw, pk, pa, pb, pv, nullptr, T_, H, N, batch, head, t0, row0);
    }
    __syncthreads();
    c.prepare(raw[ASYNC ? (ch & 1) : 0], T_, N, t0, nullptr);
    solve_u<T, NP>(c, St, Z, U, Y);
    for (int e = threadIdx.x; e < L * R; e += THREADS) {
      const int t = e / R, i = e % R;
      float y = Y[e];
      for (int s = 0; s <= t; ++s) y += c.m(2, t, s) * U[s * R + i];
      const int tg = t0 + t, row = row0 + i;
      if (tg < T_ && row < N) py[((long)(batch * T_ + tg) * H + head) * N + row] = rt::from_f<T>(y);
    }
    for (int e = threadIdx.x; e < R * NP; e += THREADS) {
      const int i = e / NP, j = e % NP;
      const float d = c.dl[j];
      float acc = St[i * S::SP + j] * d;
#pragma unroll
      for (int s = 0; s < L; ++s)
        acc += (U[s * R + i] * c.b[s * S::SP + j] + c.v[s * R + i] * c.k[s * S::SP + j]) * d;
      St[i * S::SP + j] = acc;
    }
    __syncthreads();
  }
  float* fin = checkpoints ? checkpoints + ((long)bh * (chunks + 1) + chunks) * NN : nullptr;
  for (int e = threadIdx.x; e < R * NP; e += THREADS) {
    const int i = e / NP, j = e % NP, row = row0 + i;
    if (row < N && j < N) {
      s_end[bh * NN + (long)row * N + j] = St[i * S::SP + j];
      if (fin) fin[(long)row * N + j] = St[i * S::SP + j];
    }
  }
}

template <int NP>
constexpr int padded_np() { return NP; }

int pick_np(int N) { return N <= 16 ? 16 : N <= 32 ? 32 : N <= 64 ? 64 : 128; }

bool async_ok(int N, int elem, std::initializer_list<const void*> ptrs) {
  if ((N * elem) % 16 || (N % 4)) return false;
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) & 15) return false;
  return true;
}

template <typename T, int NP, bool ASYNC>
cudaError_t launch_fwd_impl(int B, int T_, int H, int N, const void* r, const void* w, const void* k, const void* v,
                            const void* a, const void* b, const float* s0, void* y, float* s_end, float* ckpt,
                            cudaStream_t stream) {
  using S = Smem<NP>;
  constexpr int ST = ASYNC ? 2 : 1;
  const size_t bytes = (ST * Raw<T, NP>::FLOATS + Chunk<T, NP>::FLOATS + S::STATE + 3 * S::ROWS) * sizeof(float);
  auto kern = wkv7_forward_kernel<T, NP, ASYNC>;
  RT_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  dim3 grid(NP / R, B * H);
  kern<<<grid, THREADS, bytes, stream>>>(T_, H, N, (const T*)r, (const T*)w, (const T*)k, (const T*)v,
                                         (const T*)a, (const T*)b, s0, (T*)y, s_end, ckpt);
  return cudaGetLastError();
}

template <typename T, int NP>
cudaError_t launch_fwd(int B, int T_, int H, int N, const void* r, const void* w, const void* k, const void* v,
                       const void* a, const void* b, const float* s0, void* y, float* s_end, float* ckpt,
                       cudaStream_t stream) {
  if (async_ok(N, sizeof(T), {r, w, k, v, a, b}))
    return launch_fwd_impl<T, NP, true>(B, T_, H, N, r, w, k, v, a, b, s0, y, s_end, ckpt, stream);
  return launch_fwd_impl<T, NP, false>(B, T_, H, N, r, w, k, v, a, b, s0, y, s_end, ckpt, stream);
}

}  // namespace

// Chunk length used by the checkpoint layout [B, H, ceil(T/16) + 1, N, N].
extern "C" int rt_wkv7_chunk_len() { return L; }

extern "C" cudaError_t rt_wkv7_step(int dtype, int B, int T_, int H, int N, const void* r, const void* w,
                                    const void* k, const void* v, const void* a, const void* b, const float* s0,
                                    void* y, float* s_end, cudaStream_t stream);

// Decode-sized calls without checkpoints (T <= 4) take the token-by-token kernel (wkv7_step.cu).
constexpr int STEP_MAX_T = 4;

extern "C" cudaError_t rt_wkv7_forward(int dtype, int B, int T_, int H, int N, const void* r, const void* w,
                                       const void* k, const void* v, const void* a, const void* b,
                                       const float* s0, void* y, float* s_end, float* checkpoints,
                                       cudaStream_t stream) {
  if (!checkpoints && T_ <= STEP_MAX_T && (N == 32 || N == 64 || N == 128))
    return rt_wkv7_step(dtype, B, T_, H, N, r, w, k, v, a, b, s0, y, s_end, stream);
  const int np = pick_np(N);
#define RT_FWD(TYPE, NPV) return launch_fwd<TYPE, NPV>(B, T_, H, N, r, w, k, v, a, b, s0, y, s_end, checkpoints, stream)
#define RT_FWD_NP(TYPE)                                   \
  switch (np) {                                           \
    case 16: RT_FWD(TYPE, 16);                            \
    case 32: RT_FWD(TYPE, 32);                            \
    case 64: RT_FWD(TYPE, 64);                            \
    default: RT_FWD(TYPE, 128);                           \
  }
  if (dtype == (int)rt::DType::BF16) { RT_FWD_NP(__nv_bfloat16) } else { RT_FWD_NP(float) }
#undef RT_FWD_NP
#undef RT_FWD
}

