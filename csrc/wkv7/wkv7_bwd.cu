// WKV7 backward for sm_100a in three kernels (chunk length 16):
// The recurrence is RWKV7's (RWKV-LM, Apache-2.0; see NOTICE at the project root); this code is our own.
//
//   1. prep   (one CTA per head and chunk, parallel): cumulative log decay,
//             decayed vectors r~, a~, b^ = b~ D_L, D_L, the chunk matrix M_rb
//             and W = (I - M_ab)^{-1} (forward substitution per column).
//   2. state  (per head and 16 value rows, serial over chunks in reverse):
//             only the state-gradient recurrence
//                 dU = M_rb^T dY + B^ dS^T,  dZ = W^T dU,
//                 dS <- dS diag(D_L) + dY^T R~ + dZ^T A~,
//             writing dS at the end of every chunk. Small shared memory so
//             every CTA of the grid is resident; the next chunk's inputs are
//             copied with cp.async while the current one computes.
//   3. grads  (one CTA per head and chunk, parallel, all value rows): with the
//             chunk-start state S0 (forward checkpoint) and the chunk-end
//             gradient dS (kernel 2) it recomputes U and forms every input
//             gradient: dv row-wise, and the key-side gradients (dr, dw, dk,
//             da, db) as sums over all value rows inside one CTA — no cluster,
//             no atomics, deterministic.
//
// Notation (per chunk, t/s steps, i value rows, j keys): Lambda_t cumulative
// log decay, a~_t = a_t e^{Lambda_{t-1}}, r~_t = r_t e^{Lambda_t}, b~_s = b_s
// e^{-Lambda_s}, k~_s = k_s e^{-Lambda_s}; M_xy[t][s] = x~_t . y~_s (strict
// lower for a-rows, inclusive for r-rows); forward: U = W (A~ S0^T + M_ak V),
// Y = R~ S0^T + M_rb U + M_rk V, S_L = S0 D_L + U^T B^ + V^T K^ with B^ = B~ D_L.
#include <initializer_list>
#include "../common/common.cuh"

namespace {

constexpr int L = 16;
constexpr int R = 16;
constexpr float DECAY_SCALE = 0.6065306597126334f;

// ---------------------------------------------------------------- shared chunk preparation
// Loads one chunk of r, w, k, a, b (and optionally v, dy as [L][NP] value-major rows) for all keys of a
// head, builds decays and the requested chunk matrices. Arrays are [L][SP] fp32 in shared memory.
template <int NP>
struct Keys {
  static constexpr int SP = NP + 4;
  static constexpr int KEY = L * SP;
  static constexpr int MAT = L * (L + 1);
  float *r, *a, *b, *k, *lam, *sig, *dl;
  RT_DEVICE static int floats() { return 6 * KEY + NP; }
  RT_DEVICE void bind(float* p) {
    r = p; a = r + KEY; b = a + KEY; k = b + KEY; lam = k + KEY; sig = lam + KEY; dl = sig + KEY;
  }
};

template <typename T, int NP>
RT_DEVICE void load_keys(Keys<NP>& c, const T* pr, const T* pw, const T* pk, const T* pa, const T* pb, int T_, int H,
                         int N, int batch, int head, int t0, int threads) {
  constexpr int SP = Keys<NP>::SP;
  for (int e = threadIdx.x; e < L * NP; e += threads) {
    const int tt = e / NP, j = e % NP, t = t0 + tt;
    const bool ok = (t < T_) && (j < N);
    const long idx = ((long)(batch * T_ + t) * H + head) * N + j;
    const int o = tt * SP + j;
    c.r[o] = ok ? rt::to_f<T>(pr[idx]) : 0.f;
    c.k[o] = ok ? rt::to_f<T>(pk[idx]) : 0.f;
    c.a[o] = ok ? rt::to_f<T>(pa[idx]) : 0.f;
    c.b[o] = ok ? rt::to_f<T>(pb[idx]) : 0.f;
    const float sg = ok ? rt::sigmoidf_(rt::to_f<T>(pw[idx])) : 0.f;
    c.sig[o] = sg;
    c.lam[o] = -DECAY_SCALE * sg;
  }
  __syncthreads();
  if (threadIdx.x < NP) {
    float run = 0.f;
#pragma unroll
    for (int tt = 0; tt < L; ++tt) {
      run += c.lam[tt * SP + threadIdx.x];
      c.lam[tt * SP + threadIdx.x] = run;
    }
    c.dl[threadIdx.x] = expf(run);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < L * NP; e += threads) {
    const int tt = e / NP, j = e % NP, o = tt * SP + j;
    const float cur = c.lam[o], prev = tt ? c.lam[o - SP] : 0.f;
    const float ec = expf(cur), inv = 1.f / ec;
    c.r[o] *= ec;
    c.a[o] *= expf(prev);
    c.b[o] *= inv;
    c.k[o] *= inv;
  }
  __syncthreads();
}

// dot of two [.][SP] rows over NP (float4)
template <int NP>
RT_DEVICE float rowdot(const float* x, const float* y) {
  const float4* p = reinterpret_cast<const float4*>(x);
  const float4* q = reinterpret_cast<const float4*>(y);
  float acc = 0.f;
#pragma unroll 4
  for (int u = 0; u < NP / 4; ++u) {
    const float4 m = p[u], n = q[u];
    acc += m.x * n.x + m.y * n.y + m.z * n.z + m.w * n.w;
  }
  return acc;
}

// sum_j x[j] y[j] z[j] over NP (float4; all three 16-byte aligned)
template <int NP>
RT_DEVICE float dot3(const float* x, const float* y, const float* z) {
  const float4* p = reinterpret_cast<const float4*>(x);
  const float4* q = reinterpret_cast<const float4*>(y);
  const float4* w = reinterpret_cast<const float4*>(z);
  float acc = 0.f;
#pragma unroll 4
  for (int u = 0; u < NP / 4; ++u) {
    const float4 a = p[u], b = q[u], c = w[u];
    acc += a.x * b.x * c.x + a.y * b.y * c.y + a.z * b.z * c.z + a.w * b.w * c.w;
  }
  return acc;
}

// Register tile of a chunk product over keys: acc[r][k] += sum_j X[tb + r][j] (dl[j]) Y[i_k][j] for 4 steps
// tb..tb+3 and two value rows i0, i1 (rows of stride SP, NP keys, float4 loads). X rows are shared by a warp
// (broadcast); Y rows i0 = consecutive per thread (conflict-free for SP = NP + 4).
template <int NP, bool SCALE>
RT_DEVICE void tile42(const float* X, int tb, const float* Y, int i0, int i1, const float* dl, int SP,
                      float (&acc)[4][2]) {
#pragma unroll 4
  for (int q = 0; q < NP / 4; ++q) {
    float4 y0 = reinterpret_cast<const float4*>(Y + i0 * SP)[q];
    float4 y1 = reinterpret_cast<const float4*>(Y + i1 * SP)[q];
    if (SCALE) {
      const float4 d = reinterpret_cast<const float4*>(dl)[q];
      y0.x *= d.x; y0.y *= d.y; y0.z *= d.z; y0.w *= d.w;
      y1.x *= d.x; y1.y *= d.y; y1.z *= d.z; y1.w *= d.w;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float4 x = reinterpret_cast<const float4*>(X + (tb + r) * SP)[q];
      acc[r][0] += x.x * y0.x + x.y * y0.y + x.z * y0.z + x.w * y0.w;
      acc[r][1] += x.x * y1.x + x.y * y1.y + x.z * y1.z + x.w * y1.w;
    }
  }
}

// W = (I - Mab)^{-1} for strictly lower Mab ([L][L+1]); 16 threads, one column each.
RT_DEVICE void unit_lower_inverse(const float* Mab, float* W) {
  if (threadIdx.x < L) {
    const int c = threadIdx.x;
    for (int t = 0; t < L; ++t) {
      float w = (t == c) ? 1.f : 0.f;
      if (t > c)
        for (int s = c; s < t; ++s) w += Mab[t * (L + 1) + s] * W[s * (L + 1) + c];
      W[t * (L + 1) + c] = w;
    }
  }
}

// ---------------------------------------------------------------- 1. prep
// prep record per (bh, chunk): Rt[L][NP], At[L][NP], Bh[L][NP], DL[NP], W[L][L], Mrb[L][L], DY[L][NP]
// (dy rows in fp32, value-major, so the state pass copies 16-byte aligned slices for any head size).
template <int NP>
struct Prep {
  static constexpr int KEYS = 3 * L * NP + NP + 2 * L * L;
  static constexpr int FLOATS = KEYS + L * NP;
};

template <int NP>
constexpr int prep_smem_floats() { return 6 * Keys<NP>::KEY + NP + 3 * Keys<NP>::MAT; }

template <typename T, int NP>
__global__ void __launch_bounds__(128)
wkv7_bwd_prep_kernel(int T_, int H, int N, const T* __restrict__ pr, const T* __restrict__ pw,
                     const T* __restrict__ pk, const T* __restrict__ pa, const T* __restrict__ pb,
                     const T* __restrict__ pdy, float* __restrict__ prep) {
  using K = Keys<NP>;
  extern __shared__ __align__(16) float sm[];
  K c;
  c.bind(sm);
  float* Mab = sm + 6 * K::KEY + NP;
  float* Mrb = Mab + K::MAT;
  float* W = Mrb + K::MAT;
  const int ch = blockIdx.x, bh = blockIdx.y, batch = bh / H, head = bh % H;
  const int chunks = gridDim.x;
  load_keys<T, NP>(c, pr, pw, pk, pa, pb, T_, H, N, batch, head, ch * L, 128);
  for (int e = threadIdx.x; e < 2 * L * L; e += 128) {
    const int which = e / (L * L), t = (e % (L * L)) / L, s = e % L;
    if (which == 0) Mab[t * (L + 1) + s] = s < t ? rowdot<NP>(c.a + t * K::SP, c.b + s * K::SP) : 0.f;
    else Mrb[t * (L + 1) + s] = s <= t ? rowdot<NP>(c.r + t * K::SP, c.b + s * K::SP) : 0.f;
  }
  __syncthreads();
  unit_lower_inverse(Mab, W);
  __syncthreads();
  float* out = prep + ((long)bh * chunks + ch) * Prep<NP>::FLOATS;
  for (int e = threadIdx.x; e < L * NP; e += 128) {
    const int tt = e / NP, j = e % NP, o = tt * K::SP + j;
    out[e] = c.r[o];
    out[L * NP + e] = c.a[o];
    out[2 * L * NP + e] = c.b[o] * c.dl[j];
  }
  if (threadIdx.x < NP) out[3 * L * NP + threadIdx.x] = c.dl[threadIdx.x];
  for (int e = threadIdx.x; e < L * L; e += 128) {
    const int t = e / L, s = e % L;
    out[3 * L * NP + NP + e] = W[t * (L + 1) + s];
    out[3 * L * NP + NP + L * L + e] = Mrb[t * (L + 1) + s];
  }
  for (int e = threadIdx.x; e < L * NP; e += 128) {
    const int tt = e / NP, i = e % NP, t = ch * L + tt;
    const bool ok = t < T_ && i < N;
    out[Prep<NP>::KEYS + e] = ok ? rt::to_f<T>(pdy[((long)(batch * T_ + t) * H + head) * N + i]) : 0.f;
  }
}

// ---------------------------------------------------------------- 2. state-gradient pass
template <int NP>
struct StateSmem {
  static constexpr int SP = NP + 4;
  static constexpr int KEYS = Prep<NP>::KEYS;
  static constexpr int STAGE = KEYS + L * R;  // key-side record + this CTA's dy columns [L][R]
  static constexpr int FLOATS = 2 * STAGE + R * SP + 3 * L * R;
};

template <int NP>
RT_DEVICE void state_issue(float* stage, const float* prep_rec, int row0) {
  using SS = StateSmem<NP>;
  for (int e = threadIdx.x; e < SS::KEYS / 4; e += 128) rt::cp_async16(stage + 4 * e, prep_rec + 4 * e, true);
  const float* dy = prep_rec + Prep<NP>::KEYS;
  for (int e = threadIdx.x; e < L * (R / 4); e += 128) {
    const int tt = e / (R / 4), i = (e % (R / 4)) * 4;
    rt::cp_async16(stage + SS::KEYS + tt * R + i, dy + tt * NP + row0 + i, true);
  }
  rt::cp_async_commit();
}

template <int NP>
__global__ void __launch_bounds__(128)
wkv7_bwd_state_kernel(int T_, int H, int N, const float* __restrict__ prep, const float* __restrict__ dend,
                      float* __restrict__ dstate, float* __restrict__ ds0) {
  using SS = StateSmem<NP>;
  constexpr int PREP = Prep<NP>::FLOATS;
  constexpr int SP = SS::SP;
  extern __shared__ __align__(16) float sm[];
  float* stage[2] = {sm, sm + SS::STAGE};
  float* dS = sm + 2 * SS::STAGE;       // [R][SP]
  float* dY = dS + R * SP;              // [L][R]
  float* dU = dY + L * R;               // [L][R]
  float* dZ = dU + L * R;               // [L][R]
  const int rb = blockIdx.x, bh = blockIdx.y, row0 = rb * R;
  const int chunks = (T_ + L - 1) / L;
  const long NN = (long)N * N;
  (void)H;
  state_issue<NP>(stage[(chunks - 1) & 1], prep + ((long)bh * chunks + chunks - 1) * PREP, row0);
  for (int e = threadIdx.x; e < R * NP; e += 128) {
    const int i = e / NP, j = e % NP, row = row0 + i;
    dS[i * SP + j] = (row < N && j < N && dend) ? dend[bh * NN + (long)row * N + j] : 0.f;
  }
  for (int ch = chunks - 1; ch >= 0; --ch) {
    // gradient w.r.t. this chunk's end state
    float* out = dstate + ((long)bh * chunks + ch) * NN;
    for (int e = threadIdx.x; e < R * NP; e += 128) {
      const int i = e / NP, j = e % NP, row = row0 + i;
      if (row < N && j < N) out[(long)row * N + j] = dS[i * SP + j];
    }
    if (ch > 0) {
      state_issue<NP>(stage[(ch - 1) & 1], prep + ((long)bh * chunks + ch - 1) * PREP, row0);
      rt::cp_async_wait<1>();
    } else {
      rt::cp_async_wait<0>();
    }
    __syncthreads();
    const float* Rt = stage[ch & 1];
    const float* At = Rt + L * NP;
    const float* Bh = At + L * NP;
    const float* DL = Bh + L * NP;
    const float* W = DL + NP;
    const float* Mrb = W + L * L;
    const float* dyr = stage[ch & 1] + SS::KEYS;
    for (int e = threadIdx.x; e < L * R; e += 128) dY[e] = dyr[e];
    __syncthreads();
    // dU[s][i] = sum_j Bh[s][j] dS[i][j] + sum_{t>=s} Mrb[t][s] dY[t][i]
    for (int e = threadIdx.x; e < L * R; e += 128) {
      const int s = e / R, i = e % R;
      float u = rowdot<NP>(Bh + s * NP, dS + i * SP);
      for (int t = s; t < L; ++t) u += Mrb[t * L + s] * dY[t * R + i];
      dU[e] = u;
    }
    __syncthreads();
    // dZ = W^T dU
    for (int e = threadIdx.x; e < L * R; e += 128) {
      const int s = e / R, i = e % R;
      float z = 0.f;
      for (int t = s; t < L; ++t) z += W[t * L + s] * dU[t * R + i];
      dZ[e] = z;
    }
    __syncthreads();
    // dS <- dS diag(D_L) + dY^T R~ + dZ^T A~
    for (int e = threadIdx.x; e < R * (NP / 4); e += 128) {  // four consecutive keys per thread
      const int i = e / (NP / 4), j = (e % (NP / 4)) * 4;
      float4 acc = *reinterpret_cast<const float4*>(dS + i * SP + j);
      const float4 d = *reinterpret_cast<const float4*>(DL + j);
      acc.x *= d.x; acc.y *= d.y; acc.z *= d.z; acc.w *= d.w;
#pragma unroll
      for (int t = 0; t < L; ++t) {
        const float y = dY[t * R + i], z = dZ[t * R + i];
        const float4 r4 = *reinterpret_cast<const float4*>(Rt + t * NP + j);
        const float4 a4 = *reinterpret_cast<const float4*>(At + t * NP + j);
        acc.x += y * r4.x + z * a4.x;
        acc.y += y * r4.y + z * a4.y;
        acc.z += y * r4.z + z * a4.z;
        acc.w += y * r4.w + z * a4.w;
      }
      *reinterpret_cast<float4*>(dS + i * SP + j) = acc;
    }
    __syncthreads();
  }
  for (int e = threadIdx.x; e < R * NP; e += 128) {
    const int i = e / NP, j = e % NP, row = row0 + i;
    if (row < N && j < N) ds0[bh * NN + (long)row * N + j] = dS[i * SP + j];
  }
}

// ---------------------------------------------------------------- 3. gradients
constexpr int GT = 512;  // threads of the gradient kernel

// Value rows are processed in passes of VR (= min(NP, 64)); sums over value rows accumulate in shared memory.
template <int NP>
struct GradSmem {
  using K = Keys<NP>;
  static constexpr int SP = K::SP;
  static constexpr int VR = NP < 64 ? NP : 64;
  static constexpr int VSP = VR + 4;
  static constexpr int KEYROWS = L * SP;  // [L][SP] arrays indexed by key j
  static constexpr int VROWS = L * VSP;   // [L][VSP] arrays indexed by value row i
  static constexpr int FLOATS = 6 * K::KEY + NP          // keys (r, a, b, k, lam, sig) + D_L
                                + 2 * VROWS              // V, DY
                                + 2 * VR * SP            // S0, DS row slices
                                + 3 * VROWS              // U (Z), DU, DZ
                                + 9 * K::MAT             // M (4), W, dM (4)
                                + 4 * KEYROWS + NP;      // RD, AD, BH, KH accumulators + direct dD_L
  // AT and DDL reuse the value-row region (V ..), which is dead once the value-row passes end; the
  // total stays under half an SM's shared memory so two CTAs (2 x 512 threads, <= 64 registers) fit.
  static_assert(2 * VROWS + 2 * VR * SP + 3 * VROWS >= 2 * KEYROWS, "AT/DDL alias");
};

template <typename T, int NP>
__global__ void __launch_bounds__(GT, NP <= 64 ? 2 : 1)
wkv7_bwd_grad_kernel(int T_, int H, int N, const T* __restrict__ pr, const T* __restrict__ pw,
                     const T* __restrict__ pk, const T* __restrict__ pv, const T* __restrict__ pa,
                     const T* __restrict__ pb, const T* __restrict__ pdy, const float* __restrict__ checkpoints,
                     const float* __restrict__ dstate, const float* __restrict__ prep, float* __restrict__ dr,
                     float* __restrict__ dw,
                     float* __restrict__ dk, float* __restrict__ dv, float* __restrict__ da,
                     float* __restrict__ db) {
  using K = Keys<NP>;
  using G = GradSmem<NP>;
  constexpr int SP = G::SP, VR = G::VR, VSP = G::VSP, MAT = K::MAT;
  extern __shared__ __align__(16) float sm[];
  K c;
  c.bind(sm);
  float* V = sm + 6 * K::KEY + NP;       // [L][VSP] v[t][i]
  float* DY = V + G::VROWS;              // [L][VSP] dy[t][i]
  float* S0 = DY + G::VROWS;             // [VR][SP] S0[i][j]
  float* DS = S0 + VR * SP;              // [VR][SP] dS[i][j] (chunk-end state gradient)
  float* U = DS + VR * SP;               // [L][VSP] Z then U
  float* DU = U + G::VROWS;              // [L][VSP]
  float* DZ = DU + G::VROWS;             // [L][VSP]
  float* M = DZ + G::VROWS;              // Mab, Mak, Mrb, Mrk
  float* W = M + 4 * MAT;
  float* dM = W + MAT;                   // 4 chunk-matrix gradients (sums over value rows)
  float* RD = dM + 4 * MAT;              // [L][SP] sum_i dy[t][i] S0[i][j]
  float* AD = RD + G::KEYROWS;           // [L][SP] sum_i dZ[t][i] S0[i][j]
  float* BH = AD + G::KEYROWS;           // [L][SP] sum_i U[t][i] dS[i][j]
  float* KH = BH + G::KEYROWS;           // [L][SP] sum_i v[t][i] dS[i][j]
  float* dDLd = KH + G::KEYROWS;         // [NP] sum_i S0[i][j] dS[i][j]
  float* AT = V;                         // [L][SP] a~-term of d Lambda (belongs to step t-1); after the passes
  float* DDL = V + G::KEYROWS;           // [L][SP] per-step b^/k^ part of dD_L; after the passes
  const int ch = blockIdx.x, bh = blockIdx.y, batch = bh / H, head = bh % H;
  const int chunks = gridDim.x;
  const int t0 = ch * L;
  const long NN = (long)N * N;
  const float* s0 = checkpoints + ((long)bh * (chunks + 1) + ch) * NN;
  const float* dse = dstate + ((long)bh * chunks + ch) * NN;
  load_keys<T, NP>(c, pr, pw, pk, pa, pb, T_, H, N, batch, head, t0, GT);
  // W = (I - Mab)^{-1} and Mrb come from the prep record; Mak and Mrk are formed here
  const float* rec = prep + ((long)bh * chunks + ch) * Prep<NP>::FLOATS + 3 * L * NP + NP;
  for (int e = threadIdx.x; e < 4 * L * L; e += GT) {
    const int which = e / (L * L), t = (e % (L * L)) / L, s = e % L;
    const bool keep = which < 2 ? s < t : s <= t;
    float m;
    if (which == 0) {
      m = 0.f;  // Mab itself is not needed once W is known
    } else if (which == 2) {
      m = rec[L * L + t * L + s];
    } else {
      const float* x = (which < 2 ? c.a : c.r) + t * SP;
      m = keep ? rowdot<NP>(x, c.k + s * SP) : 0.f;
    }
    M[which * MAT + t * (L + 1) + s] = m;
    dM[which * MAT + t * (L + 1) + s] = 0.f;
    if (which == 0) W[t * (L + 1) + s] = rec[t * L + s];
  }
  for (int e = threadIdx.x; e < L * SP; e += GT) RD[e] = AD[e] = BH[e] = KH[e] = 0.f;
  if (threadIdx.x < NP) dDLd[threadIdx.x] = 0.f;
  __syncthreads();
  const float* Mak = M + MAT;
  const float* Mrb = M + 2 * MAT;
  const float* Mrk = M + 3 * MAT;
  for (int i0 = 0; i0 < NP; i0 += VR) {
    // slices of this pass: value rows i0 .. i0+VR
    for (int e = threadIdx.x; e < L * VR; e += GT) {
      const int tt = e / VR, ii = e % VR, i = i0 + ii, t = t0 + tt;
      const bool ok = (t < T_) && (i < N);
      const long idx = ((long)(batch * T_ + t) * H + head) * N + i;
      V[tt * VSP + ii] = ok ? rt::to_f<T>(pv[idx]) : 0.f;
      DY[tt * VSP + ii] = ok ? rt::to_f<T>(pdy[idx]) : 0.f;
    }
    if (N == NP) {  // full rows: 16-byte loads
      for (int e = threadIdx.x; e < VR * (NP / 4); e += GT) {
        const int ii = e / (NP / 4), j = (e % (NP / 4)) * 4, i = i0 + ii;
        *reinterpret_cast<float4*>(S0 + ii * SP + j) = __ldg(reinterpret_cast<const float4*>(s0 + (long)i * N + j));
        *reinterpret_cast<float4*>(DS + ii * SP + j) = __ldg(reinterpret_cast<const float4*>(dse + (long)i * N + j));
      }
    } else {
      for (int e = threadIdx.x; e < VR * NP; e += GT) {
        const int ii = e / NP, j = e % NP, i = i0 + ii;
        const bool ok = i < N && j < N;
        S0[ii * SP + j] = ok ? s0[(long)i * N + j] : 0.f;
        DS[ii * SP + j] = ok ? dse[(long)i * N + j] : 0.f;
      }
    }
    __syncthreads();
    // Z (into DZ) and dU, row-local: the key products A~ S0^T and (b D_L) dS^T as 4 x 2 register tiles, then the
    // chunk-triangular terms per element
    {
      constexpr int IP = VR / 2, TILES = (L / 4) * IP;
      for (int e = threadIdx.x; e < 2 * TILES; e += GT) {
        const int which = e / TILES, r = e % TILES, tb = 4 * (r / IP), ia = r % IP, ib = ia + IP;
        float acc[4][2] = {};
        if (which == 0)
          tile42<NP, false>(c.a, tb, S0, ia, ib, nullptr, SP, acc);
        else
          tile42<NP, true>(c.b, tb, DS, ia, ib, c.dl, SP, acc);
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          const int t = tb + rr;
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int ii = k ? ib : ia;
            float v = acc[rr][k];
            if (which == 0) {
              for (int s2 = 0; s2 < t; ++s2) v += Mak[t * (L + 1) + s2] * V[s2 * VSP + ii];
              DZ[t * VSP + ii] = v;
            } else {
              for (int t2 = t; t2 < L; ++t2) v += Mrb[t2 * (L + 1) + t] * DY[t2 * VSP + ii];
              DU[t * VSP + ii] = v;
            }
          }
        }
      }
    }
    __syncthreads();
    // U = W Z
    for (int e = threadIdx.x; e < L * VR; e += GT) {
      const int t = e / VR, ii = e % VR;
      float u = 0.f;
      for (int s2 = 0; s2 <= t; ++s2) u += W[t * (L + 1) + s2] * DZ[s2 * VSP + ii];
      U[t * VSP + ii] = u;
    }
    __syncthreads();
    // dZ = W^T dU
    for (int e = threadIdx.x; e < L * VR; e += GT) {
      const int s2 = e / VR, ii = e % VR;
      float z = 0.f;
      for (int t = s2; t < L; ++t) z += W[t * (L + 1) + s2] * DU[t * VSP + ii];
      DZ[s2 * VSP + ii] = z;
    }
    __syncthreads();
    // dv (row-local, final): (k D_L) dS^T as 4 x 2 register tiles, then the chunk-triangular terms
    {
      constexpr int IP = VR / 2, TILES = (L / 4) * IP;
      for (int e = threadIdx.x; e < TILES; e += GT) {
        const int sb = 4 * (e / IP), ia = e % IP, ib = ia + IP;
        float acc[4][2] = {};
        tile42<NP, true>(c.k, sb, DS, ia, ib, c.dl, SP, acc);
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          const int s2 = sb + rr, tg = t0 + s2;
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int ii = k ? ib : ia, i = i0 + ii;
            float g = acc[rr][k];
            for (int t = s2; t < L; ++t) g += Mrk[t * (L + 1) + s2] * DY[t * VSP + ii];
            for (int t = s2 + 1; t < L; ++t) g += Mak[t * (L + 1) + s2] * DZ[t * VSP + ii];
            if (tg < T_ && i < N) dv[((long)(batch * T_ + tg) * H + head) * N + i] = g;
          }
        }
      }
    }
    // sums over this pass's value rows
    for (int e = threadIdx.x; e < 4 * L * L; e += GT) {
      const int which = e / (L * L), t = (e % (L * L)) / L, s2 = e % L;
      const bool keep = which < 2 ? s2 < t : s2 <= t;
      if (!keep) continue;
      const float4* x = reinterpret_cast<const float4*>((which < 2 ? DZ : DY) + t * VSP);
      const float4* y = reinterpret_cast<const float4*>(((which & 1) ? V : U) + s2 * VSP);
      float acc = 0.f;
#pragma unroll 4
      for (int q = 0; q < VR / 4; ++q) {
        const float4 m = x[q], n = y[q];
        acc += m.x * n.x + m.y * n.y + m.z * n.z + m.w * n.w;
      }
      dM[which * MAT + t * (L + 1) + s2] += acc;
    }
    {  // key-side sums over this pass's rows: thread = (4 steps, key j, part of the rows); 4 x 4 register block
      constexpr int TQ = L / 4;
      constexpr int PARTS0 = GT / (TQ * NP) > 0 ? GT / (TQ * NP) : 1;
      constexpr int PARTS = PARTS0 < VR / 4 ? PARTS0 : VR / 4;  // at least 4 rows (one float4) per part
      constexpr int ROWS = VR / PARTS;
      for (int e = threadIdx.x; e < TQ * NP * PARTS; e += GT) {
        const int part = e / (TQ * NP), tq = (e / NP) % TQ, j = e % NP, tb = 4 * tq;
        float rd[4] = {}, ad[4] = {}, bh[4] = {}, kh[4] = {};
        for (int i4 = part * ROWS; i4 < (part + 1) * ROWS; i4 += 4) {
          float s0v[4], dsv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            s0v[u] = S0[(i4 + u) * SP + j];
            dsv[u] = DS[(i4 + u) * SP + j];
          }
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int o = (tb + r) * VSP + i4;
            const float4 dy4 = *reinterpret_cast<const float4*>(DY + o);
            const float4 dz4 = *reinterpret_cast<const float4*>(DZ + o);
            const float4 u4 = *reinterpret_cast<const float4*>(U + o);
            const float4 v4 = *reinterpret_cast<const float4*>(V + o);
            rd[r] += dy4.x * s0v[0] + dy4.y * s0v[1] + dy4.z * s0v[2] + dy4.w * s0v[3];
            ad[r] += dz4.x * s0v[0] + dz4.y * s0v[1] + dz4.z * s0v[2] + dz4.w * s0v[3];
            bh[r] += u4.x * dsv[0] + u4.y * dsv[1] + u4.z * dsv[2] + u4.w * dsv[3];
            kh[r] += v4.x * dsv[0] + v4.y * dsv[1] + v4.z * dsv[2] + v4.w * dsv[3];
          }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int o = (tb + r) * SP + j;
          if (PARTS == 1) {
            RD[o] += rd[r]; AD[o] += ad[r]; BH[o] += bh[r]; KH[o] += kh[r];
          } else {
            atomicAdd(RD + o, rd[r]); atomicAdd(AD + o, ad[r]); atomicAdd(BH + o, bh[r]); atomicAdd(KH + o, kh[r]);
          }
        }
      }
    }
    if (threadIdx.x < NP) {
      const int j = threadIdx.x;
      float acc = 0.f;
      for (int ii = 0; ii < VR; ++ii) acc += S0[ii * SP + j] * DS[ii * SP + j];
      dDLd[j] += acc;
    }
    __syncthreads();
  }
  // chain through the chunk matrices for every (t, j); raw-input gradients
  for (int e = threadIdx.x; e < L * NP; e += GT) {
    const int t = e / NP, j = e % NP, o = t * SP + j;
    const float bhat = BH[o], khat = KH[o];
    float dat = AD[o], drt = RD[o], dbt = bhat * c.dl[j], dkt = khat * c.dl[j];
#pragma unroll
    for (int s2 = 0; s2 < L; ++s2) {
      const int ts = t * (L + 1) + s2, st = s2 * (L + 1) + t;
      dat += dM[ts] * c.b[s2 * SP + j] + dM[MAT + ts] * c.k[s2 * SP + j];
      drt += dM[2 * MAT + ts] * c.b[s2 * SP + j] + dM[3 * MAT + ts] * c.k[s2 * SP + j];
      dbt += dM[st] * c.a[s2 * SP + j] + dM[2 * MAT + st] * c.r[s2 * SP + j];
      dkt += dM[MAT + st] * c.a[s2 * SP + j] + dM[3 * MAT + st] * c.r[s2 * SP + j];
    }
    const float lam_t = c.lam[o], lam_p = t ? c.lam[o - SP] : 0.f;
    const float e_t = expf(lam_t), e_p = expf(lam_p), inv_t = 1.f / e_t;
    const int tg = t0 + t;
    if (tg < T_ && j < N) {
      const long idx = ((long)(batch * T_ + tg) * H + head) * N + j;
      dr[idx] = drt * e_t;
      da[idx] = dat * e_p;
      db[idx] = dbt * inv_t;
      dk[idx] = dkt * inv_t;
    }
    RD[o] = drt * c.r[o] - dbt * c.b[o] - dkt * c.k[o];  // d Lambda_t contributions at step t
    AT[o] = dat * c.a[o];
    DDL[o] = bhat * c.b[o] + khat * c.k[o];
  }
  __syncthreads();
  if (threadIdx.x < NP) {
    const int j = threadIdx.x;
    float ddl_sum = dDLd[j];
#pragma unroll
    for (int s2 = 0; s2 < L; ++s2) ddl_sum += DDL[s2 * SP + j];
    float run = 0.f;
    for (int t = L - 1; t >= 0; --t) {
      float g = RD[t * SP + j];
      if (t + 1 < L) g += AT[(t + 1) * SP + j];
      if (t == L - 1) g += ddl_sum * c.dl[j];
      run += g;
      const int tg = t0 + t;
      if (tg < T_ && j < N) {
        const float sg = c.sig[t * SP + j];
        dw[((long)(batch * T_ + tg) * H + head) * N + j] = run * (-DECAY_SCALE) * sg * (1.f - sg);
      }
    }
  }
}

bool aligned16(std::initializer_list<const void*> ptrs) {
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) & 15) return false;
  return true;
}

template <typename T, int NP>
cudaError_t launch(int B, int T_, int H, int N, const void* r, const void* w, const void* k, const void* v,
                   const void* a, const void* b, const float* ckpt, const void* dy, const float* dend, float* dr,
                   float* dw, float* dk, float* dv, float* da, float* db, float* ds0, float* work,
                   cudaStream_t stream) {
  const int chunks = (T_ + L - 1) / L;
  float* prep = work;
  float* dstate = work + (long)B * H * chunks * Prep<NP>::FLOATS;
  const size_t p_bytes = prep_smem_floats<NP>() * sizeof(float);
  RT_CUDA_CHECK(cudaFuncSetAttribute(wkv7_bwd_prep_kernel<T, NP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)p_bytes));
  wkv7_bwd_prep_kernel<T, NP><<<dim3(chunks, B * H), 128, p_bytes, stream>>>(
      T_, H, N, (const T*)r, (const T*)w, (const T*)k, (const T*)a, (const T*)b, (const T*)dy, prep);
  RT_CUDA_CHECK(cudaGetLastError());
  const size_t s_bytes = StateSmem<NP>::FLOATS * sizeof(float);
  RT_CUDA_CHECK(cudaFuncSetAttribute(wkv7_bwd_state_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)s_bytes));
  wkv7_bwd_state_kernel<NP><<<dim3(NP / R, B * H), 128, s_bytes, stream>>>(T_, H, N, prep, dend, dstate, ds0);
  RT_CUDA_CHECK(cudaGetLastError());
  const size_t g_bytes = GradSmem<NP>::FLOATS * sizeof(float);
  RT_CUDA_CHECK(cudaFuncSetAttribute(wkv7_bwd_grad_kernel<T, NP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)g_bytes));
  wkv7_bwd_grad_kernel<T, NP><<<dim3(chunks, B * H), GT, g_bytes, stream>>>(
      T_, H, N, (const T*)r, (const T*)w, (const T*)k, (const T*)v, (const T*)a, (const T*)b, (const T*)dy, ckpt,
      dstate, prep, dr, dw, dk, dv, da, db);
  return cudaGetLastError();
}

int pick_np(int N) { return N <= 16 ? 16 : N <= 32 ? 32 : N <= 64 ? 64 : 128; }

}  // namespace

// Floats of scratch needed by rt_wkv7_backward: chunk prep records plus per-chunk state gradients.
extern "C" long rt_wkv7_backward_workspace_floats(int B, int T_, int H, int N) {
  const long chunks = (T_ + L - 1) / L;
  const int np = pick_np(N);
  return (long)B * H * chunks * (4L * L * np + np + 2L * L * L) + (long)B * H * chunks * N * N;
}

extern "C" cudaError_t rt_wkv7_backward(int dtype, int B, int T_, int H, int N, const void* r, const void* w,
                                        const void* k, const void* v, const void* a, const void* b,
                                        const float* checkpoints, const void* dy, const float* dend, float* dr,
                                        float* dw, float* dk, float* dv, float* da, float* db, float* ds0,
                                        float* work, cudaStream_t stream) {
  const int np = pick_np(N);
  if (!aligned16({work})) return cudaErrorInvalidValue;
#define RT_B(TYPE, NPV) \
  return launch<TYPE, NPV>(B, T_, H, N, r, w, k, v, a, b, checkpoints, dy, dend, dr, dw, dk, dv, da, db, ds0, work, stream)
#define RT_NP(TYPE)                 \
  switch (np) {                     \
    case 16: RT_B(TYPE, 16);        \
    case 32: RT_B(TYPE, 32);        \
    case 64: RT_B(TYPE, 64);        \
    default: RT_B(TYPE, 128);       \
  }
  if (dtype == 1) { RT_NP(__nv_bfloat16) } else { RT_NP(float) }
#undef RT_NP
#undef RT_B
}
