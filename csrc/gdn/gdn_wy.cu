// Gated DeltaNet forward for long prefills, sm_100a: WY form with 64-token chunks.
//
// Recurrence (per value head, state S[key j][value i], chunk-local cumulative log-decay Lambda_t with
// Lambda_{-1} = 0, normalised q (scaled by D^-1/2) and k):
//   S_t = e^{g_t} S_{t-1} + k_t Vt_t^T,   Vt_t = beta_t (v_t - e^{g_t} S_{t-1}^T k_t),   o_t = S_t^T q_t.
// Unrolling S_{t-1} inside a chunk from its start state S0 gives, with A[t][s] = beta_t e^{Lambda_t -
// Lambda_s} (k_t . k_s) for s < t and T = (I + A)^{-1} (unit lower triangular):
//   Vt  = U0 + W S0,            U0 = T (beta o v),   W = -T diag(beta_t e^{Lambda_t}) K        (state-free)
//   S_L = e^{Lambda_{L-1}} S0 + sum_s e^{Lambda_{L-1} - Lambda_s} k_s Vt_s^T
//   o_t = e^{Lambda_t} S0^T q_t + sum_{s<=t} e^{Lambda_t - Lambda_s} (q_t . k_s) Vt_s
// Every exponent is <= 0, so large negative gates are safe. Three kernels:
//   1 (parallel over chunks and heads)  T by blocked 16x16 inversion, U0 and W;
//   2 (serial over chunks, parallel over heads and 32-column value blocks)  Vt = U0 + W S0, the chunk-start
//     state is stored, S advanced -- the only sequential work is two 64x128x32 products per chunk;
//   3 (parallel)  outputs from the stored chunk-start states and Vt.
// Padded steps past T get beta = 0 and g = 0, so they add nothing.
// Reference semantics: HF Qwen3_5GatedDeltaNet chunk rule (torch_chunk_gated_delta_rule), as invoked from the
// reference's teacher adapter (theseus/hf_model.py:38-52).
#include <cstdlib>

#include "../common/common.cuh"
#include "../common/sm100.cuh"
#include "../common/tmap.cuh"
#include "../wkv7/wkv7_tc.cuh"  // tile layouts, triangular solve, tf32 MMA issue

namespace rt_gdn_wy {

using bf16 = __nv_bfloat16;
constexpr int LC = 64;       // chunk length
constexpr int NT = 256;      // threads per CTA
constexpr int VB = 32;       // value columns per CTA in the serial kernel
constexpr int OB = 64;       // value columns per CTA in the output kernel

template <int D>
struct Dims {
  static constexpr int SP = D + 4;   // padded fp32 row (16-byte aligned, conflict-free float4 columns)
};

RT_DEVICE float gate_g(float a, float dtb, float neg_a) {
  const float av = a + dtb;
  return neg_a * (av > 20.f ? av : log1pf(expf(av)));
}

// Inclusive scan of x over 64 threads (threads 0..63 hold the values; returns the scan for those threads).
RT_DEVICE float scan64(float x, float* tmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (warp == 0 && lane == 31) tmp[0] = x;
  __syncthreads();
  if (warp == 1) x += tmp[0];
  return x;
}

// ---------------------------------------------------------------- 1: T, U0, W per (chunk, value head)
// grid (chunks, Hv, B). qn/kn: [B, T, Hk, D] fp32 normalised. Writes W, U0: [B, Hv, Tp, D] fp32 and
// lam: [B, Hv, Tp] (chunk-local cumulative log decay).
template <int D>
struct WySmem {
  static constexpr int SP = Dims<D>::SP;
  static constexpr int FLOATS = 2 * LC * SP + 2 * LC * (LC + 1) + 3 * 16 * 17 + 4 * LC + 32;
};

template <int D>
__global__ void __launch_bounds__(NT)
gdn_wy_kernel(const float* __restrict__ kn, const bf16* __restrict__ qkv, long row_stride, const bf16* __restrict__ pa,
              const bf16* __restrict__ pb, long ab_stride, const float* __restrict__ A_log,
              const float* __restrict__ dt_bias, float* __restrict__ Wout, float* __restrict__ Uout,
              float* __restrict__ lam_out, int T, int Tp, int Hk, int Hv) {
  constexpr int SP = Dims<D>::SP;
  constexpr int MP = LC + 1;
  extern __shared__ __align__(16) float sm[];
  float* K = sm;                 // [LC][SP]  k, later diag(beta e^Lambda) k
  float* V = K + LC * SP;        // [LC][SP]  beta v
  float* A = V + LC * SP;        // [LC][MP]
  float* Ti = A + LC * MP;       // [LC][MP]  (I + A)^{-1}
  float* P = Ti + LC * MP;       // [3][16][17]  scratch blocks of the blocked inversion
  float* lam = P + 3 * 16 * 17;  // [LC]
  float* beta = lam + LC;        // [LC]
  float* elam = beta + LC;       // [LC]  e^{Lambda_t}
  float* tmp = elam + LC;
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (Hv / Hk);
  const int t0 = c * LC;
  const long vcol = 2L * Hk * D + (long)h * D;
  // k rows (fp32, cp.async) and v rows (bf16 -> fp32)
  for (int e = threadIdx.x; e < LC * (D / 4); e += NT) {
    const int tt = e / (D / 4), j = (e % (D / 4)) * 4, t = t0 + tt;
    const bool ok = t < T;
    rt::cp_async16(K + tt * SP + j, kn + (ok ? (((long)b * T + t) * Hk + kh) * D + j : 0), ok);
  }
  rt::cp_async_commit();
  float g = 0.f, bt = 0.f;
  if (threadIdx.x < LC) {
    const int t = t0 + threadIdx.x;
    if (t < T) {
      g = gate_g(rt::to_f(pa[((long)b * T + t) * ab_stride + h]), dt_bias[h], -expf(A_log[h]));
      bt = __bfloat162float(__float2bfloat16_rn(rt::sigmoidf_(rt::to_f(pb[((long)b * T + t) * ab_stride + h]))));
    }
  }
  const float lt = scan64(threadIdx.x < LC ? g : 0.f, tmp);
  if (threadIdx.x < LC) {
    lam[threadIdx.x] = lt;
    beta[threadIdx.x] = bt;
    elam[threadIdx.x] = expf(lt);
    lam_out[((long)b * Hv + h) * Tp + t0 + threadIdx.x] = lt;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < LC * (D / 8); e += NT) {
    const int tt = e / (D / 8), i = (e % (D / 8)) * 8, t = t0 + tt;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (t < T) {
      const uint4 raw = *reinterpret_cast<const uint4*>(qkv + ((long)b * T + t) * row_stride + vcol + i);
      const bf16* hv = reinterpret_cast<const bf16*>(&raw);
      const float bv = beta[tt];
#pragma unroll
      for (int u = 0; u < 8; ++u) f[u] = __bfloat162float(hv[u]) * bv;
    }
    *reinterpret_cast<float4*>(V + tt * SP + i) = make_float4(f[0], f[1], f[2], f[3]);
    *reinterpret_cast<float4*>(V + tt * SP + i + 4) = make_float4(f[4], f[5], f[6], f[7]);
  }
  rt::cp_async_wait<0>();
  __syncthreads();
  // A[t][s] = beta_t e^{Lambda_t - Lambda_s} (k_t . k_s), s < t. Thread: rows t = 4*ty..+3, cols s = tx + 16*u.
  {
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    float acc[4][4] = {};
    for (int j = 0; j < D; j += 4) {
      float4 kt[4], ks[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) kt[r] = *reinterpret_cast<const float4*>(K + (4 * ty + r) * SP + j);
#pragma unroll
      for (int u = 0; u < 4; ++u) ks[u] = *reinterpret_cast<const float4*>(K + (tx + 16 * u) * SP + j);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int u = 0; u < 4; ++u)
          acc[r][u] += kt[r].x * ks[u].x + kt[r].y * ks[u].y + kt[r].z * ks[u].z + kt[r].w * ks[u].w;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = 4 * ty + r, s = tx + 16 * u;
        A[t * MP + s] = s < t ? beta[t] * expf(lam[t] - lam[s]) * acc[r][u] : 0.f;
      }
  }
  __syncthreads();
  // Blocked inverse of the unit lower-triangular (I + A), 16x16 blocks. Diagonal blocks by forward substitution
  // (one thread per column of each block); then block diagonals d = 1..3: T_ij = -T_ii sum_{k=j}^{i-1} A_ik T_kj.
  if (threadIdx.x < LC) {
    const int blk = threadIdx.x >> 4, col = threadIdx.x & 15, o = 16 * blk, s = o + col;
    for (int t = o; t < o + 16; ++t) {
      float v = t == s ? 1.f : 0.f;
      if (t > s)
        for (int r = s; r < t; ++r) v -= A[t * MP + r] * Ti[r * MP + s];
      Ti[t * MP + s] = v;
    }
  }
  // zero the strictly upper blocks
  for (int e = threadIdx.x; e < LC * LC; e += NT) {
    const int t = e / LC, s = e % LC;
    if ((t >> 4) < (s >> 4)) Ti[t * MP + s] = 0.f;
  }
  __syncthreads();
  for (int d = 1; d < 4; ++d) {
    // P_ij = sum_{k=j}^{i-1} A_ik T_kj for the 4-d blocks (i, j = i-d)
    for (int e = threadIdx.x; e < (4 - d) * 256; e += NT) {
      const int bi = e / 256 + d, bj = bi - d, r = (e % 256) / 16, cc = e % 16;
      const int t = 16 * bi + r, s = 16 * bj + cc;
      float v = 0.f;
      for (int k = 16 * bj; k < 16 * bi; ++k) v += A[t * MP + k] * Ti[k * MP + s];
      P[(bi - d) * 272 + r * 17 + cc] = v;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < (4 - d) * 256; e += NT) {
      const int bi = e / 256 + d, bj = bi - d, r = (e % 256) / 16, cc = e % 16;
      const int t = 16 * bi + r, s = 16 * bj + cc;
      float v = 0.f;
      for (int k = 16 * bi; k <= t; ++k) v -= Ti[t * MP + k] * P[(bi - d) * 272 + (k - 16 * bi) * 17 + cc];
      Ti[t * MP + s] = v;
    }
    __syncthreads();
  }
  // K <- diag(beta e^Lambda) K
  for (int e = threadIdx.x; e < LC * (D / 4); e += NT) {
    const int tt = e / (D / 4), j = (e % (D / 4)) * 4;
    const float f = beta[tt] * elam[tt];
    float4 k4 = *reinterpret_cast<float4*>(K + tt * SP + j);
    k4.x *= f; k4.y *= f; k4.z *= f; k4.w *= f;
    *reinterpret_cast<float4*>(K + tt * SP + j) = k4;
  }
  __syncthreads();
  // W = -T K', U0 = T V'. Thread: rows t = 4*ty..+3 (ty < 16), columns j = 4*tx.. (tx < 16), D / 64 passes.
  {
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    const long rowbase = ((long)b * Hv + h) * Tp + t0;
    for (int jb = 0; jb < D; jb += 64) {
      const int j = jb + 4 * tx;
      float4 w[4], u[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) w[r] = u[r] = make_float4(0.f, 0.f, 0.f, 0.f);
      const int tmax = 4 * ty + 3;
      for (int s = 0; s <= tmax; ++s) {
        const float4 k4 = *reinterpret_cast<const float4*>(K + s * SP + j);
        const float4 v4 = *reinterpret_cast<const float4*>(V + s * SP + j);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const float tv = Ti[(4 * ty + r) * MP + s];
          w[r].x += tv * k4.x; w[r].y += tv * k4.y; w[r].z += tv * k4.z; w[r].w += tv * k4.w;
          u[r].x += tv * v4.x; u[r].y += tv * v4.y; u[r].z += tv * v4.z; u[r].w += tv * v4.w;
        }
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const long row = rowbase + 4 * ty + r;
        w[r].x = -w[r].x; w[r].y = -w[r].y; w[r].z = -w[r].z; w[r].w = -w[r].w;
        *reinterpret_cast<float4*>(Wout + row * D + j) = w[r];
        *reinterpret_cast<float4*>(Uout + row * D + j) = u[r];
      }
    }
  }
}

// ---------------------------------------------------------------- 2: serial state pass
// grid (D / VB, Hv, B). Per chunk: Vt = U0 + W S (stored over U0), chunk-start S stored to S0 [B,Hv,C,D(i),D(j)],
// S <- e^{Lambda_{L-1}} S + sum_s e^{Lambda_{L-1} - Lambda_s} k_s Vt_s^T. The state block is value-major
// (S[i][j]) so products over keys use float4 rows.
template <int D>
struct StSmem {
  static constexpr int SP = Dims<D>::SP;
  static constexpr int FLOATS = VB * SP + 2 * LC * SP + 2 * LC * VB + 2 * LC;
};

template <int D>
__global__ void __launch_bounds__(NT)
gdn_state_kernel(const float* __restrict__ kn, const float* __restrict__ W, float* __restrict__ U,
                 const float* __restrict__ lam_in, float* __restrict__ state, float* __restrict__ S0out, int T, int Tp,
                 int Hk, int Hv) {
  constexpr int SP = Dims<D>::SP;
  extern __shared__ __align__(16) float sm[];
  float* S = sm;                  // [VB][SP]
  float* Ws = S + VB * SP;        // [LC][SP]
  float* Ks = Ws + LC * SP;       // [LC][SP]
  float* Us = Ks + LC * SP;       // [LC][VB]  U0 block, then Vt
  float* Vh = Us + LC * VB;       // [LC][VB]  e^{Lambda_L - Lambda_s} Vt
  float* lam = Vh + LC * VB;      // [LC]
  float* fac = lam + LC;          // [LC]
  const int vb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (Hv / Hk);
  const int col0 = vb * VB;
  const int chunks = Tp / LC;
  float* st = state + ((long)b * Hv + h) * D * D;  // [j][i]
  const long rowbase = ((long)b * Hv + h) * Tp;
  // Two cp.async groups per chunk: {W, U0 block, lam} (needed first) and {K} (needed by the state update), so
  // K of chunk c+1 streams in during the Vt product of chunk c+1 and W of chunk c+1 during the update of chunk c.
  auto load_w = [&](int c) {
    for (int e = threadIdx.x; e < LC * (D / 4); e += NT) {
      const int tt = e / (D / 4), j = (e % (D / 4)) * 4;
      rt::cp_async16(Ws + tt * SP + j, W + (rowbase + c * LC + tt) * D + j, true);
    }
    for (int e = threadIdx.x; e < LC * (VB / 4); e += NT) {
      const int tt = e / (VB / 4), i = (e % (VB / 4)) * 4;
      rt::cp_async16(Us + tt * VB + i, U + (rowbase + c * LC + tt) * D + col0 + i, true);
    }
    if (threadIdx.x < LC / 4) rt::cp_async16(lam + 4 * threadIdx.x, lam_in + rowbase + c * LC + 4 * threadIdx.x, true);
    rt::cp_async_commit();
  };
  auto load_k = [&](int c) {
    for (int e = threadIdx.x; e < LC * (D / 4); e += NT) {
      const int tt = e / (D / 4), j = (e % (D / 4)) * 4, t = c * LC + tt;
      const bool ok = t < T;
      rt::cp_async16(Ks + tt * SP + j, kn + (ok ? (((long)b * T + t) * Hk + kh) * D + j : 0), ok);
    }
    rt::cp_async_commit();
  };
  load_w(0);
  load_k(0);
  for (int e = threadIdx.x; e < D * VB; e += NT) {
    const int j = e / VB, i = e % VB;
    S[i * SP + j] = st[(long)j * D + col0 + i];
  }
  for (int c = 0; c < chunks; ++c) {
    rt::cp_async_wait<1>();  // W, U0, lam of chunk c (K of chunk c may still be in flight)
    __syncthreads();
    // chunk-start state to S0 (value-major rows)
    float* s0 = S0out + (((long)b * Hv + h) * chunks + c) * D * D;
    for (int e = threadIdx.x; e < VB * (D / 4); e += NT) {
      const int i = e / (D / 4), j = (e % (D / 4)) * 4;
      *reinterpret_cast<float4*>(s0 + (long)(col0 + i) * D + j) = *reinterpret_cast<const float4*>(S + i * SP + j);
    }
    if (threadIdx.x < LC) fac[threadIdx.x] = expf(lam[LC - 1] - lam[threadIdx.x]);
    const float eL = expf(lam[LC - 1]);  // read before lam is refilled for the next chunk
    // Vt = U0 + W S: thread rows t = 4*ty..+3 (ty < 16), columns i = tx, tx + 16 (tx < 16)
    {
      const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
      float acc[4][2] = {};
      const float4* s_a = reinterpret_cast<const float4*>(S + tx * SP);
      const float4* s_b = reinterpret_cast<const float4*>(S + (tx + 16) * SP);
#pragma unroll 4
      for (int q = 0; q < D / 4; ++q) {
        const float4 a4 = s_a[q], b4 = s_b[q];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const float4 w4 = reinterpret_cast<const float4*>(Ws + (4 * ty + r) * SP)[q];
          acc[r][0] += w4.x * a4.x + w4.y * a4.y + w4.z * a4.z + w4.w * a4.w;
          acc[r][1] += w4.x * b4.x + w4.y * b4.y + w4.z * b4.z + w4.w * b4.w;
        }
      }
      __syncthreads();  // fac visible; every thread done reading Ws
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int t = 4 * ty + r;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int i = tx + 16 * k;
          const float v = Us[t * VB + i] + acc[r][k];
          Us[t * VB + i] = v;
          Vh[t * VB + i] = v * fac[t];
          U[(rowbase + c * LC + t) * D + col0 + i] = v;
        }
      }
    }
    if (c + 1 < chunks) {
      load_w(c + 1);
      rt::cp_async_wait<1>();  // K of chunk c
    } else {
      rt::cp_async_wait<0>();
    }
    __syncthreads();
    // S[i][j] = e^{Lambda_L} S[i][j] + sum_t Vh[t][i] K[t][j]; thread: IPT rows i = IPT*iy.., 4 columns j = 4*jx
    {
      constexpr int JT = D / 4, IT = NT / JT, IPT = VB / IT;
      const int iy = threadIdx.x / JT, jx = threadIdx.x % JT, j = 4 * jx;
      float4 acc[IPT];
#pragma unroll
      for (int r = 0; r < IPT; ++r) {
        acc[r] = *reinterpret_cast<const float4*>(S + (IPT * iy + r) * SP + j);
        acc[r].x *= eL; acc[r].y *= eL; acc[r].z *= eL; acc[r].w *= eL;
      }
#pragma unroll 4
      for (int t = 0; t < LC; ++t) {
        const float4 k4 = *reinterpret_cast<const float4*>(Ks + t * SP + j);
#pragma unroll
        for (int r = 0; r < IPT; ++r) {
          const float vv = Vh[t * VB + IPT * iy + r];
          acc[r].x += vv * k4.x; acc[r].y += vv * k4.y; acc[r].z += vv * k4.z; acc[r].w += vv * k4.w;
        }
      }
      __syncthreads();  // all reads of S and Ks done
#pragma unroll
      for (int r = 0; r < IPT; ++r) *reinterpret_cast<float4*>(S + (IPT * iy + r) * SP + j) = acc[r];
    }
    if (c + 1 < chunks) load_k(c + 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < D * VB; e += NT) {
    const int j = e / VB, i = e % VB;
    st[(long)j * D + col0 + i] = S[i * SP + j];
  }
}

// ---------------------------------------------------------------- 3: outputs
// grid (chunks, Hv, B * D / OB). o_t[i] = e^{Lambda_t} sum_j q_t[j] S0[i][j] + sum_{s<=t} M[t][s] Vt_s[i],
// M[t][s] = e^{Lambda_t - Lambda_s} (q_t . k_s).
template <int D>
struct OutSmem {
  static constexpr int SP = Dims<D>::SP;
  static constexpr int OP = OB + 4;
  static constexpr int FLOATS = 2 * LC * SP + LC * OP + LC * (LC + 1) + LC;
};

template <int D>
__global__ void __launch_bounds__(NT)
gdn_out_kernel(const float* __restrict__ qn, const float* __restrict__ kn, const float* __restrict__ U,
               const float* __restrict__ lam_in, const float* __restrict__ S0, bf16* __restrict__ out, int T, int Tp,
               int Hk, int Hv) {
  constexpr int SP = Dims<D>::SP;
  constexpr int OP = OutSmem<D>::OP;
  constexpr int MP = LC + 1;
  extern __shared__ __align__(16) float sm[];
  float* Q = sm;                 // [LC][SP]
  float* KS = Q + LC * SP;       // [LC][SP]  k rows, then the S0 value block (OB rows of D)
  float* Vt = KS + LC * SP;      // [LC][OP]
  float* M = Vt + LC * OP;       // [LC][MP]
  float* lam = M + LC * MP;      // [LC]
  const int c = blockIdx.x, h = blockIdx.y;
  const int b = blockIdx.z / (D / OB), ob = blockIdx.z % (D / OB);
  const int kh = h / (Hv / Hk);
  const int chunks = Tp / LC;
  const int col0 = ob * OB;
  const long rowbase = ((long)b * Hv + h) * Tp + c * LC;
  for (int e = threadIdx.x; e < LC * (D / 4); e += NT) {
    const int tt = e / (D / 4), j = (e % (D / 4)) * 4, t = c * LC + tt;
    const bool ok = t < T;
    const long src = ok ? (((long)b * T + t) * Hk + kh) * D + j : 0;
    rt::cp_async16(Q + tt * SP + j, qn + src, ok);
    rt::cp_async16(KS + tt * SP + j, kn + src, ok);
  }
  for (int e = threadIdx.x; e < LC * (OB / 4); e += NT) {
    const int tt = e / (OB / 4), i = (e % (OB / 4)) * 4;
    rt::cp_async16(Vt + tt * OP + i, U + (rowbase + tt) * D + col0 + i, true);
  }
  if (threadIdx.x < LC / 4) rt::cp_async16(lam + 4 * threadIdx.x, lam_in + rowbase + 4 * threadIdx.x, true);
  rt::cp_async_commit();
  rt::cp_async_wait<0>();
  __syncthreads();
  {  // M, rows t = 4*ty..+3, cols s = tx + 16u
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    float acc[4][4] = {};
    for (int j = 0; j < D; j += 4) {
      float4 qt[4], ks[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) qt[r] = *reinterpret_cast<const float4*>(Q + (4 * ty + r) * SP + j);
#pragma unroll
      for (int u = 0; u < 4; ++u) ks[u] = *reinterpret_cast<const float4*>(KS + (tx + 16 * u) * SP + j);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int u = 0; u < 4; ++u)
          acc[r][u] += qt[r].x * ks[u].x + qt[r].y * ks[u].y + qt[r].z * ks[u].z + qt[r].w * ks[u].w;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = 4 * ty + r, s = tx + 16 * u;
        M[t * MP + s] = s <= t ? expf(lam[t] - lam[s]) * acc[r][u] : 0.f;
      }
  }
  __syncthreads();
  {  // S0 value block -> KS rows (value-major)
    const float* s0 = S0 + (((long)b * Hv + h) * chunks + c) * D * D + (long)col0 * D;
    for (int e = threadIdx.x; e < OB * (D / 4); e += NT) {
      const int i = e / (D / 4), j = (e % (D / 4)) * 4;
      rt::cp_async16(KS + i * SP + j, s0 + (long)i * D + j, true);
    }
    rt::cp_async_commit();
    rt::cp_async_wait<0>();
  }
  __syncthreads();
  {  // thread: rows t = 4*ty..+3 (ty < 16), columns i = tx + 16u (tx < 16, u < 4)
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    float acc[4][4] = {};
    for (int j = 0; j < D; j += 4) {
      float4 qt[4], sv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) qt[r] = *reinterpret_cast<const float4*>(Q + (4 * ty + r) * SP + j);
#pragma unroll
      for (int u = 0; u < 4; ++u) sv[u] = *reinterpret_cast<const float4*>(KS + (tx + 16 * u) * SP + j);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int u = 0; u < 4; ++u)
          acc[r][u] += qt[r].x * sv[u].x + qt[r].y * sv[u].y + qt[r].z * sv[u].z + qt[r].w * sv[u].w;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int t = 4 * ty + r;
      const float el = expf(lam[t]);
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[r][u] *= el;
      for (int s = 0; s <= t; ++s) {
        const float m = M[t * MP + s];
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[r][u] += m * Vt[s * OP + tx + 16 * u];
      }
      const int tg = c * LC + t;
      if (tg < T) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          out[(((long)b * T + tg) * Hv + h) * D + col0 + tx + 16 * u] = __float2bfloat16_rn(acc[r][u]);
      }
    }
  }
}

// ---------------------------------------------------------------- 3 (D = 128): outputs on tcgen05
// Same outputs as gdn_out_kernel, as three bf16 MMAs per (chunk, value head) with fp32 accumulators in TMEM:
//   D_M = [Q; K] K^T   (128 x 64, rows 0..63 = q_t . k_s; the K K^T half is unused)
//   D_1 = S0 Q^T       (128 value rows i x 64 steps t)
//   D_2 = Vt^T M'^T    (128 x 64), M'[t][s] = e^{Lambda_t - Lambda_s} (q_t . k_s) for s <= t, built from D_M
//   o[t][i] = e^{Lambda_t} D_1[i][t] + D_2[i][t].
// Operands are written by the threads as K-major 128-byte-swizzled tiles (16-byte chunk c of row r at
// c ^ (r & 7)); one elected thread issues the MMAs; waits are bounded (2 s) and give up cleanly.
namespace tc {
constexpr int ATOM = 128 * 128;  // one 64-wide K atom of a 128-row bf16 tile, bytes
constexpr int QK_OFF = 0, S_OFF = 2 * ATOM, VT_OFF = 4 * ATOM, MP_OFF = 5 * ATOM;
constexpr int BYTES = MP_OFF + 64 * 128 + 1024 /*align*/ + 512 /*lam, barriers*/;

RT_DEVICE void put_chunk(uint8_t* tile, int rows, int r, int k8, const float* v) {  // k8: 16-byte chunk index along K
  const int atom = k8 >> 3, c = k8 & 7;
  __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[1]), p1 = __floats2bfloat162_rn(v[2], v[3]);
  __nv_bfloat162 p2 = __floats2bfloat162_rn(v[4], v[5]), p3 = __floats2bfloat162_rn(v[6], v[7]);
  uint4 u;
  u.x = *reinterpret_cast<uint32_t*>(&p0); u.y = *reinterpret_cast<uint32_t*>(&p1);
  u.z = *reinterpret_cast<uint32_t*>(&p2); u.w = *reinterpret_cast<uint32_t*>(&p3);
  *reinterpret_cast<uint4*>(tile + atom * rows * 128 + r * 128 + ((c ^ (r & 7)) << 4)) = u;
}
RT_DEVICE void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
}  // namespace tc

__global__ void __launch_bounds__(128)
gdn_out_tc_kernel(const float* __restrict__ qn, const float* __restrict__ kn, const float* __restrict__ U,
                  const float* __restrict__ lam_in, const float* __restrict__ S0, bf16* __restrict__ out, int T,
                  int Tp, int Hk, int Hv, int* __restrict__ status) {
  constexpr int D = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = sm100::align_smem_1024(smem_raw);
  uint8_t* QK = sm + tc::QK_OFF;   // 128 rows (q_0..63, k_0..63) x 128 keys
  uint8_t* Sx = sm + tc::S_OFF;    // 128 value rows x 128 keys
  uint8_t* VT = sm + tc::VT_OFF;   // 128 value rows x 64 steps
  uint8_t* MP = sm + tc::MP_OFF;   // 64 steps t x 64 steps s
  float* lam = reinterpret_cast<float*>(MP + 64 * 128);
  uint64_t* bars = reinterpret_cast<uint64_t*>(lam + LC);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z, kh = h / (Hv / Hk);
  const int chunks = Tp / LC, t0 = c * LC, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long rowbase = ((long)b * Hv + h) * Tp + t0;
  if (tid == 0) {
    sm100::mbar_init(&bars[0], 1);
    sm100::mbar_init(&bars[1], 1);
    sm100::fence_barrier_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tslot, 256);
    sm100::tmem_relinquish();
  }
  // operands: q/k rows (fp32 -> bf16), S0 rows, Vt transposed, Lambda. Loads of four iterations are issued
  // before their shared-memory stores so that 16 (then 32) global loads per thread are in flight.
  const float* s0c = S0 + (((long)b * Hv + h) * chunks + c) * D * D;
#pragma unroll 1
  for (int e0 = tid; e0 < 128 * 16; e0 += 4 * 128) {
    float4 qk[4][2], sv[4][2];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int e = e0 + g * 128, r = e >> 4, k8 = e & 15, t = t0 + (r & 63);
      if (t < T) {
        const float* src = (r < 64 ? qn : kn) + (((long)b * T + t) * Hk + kh) * D + 8 * k8;
        qk[g][0] = __ldg(reinterpret_cast<const float4*>(src));
        qk[g][1] = __ldg(reinterpret_cast<const float4*>(src + 4));
      } else {
        qk[g][0] = qk[g][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      const float* srow = s0c + (long)r * D + 8 * k8;
      sv[g][0] = __ldg(reinterpret_cast<const float4*>(srow));
      sv[g][1] = __ldg(reinterpret_cast<const float4*>(srow + 4));
    }
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int e = e0 + g * 128, r = e >> 4, k8 = e & 15;
      const float v[8] = {qk[g][0].x, qk[g][0].y, qk[g][0].z, qk[g][0].w, qk[g][1].x, qk[g][1].y, qk[g][1].z, qk[g][1].w};
      tc::put_chunk(QK, 128, r, k8, v);
      const float w[8] = {sv[g][0].x, sv[g][0].y, sv[g][0].z, sv[g][0].w, sv[g][1].x, sv[g][1].y, sv[g][1].z, sv[g][1].w};
      tc::put_chunk(Sx, 128, r, k8, w);
    }
  }
  {  // Vt^T: thread = value row i, 64 steps (32 loads in flight)
    const int i = tid;
#pragma unroll 1
    for (int k0 = 0; k0 < 8; k0 += 4) {
      float v[4][8];
#pragma unroll
      for (int g = 0; g < 4; ++g)
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int tt = 8 * (k0 + g) + u;
          v[g][u] = t0 + tt < T ? __ldg(U + (rowbase + tt) * D + i) : 0.f;
        }
#pragma unroll
      for (int g = 0; g < 4; ++g) tc::put_chunk(VT, 128, i, k0 + g, v[g]);
    }
  }
  if (tid < LC) lam[tid] = lam_in[rowbase + tid];
  tc::fence_proxy_async();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t idesc = sm100::idesc_bf16(128, 64, false, false);
  bool ok = true;
  if (warp == 0 && sm100::elect_one()) {
    const uint32_t qk = sm100::smem_u32(QK), sx = sm100::smem_u32(Sx);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {  // K = 128 keys: two atoms, four 16-wide steps each
      const uint32_t off = (ks >> 2) * tc::ATOM + (ks & 3) * 32;
      sm100::mma_bf16(tmem + 0, sm100::smem_desc(qk + off, 16, 1024), sm100::smem_desc(qk + off + 64 * 128, 16, 1024),
                      idesc, ks > 0);
      sm100::mma_bf16(tmem + 64, sm100::smem_desc(sx + off, 16, 1024), sm100::smem_desc(qk + off, 16, 1024), idesc,
                      ks > 0);
    }
    sm100::mma_commit(&bars[0]);
  }
  if (!sm100::mbar_wait_bounded(&bars[0], 0)) ok = false;
  sm100::tc_fence_after();
  if (ok && warp < 2) {  // M' rows t = 32 warp + lane
    const int t = 32 * warp + lane;
    float m[64];
    sm100::tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16) + 0, *reinterpret_cast<float(*)[32]>(m));
    sm100::tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16) + 32, *reinterpret_cast<float(*)[32]>(m + 32));
    sm100::tmem_wait_ld();
    const float lt = lam[t];
#pragma unroll
    for (int s = 0; s < 64; ++s) m[s] = s <= t ? expf(lt - lam[s]) * m[s] : 0.f;
#pragma unroll
    for (int k8 = 0; k8 < 8; ++k8) tc::put_chunk(MP, 64, t, k8, m + 8 * k8);
  }
  tc::fence_proxy_async();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (ok && warp == 0 && sm100::elect_one()) {
    const uint32_t vt = sm100::smem_u32(VT), mp = sm100::smem_u32(MP);
#pragma unroll
    for (int ks = 0; ks < LC / 16; ++ks)
      sm100::mma_bf16(tmem + 128, sm100::smem_desc(vt + ks * 32, 16, 1024), sm100::smem_desc(mp + ks * 32, 16, 1024),
                      idesc, ks > 0);
    sm100::mma_commit(&bars[1]);
  }
  if (ok && !sm100::mbar_wait_bounded(&bars[1], 0)) ok = false;
  sm100::tc_fence_after();
  if (ok) {  // rows i = 32 warp + lane; 64 steps
    const int i = 32 * warp + lane;
    const uint32_t row = tmem + ((uint32_t)(32 * warp) << 16);
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      float d1[32], d2[32];
      sm100::tmem_ld32(row + 64 + 32 * half, d1);
      sm100::tmem_ld32(row + 128 + 32 * half, d2);
      sm100::tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const int t = 32 * half + u, tg = t0 + t;
        if (tg < T) out[(((long)b * T + tg) * Hv + h) * D + i] = __float2bfloat16_rn(expf(lam[t]) * d1[u] + d2[u]);
      }
    }
  }
  if (!ok && tid == 0 && status) atomicExch(status, 1);
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 256);
  }
}

// ---------------------------------------------------------------- 2 (D = 128): state pass on tcgen05
// Same recurrence as gdn_state_kernel, one CTA (128 threads, thread i = value row i = TMEM lane i) per head. The
// fp32 state S[i][j] lives in TMEM columns [0, 128) as the accumulator of the chunk's rank-64 update, so it sums in
// fp32; only the products take tf32 operands. Per chunk:
//   1. S (TMEM) -> registers -> chunk-start state S0out and the K-major operand tile A1 = S; TMEM <- e^{Lambda_L} S;
//   2. D1 (TMEM cols [128, 192)) = A1 W^T             (M = 128 i, N = 64 t, K = 128 j, 16 tf32 MMAs);
//   3. Vt[t][i] = U0[t][i] + D1[i][t] (to U), A2[i][t] = Vt[t][i] e^{Lambda_L - Lambda_t};
//   4. S += A2 K                                      (M = 128 i, N = 128 j, K = 64 t, 8 tf32 MMAs).
// Operand tiles are 128-byte-swizzled K-major (16-byte chunk c of row r at c ^ (r & 7)); W, U0 and Lambda of the
// next chunk stream in with cp.async during step 4; K is transposed to [j][t] by the threads from registers loaded
// one chunk ahead (the loads are in flight during the MMAs). Waits are bounded.
namespace tcs {
constexpr int A1_OFF = 0;                    // S: 128 rows x 128 fp32 (4 atoms of 16 KB)
constexpr int B1_OFF = A1_OFF + 64 * 1024;   // W: 64 rows x 128 fp32 (4 atoms of 8 KB)
constexpr int A2_OFF = B1_OFF + 32 * 1024;   // Vt^T scaled: 128 rows x 64 fp32 (2 atoms of 16 KB)
constexpr int B2_OFF = A2_OFF + 32 * 1024;   // K^T: 128 rows x 64 fp32 (2 atoms of 16 KB)
constexpr int U0_OFF = B2_OFF + 32 * 1024;   // U0: [64 t][128 i] fp32, natural layout
constexpr int MISC_OFF = U0_OFF + 32 * 1024; // lam[64], fac[64], barrier, TMEM slot
constexpr int BYTES = MISC_OFF + 1024 + 1024 /*align*/;

// 16-byte chunk q (4 fp32) of row r in a K-major SW128 tile of `rows` rows
RT_DEVICE uint32_t chunk_off(int rows, int r, int q) {
  return (uint32_t)((q >> 3) * rows * 128 + r * 128 + (((q & 7) ^ (r & 7)) << 4));
}
}  // namespace tcs

// 256 threads: two warpgroups address the same 128 TMEM lanes (thread i and i + 128 own value row i) and split
// every per-row pass by columns (state columns j, steps t, K rows).
__global__ void __launch_bounds__(256)
gdn_state_tc_kernel(const float* __restrict__ kn, const float* __restrict__ W, float* __restrict__ U,
                    const float* __restrict__ lam_in, float* __restrict__ state, float* __restrict__ S0out, int T,
                    int Tp, int Hk, int Hv, int* __restrict__ status) {
  constexpr int D = 128, NTH = 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = sm100::align_smem_1024(smem_raw);
  float* U0s = reinterpret_cast<float*>(sm + tcs::U0_OFF);
  float* lam = reinterpret_cast<float*>(sm + tcs::MISC_OFF);
  float* fac = lam + LC;
  uint64_t* bar = reinterpret_cast<uint64_t*>(fac + LC);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  const int h = blockIdx.x, b = blockIdx.y, kh = h / (Hv / Hk);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = tid & 127, half = tid >> 7;  // value row i (TMEM lane) and column half
  const int chunks = Tp / LC;
  const long rowbase = ((long)b * Hv + h) * Tp;
  float* st = state + ((long)b * Hv + h) * D * D;  // [j][i]
  if (tid == 0) {
    sm100::mbar_init(bar, 1);
    sm100::fence_barrier_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tslot, 256);
    sm100::tmem_relinquish();
  }
  auto prefetch = [&](int c) {  // W (swizzled B1), U0 (natural), lam of chunk c: one cp.async group
    for (int e = tid; e < LC * 32; e += NTH) {
      const int t = e >> 5, q = e & 31;
      rt::cp_async16(sm + tcs::B1_OFF + tcs::chunk_off(LC, t, q), W + (rowbase + c * LC + t) * D + 4 * q, true);
      rt::cp_async16(U0s + t * D + 4 * q, U + (rowbase + c * LC + t) * D + 4 * q, true);
    }
    if (tid < LC / 4) rt::cp_async16(lam + 4 * tid, lam_in + rowbase + c * LC + 4 * tid, true);
    rt::cp_async_commit();
  };
  prefetch(0);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tm = *tslot;
  const uint32_t trow = tm + ((uint32_t)((warp & 3) * 32) << 16);
  {  // initial state: lane i, this half's columns j
#pragma unroll 1
    for (int q = 2 * half; q < 2 * half + 2; ++q) {
      float v[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) v[u] = st[(long)(32 * q + u) * D + row];
      sm100::tmem_st32(trow + 32 * q, v);
    }
    sm100::tmem_wait_st();
  }
  const uint32_t idesc1 = sm100::idesc_tf32(128, 64), idesc2 = sm100::idesc_tf32(128, 128);
  const uint32_t a1 = sm100::smem_u32(sm + tcs::A1_OFF), b1 = sm100::smem_u32(sm + tcs::B1_OFF);
  const uint32_t a2 = sm100::smem_u32(sm + tcs::A2_OFF), b2 = sm100::smem_u32(sm + tcs::B2_OFF);
  uint32_t phase = 0;
  bool ok = true;
  // K[t][j = row] for this half's 32 steps of a chunk (rows t < T, zero beyond): 32 independent loads in flight
  float kreg[LC / 2];
  auto load_k = [&](int c) {
#pragma unroll
    for (int u = 0; u < LC / 2; ++u) {
      const int tg = c * LC + (LC / 2) * half + u;
      kreg[u] = tg < T ? __ldg(kn + (((long)b * T + tg) * Hk + kh) * D + row) : 0.f;
    }
  };
  load_k(0);
#pragma unroll 1
  for (int c = 0; c < chunks && ok; ++c) {
    // ---- 1. S -> S0out, A1; TMEM <- e^{Lambda_L} S (this half's 64 columns)
    rt::cp_async_wait<0>();
    __syncthreads();  // W, U0, lam of chunk c visible to every thread
    if (tid < LC) fac[tid] = expf(lam[LC - 1] - lam[tid]);
    const float eL = expf(lam[LC - 1]);
#pragma unroll 1
    for (int q = 2 * half; q < 2 * half + 2; ++q) {
      float v[32];
      sm100::tmem_ld32(trow + 32 * q, v);
      sm100::tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 8; ++u)
        *reinterpret_cast<float4*>(sm + tcs::A1_OFF + tcs::chunk_off(128, row, 8 * q + u)) =
            make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
#pragma unroll
      for (int u = 0; u < 32; ++u) v[u] *= eL;
      sm100::tmem_st32(trow + 32 * q, v);
    }
    // K^T rows j = row, this half's steps (chunks q of 4 steps), from registers loaded during the previous chunk
#pragma unroll
    for (int q = 0; q < LC / 8; ++q)
      *reinterpret_cast<float4*>(sm + tcs::B2_OFF + tcs::chunk_off(128, row, (LC / 8) * half + q)) =
          make_float4(kreg[4 * q], kreg[4 * q + 1], kreg[4 * q + 2], kreg[4 * q + 3]);
    sm100::tmem_wait_st();
    tc::fence_proxy_async();
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    // ---- 2. D1 = A1 W^T; meanwhile the chunk-start state goes from the A1 tile to S0out, one row per warp
    // instruction (coalesced; MMA and copy only read A1)
    if (tid == 0) {
#pragma unroll
      for (int ks = 0; ks < D / 8; ++ks) {
        const uint32_t ka = (ks >> 2) * (128 * 128) + (ks & 3) * 32, kb = (ks >> 2) * (LC * 128) + (ks & 3) * 32;
        sm100::mma_tf32(tm + 128, sm100::smem_desc(a1 + ka, 16, 1024), sm100::smem_desc(b1 + kb, 16, 1024), idesc1,
                        ks > 0);
      }
      sm100::mma_commit(bar);
    }
    {
      float* s0 = S0out + (((long)b * Hv + h) * chunks + c) * D * D;
      for (int e = tid; e < 128 * 32; e += NTH) {  // e: row (e / 32), 16-byte chunk (e % 32)
        const int r = e >> 5, qq = e & 31;
        *reinterpret_cast<float4*>(s0 + (long)r * D + 4 * qq) =
            *reinterpret_cast<const float4*>(sm + tcs::A1_OFF + tcs::chunk_off(128, r, qq));
      }
    }
    if (c + 1 < chunks) load_k(c + 1);  // B2 was written from kreg above; these loads land during the MMAs
    ok = __syncthreads_and(sm100::mbar_wait_bounded(bar, phase) ? 1 : 0) != 0;  // uniform: every thread agrees
    phase ^= 1;
    sm100::tc_fence_after();
    if (!ok) break;
    // ---- 3. Vt = U0 + D1 (to U), A2 = Vt^T scaled: this half's 32 steps
    {
      float d[32];
      sm100::tmem_ld32(trow + 128 + 32 * half, d);
      sm100::tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const int t = 32 * half + u;
        const float v = U0s[t * D + row] + d[u];
        U[(rowbase + c * LC + t) * D + row] = v;
        d[u] = v * fac[t];
      }
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<float4*>(sm + tcs::A2_OFF + tcs::chunk_off(128, row, 8 * half + q)) =
            make_float4(d[4 * q], d[4 * q + 1], d[4 * q + 2], d[4 * q + 3]);
    }
    tc::fence_proxy_async();
    sm100::tc_fence_before();
    __syncthreads();  // A2 complete; W, U0, lam, fac of chunk c no longer read
    sm100::tc_fence_after();
    if (c + 1 < chunks) prefetch(c + 1);
    // ---- 4. S += A2 K
    if (tid == 0) {
#pragma unroll
      for (int ks = 0; ks < LC / 8; ++ks) {
        const uint32_t ko = (ks >> 2) * (128 * 128) + (ks & 3) * 32;
        sm100::mma_tf32(tm, sm100::smem_desc(a2 + ko, 16, 1024), sm100::smem_desc(b2 + ko, 16, 1024), idesc2, 1);
      }
      sm100::mma_commit(bar);
    }
    ok = __syncthreads_and(sm100::mbar_wait_bounded(bar, phase) ? 1 : 0) != 0;
    phase ^= 1;
    sm100::tc_fence_after();
  }
  rt::cp_async_wait<0>();
  if (ok) {  // final state, [j][i]: this half's columns
#pragma unroll 1
    for (int q = 2 * half; q < 2 * half + 2; ++q) {
      float v[32];
      sm100::tmem_ld32(trow + 32 * q, v);
      sm100::tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 32; ++u) st[(long)(32 * q + u) * D + row] = v[u];
    }
  } else if (tid == 0 && status) {
    atomicExch(status, 1);
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tm, 256);
  }
}

// q/k normalisation: qn = q / |q| * D^-1/2, kn = k / |k| (eps 1e-6), fp32 rows [B, T, Hk, D]. grid (T, B).
template <int D>
__global__ void __launch_bounds__(128) gdn_norm_kernel(const bf16* __restrict__ qkv, long row_stride, int T, int Hk,
                                                       float* __restrict__ qn, float* __restrict__ kn) {
  const int t = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float scale = rsqrtf((float)D);
  const bf16* row = qkv + ((long)b * T + t) * row_stride;
  for (int hh = warp; hh < 2 * Hk; hh += 4) {
    const bool is_k = hh >= Hk;
    const int kh = is_k ? hh - Hk : hh;
    float x[D / 32];
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < D / 32; ++u) {
      x[u] = rt::to_f(row[(long)hh * D + lane + 32 * u]);
      ss += x[u] * x[u];
    }
    ss = rt::warp_sum(ss);
    const float f = rsqrtf(ss + 1e-6f) * (is_k ? 1.f : scale);
    float* dst = (is_k ? kn : qn) + (((long)b * T + t) * Hk + kh) * D;
#pragma unroll
    for (int u = 0; u < D / 32; ++u) dst[lane + 32 * u] = x[u] * f;
  }
}

// ---------------------------------------------------------------- 1 on tcgen05 (head dim 128)
// Per (chunk, value head, batch), 256 threads: TMA brings the chunk's normalised k rows (fp32, K-major 128-byte
// swizzled) and raw v rows (bf16); K K^T is one tf32 MMA into TMEM; T = (I + A)^{-1} comes column by column from
// an fp32 forward substitution (threads 0..63, one unit right-hand side each) while the other threads build the
// B operand [V'^T; K'^T] with V' = beta v and K' = diag(beta e^Lambda) k; then [U0 | -W] = T [V' | K'] is a
// second tf32 MMA (N = 256). Waits are bounded; a failure is recorded in the status word.
namespace wyt {
constexpr int KB = 1024;
constexpr int KT = 0;          // k rows: 64 x 128 fp32, 4 atoms (read as 128 rows: the next 8 KB stay in bounds)
constexpr int VR = 32 * KB;    // v rows: two bf16 64 x 64 swizzled boxes
constexpr int MPL = 48 * KB;   // -A, plain swizzled 64 x 64 fp32
constexpr int TA = 64 * KB;    // T (rows t, K = s), 2 atoms (read as 128 rows)
constexpr int BT = 80 * KB;    // [V'^T; K'^T]: 256 rows, K = s, 2 atoms of 32 KB
constexpr int MISC = 144 * KB; // barriers, TMEM slot, lam / beta / e^lam, scan scratch
constexpr int BYTES = 145 * KB + 1024;
}  // namespace wyt

__global__ void __launch_bounds__(256, 1)
gdn_wy_tc_kernel(const __grid_constant__ CUtensorMap m_k, const __grid_constant__ CUtensorMap m_v,
                 const bf16* __restrict__ pa, const bf16* __restrict__ pb, long ab_stride,
                 const float* __restrict__ A_log, const float* __restrict__ dt_bias, float* __restrict__ Wout,
                 float* __restrict__ Uout, float* __restrict__ lam_out, int T, int Tp, int Hk, int Hv,
                 int* __restrict__ status) {
  constexpr int D = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = sm100::align_smem_1024(smem_raw);
  uint8_t *KTt = sm + wyt::KT, *VR = sm + wyt::VR, *TA = sm + wyt::TA, *BT = sm + wyt::BT;
  float* MPL = reinterpret_cast<float*>(sm + wyt::MPL);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + wyt::MISC);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + wyt::MISC + 16);
  float* lam = reinterpret_cast<float*>(sm + wyt::MISC + 64);
  float* beta = lam + LC;
  float* elam = beta + LC;
  float* tmp = elam + LC;
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, quarter = warp & 3, colh = warp >> 2;
  const int kh = h / (Hv / Hk);
  const int t0 = c * LC;
  if (tid == 0) {
    sm100::mbar_init(&bars[0], 1);
    sm100::mbar_init(&bars[1], 1);
    sm100::fence_barrier_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tslot, 256);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    sm100::mbar_expect_tx(&bars[0], 48 * wyt::KB);
#pragma unroll
    for (int a = 0; a < 4; ++a) sm100::tma_load_3d(KTt + a * 8 * wyt::KB, &m_k, &bars[0], kh * D + 32 * a, t0, b);
    const int vcol = 2 * Hk * D + h * D;
#pragma unroll
    for (int a = 0; a < 2; ++a) sm100::tma_load_3d(VR + a * 8 * wyt::KB, &m_v, &bars[0], vcol + 64 * a, t0, b);
  }
  // gates of the chunk's steps (padded steps: beta = 0, g = 0)
  float g = 0.f, bt = 0.f;
  if (tid < LC) {
    const int t = t0 + tid;
    if (t < T) {
      g = gate_g(rt::to_f(pa[((long)b * T + t) * ab_stride + h]), dt_bias[h], -expf(A_log[h]));
      bt = __bfloat162float(__float2bfloat16_rn(rt::sigmoidf_(rt::to_f(pb[((long)b * T + t) * ab_stride + h]))));
    }
  }
  const float lt = scan64(tid < LC ? g : 0.f, tmp);
  if (tid < LC) {
    lam[tid] = lt;
    beta[tid] = bt;
    elam[tid] = expf(lt);
    lam_out[((long)b * Hv + h) * Tp + t0 + tid] = lt;
  }
  int stage = 1;
  bool ok = sm100::mbar_wait_bounded(&bars[0], 0);
  ok = __syncthreads_and(ok ? 1 : 0) != 0;  // also publishes lam / beta
  uint32_t mph = 0;
  if (ok) {
    if (tid == 0) {  // K K^T (cols 0..63): A = k rows (64, read as 128), B = k rows; K = 128
      wtc::fence_async_smem();
      sm100::tc_fence_after();
      wtc::mma_tf32_tiles(tmem, sm100::smem_u32(KTt), 64, sm100::smem_u32(KTt), 64, 16, sm100::idesc_tf32(128, 64),
                          false);
      sm100::mma_commit(&bars[1]);
    }
    // B operand rows while the MMA runs: row r < 128: V'^T row i = r (beta_s v_s[i]); else K'^T row j = r - 128
    // (beta_s e^{Lambda_s} k_s[j]); K = s, 64 steps.
    {
      const int r = tid;
#pragma unroll 1
      for (int s0 = 0; s0 < LC; s0 += 16) {
        float x[16];
        if (r < D) {
          const uint8_t* box = VR + (r >> 6) * 8 * wyt::KB;
#pragma unroll
          for (int q = 0; q < 16; ++q) x[q] = wtc::raw(box, s0 + q, r & 63) * beta[s0 + q];
        } else {
          const int j = r - D;
#pragma unroll
          for (int q = 0; q < 16; ++q) x[q] = wtc::get1(KTt, 64, s0 + q, j) * (beta[s0 + q] * elam[s0 + q]);
        }
#pragma unroll
        for (int q = 0; q < 16; q += 4) wtc::put4(BT, 256, r, s0 + q, x[q], x[q + 1], x[q + 2], x[q + 3]);
      }
    }
    stage = 2;
    ok = sm100::mbar_wait_bounded(&bars[1], mph);
    ok = __syncthreads_and(ok ? 1 : 0) != 0;
    mph ^= 1;
    sm100::tc_fence_after();
  }
  if (ok) {
    // -A[t][s] = -beta_t e^{Lambda_t - Lambda_s} (k_t . k_s) for s < t (lanes 0..63, 32 columns per thread)
    if (quarter < 2) {
      const int t = 32 * quarter + (tid & 31), s0 = 32 * colh;
      float d[32];
      sm100::tmem_ld32(tmem + ((uint32_t)(32 * quarter) << 16) + s0, d);
      sm100::tmem_wait_ld();
      const float bl = beta[t], lt = lam[t];
#pragma unroll
      for (int u = 0; u < 32; u += 4) {
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int s = s0 + u + e;
          v[e] = s < t ? -bl * expf(lt - lam[s]) * d[u + e] : 0.f;
        }
        *reinterpret_cast<float4*>(&MPL[wtc::poff(t, s0 + u)]) = make_float4(v[0], v[1], v[2], v[3]);
      }
    }
    __syncthreads();
    // T column c = (I - M)^{-1} e_c with M = -A (threads 0..63), into the A operand tile (rows t, K = s)
    if (tid < LC) {
      float x[64];
#pragma unroll
      for (int t = 0; t < 64; ++t) x[t] = t == tid ? 1.f : 0.f;
      wtc::solve_lower(MPL, x);
#pragma unroll
      for (int t = 0; t < 64; ++t) wtc::put1(TA, 64, t, tid, x[t]);
    }
    wtc::tc_sync();
    if (tid == 0) {  // [U0 | -W] = T [V' | K'] (cols 0..255)
      wtc::mma_tf32_tiles(tmem, sm100::smem_u32(TA), 64, sm100::smem_u32(BT), 256, 8, sm100::idesc_tf32(128, 256),
                          false);
      sm100::mma_commit(&bars[1]);
    }
    stage = 3;
    ok = sm100::mbar_wait_bounded(&bars[1], mph);
    ok = __syncthreads_and(ok ? 1 : 0) != 0;
    mph ^= 1;
    sm100::tc_fence_after();
  }
  if (ok && quarter < 2) {  // rows t: U0 (warps with colh 0: cols 0..127), W = -(cols 128..255) (colh 1)
    const int t = 32 * quarter + (tid & 31);
    const long row = ((long)b * Hv + h) * Tp + t0 + t;
    float* dst = (colh ? Wout : Uout) + row * D;
    const float sign = colh ? -1.f : 1.f;
    const uint32_t base = tmem + ((uint32_t)(32 * quarter) << 16) + 128 * colh;
#pragma unroll 1
    for (int part = 0; part < 4; ++part) {
      float d[32];
      sm100::tmem_ld32(base + 32 * part, d);
      sm100::tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 32; u += 4)
        *reinterpret_cast<float4*>(dst + 32 * part + u) =
            make_float4(sign * d[u], sign * d[u + 1], sign * d[u + 2], sign * d[u + 3]);
    }
  }
  if (!ok && tid == 0 && status) atomicCAS(status, 0, 0x500 | stage);
  if (!ok && stage > 1) sm100::mbar_wait_bounded(&bars[1], mph);
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 256);
  }
}

// TMA maps of the tcgen05 WY kernel; false if the layouts do not allow them (the SIMT kernel is used then).
bool wy_tc_maps(CUtensorMap* mk, CUtensorMap* mv, const float* kn, const void* qkv, long row_stride, int B, int T,
                int Hk) {
  if ((row_stride % 8) || (reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(kn) & 15))
    return false;
  const uint64_t kd[3] = {(uint64_t)Hk * 128, (uint64_t)T, (uint64_t)B};
  const uint64_t ks[2] = {(uint64_t)Hk * 128 * 4, (uint64_t)T * Hk * 128 * 4};
  const uint32_t kbox[3] = {32, 64, 1};
  const uint64_t vd[3] = {(uint64_t)row_stride, (uint64_t)T, (uint64_t)B};
  const uint64_t vs[2] = {(uint64_t)row_stride * 2, (uint64_t)T * row_stride * 2};
  const uint32_t vbox[3] = {64, 64, 1};
  return tmap::encode(mk, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, kn, kd, ks, kbox) &&
         tmap::encode(mv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, qkv, vd, vs, vbox);
}

template <int D>
long workspace(int B, int T, int Hk, int Hv) {
  const long Tp = (T + LC - 1) / LC * LC, chunks = Tp / LC;
  return 2L * B * T * Hk * D            // qn, kn
         + 2L * B * Hv * Tp * D         // W, U0 / Vt
         + (long)B * Hv * Tp            // lam
         + (long)B * Hv * chunks * D * D;  // chunk-start states
}

template <int D>
cudaError_t launch(const void* qkv, long row_stride, const void* a, const void* bb, long ab_stride,
                   const float* A_log, const float* dt_bias, float* state, void* out, float* work, int B, int T,
                   int Hk, int Hv, cudaStream_t stream) {
  const int Tp = (T + LC - 1) / LC * LC, chunks = Tp / LC;
  float* qn = work;
  float* kn = qn + (long)B * T * Hk * D;
  float* W = kn + (long)B * T * Hk * D;
  float* U = W + (long)B * Hv * Tp * D;
  float* lam = U + (long)B * Hv * Tp * D;
  float* S0 = lam + (long)B * Hv * Tp;
  gdn_norm_kernel<D><<<dim3(T, B), 128, 0, stream>>>((const bf16*)qkv, row_stride, T, Hk, qn, kn);
  RT_CUDA_CHECK(cudaGetLastError());
  const int s1 = WySmem<D>::FLOATS * 4, s2 = StSmem<D>::FLOATS * 4, s3 = OutSmem<D>::FLOATS * 4;
  RT_CUDA_CHECK(cudaFuncSetAttribute(gdn_wy_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, s1));
  RT_CUDA_CHECK(cudaFuncSetAttribute(gdn_state_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, s2));
  RT_CUDA_CHECK(cudaFuncSetAttribute(gdn_out_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, s3));
  // WY pass: tcgen05 form for head dim 128 (THESEUS_GDN_WY_TC=0 selects the SIMT kernel, which other sizes use)
  static const bool wy_tc = [] {
    const char* e = getenv("THESEUS_GDN_WY_TC");
    return !(e && e[0] == '0');
  }();
  CUtensorMap mk, mv;
  if (D == 128 && wy_tc && wy_tc_maps(&mk, &mv, kn, qkv, row_stride, B, T, Hk)) {
    RT_CUDA_CHECK(cudaFuncSetAttribute(gdn_wy_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, wyt::BYTES));
    gdn_wy_tc_kernel<<<dim3(chunks, Hv, B), 256, wyt::BYTES, stream>>>(mk, mv, (const bf16*)a, (const bf16*)bb,
                                                                        ab_stride, A_log, dt_bias, W, U, lam, T, Tp,
                                                                        Hk, Hv, nullptr);
  } else {
    gdn_wy_kernel<D><<<dim3(chunks, Hv, B), NT, s1, stream>>>(kn, (const bf16*)qkv, row_stride, (const bf16*)a,
                                                               (const bf16*)bb, ab_stride, A_log, dt_bias, W, U, lam,
                                                               T, Tp, Hk, Hv);
  }
  RT_CUDA_CHECK(cudaGetLastError());
  // tcgen05 state pass for head dim 128 (THESEUS_GDN_STATE_TC=0 selects the SIMT pass, which other sizes use)
  static const bool state_tc = [] {
    const char* e = getenv("THESEUS_GDN_STATE_TC");
    return !(e && e[0] == '0');
  }();
  if (D == 128 && state_tc) {
    RT_CUDA_CHECK(cudaFuncSetAttribute(gdn_state_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, tcs::BYTES));
    gdn_state_tc_kernel<<<dim3(Hv, B), 256, tcs::BYTES, stream>>>(kn, W, U, lam, state, S0, T, Tp, Hk, Hv, nullptr);
  } else {
    gdn_state_kernel<D><<<dim3(D / VB, Hv, B), NT, s2, stream>>>(kn, W, U, lam, state, S0, T, Tp, Hk, Hv);
  }
  RT_CUDA_CHECK(cudaGetLastError());
  if constexpr (D == 128) {
    RT_CUDA_CHECK(cudaFuncSetAttribute(gdn_out_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::BYTES));
    gdn_out_tc_kernel<<<dim3(chunks, Hv, B), 128, tc::BYTES, stream>>>(qn, kn, U, lam, S0, (bf16*)out, T, Tp, Hk, Hv,
                                                                       nullptr);
  } else {
    gdn_out_kernel<D><<<dim3(chunks, Hv, B * (D / OB)), NT, s3, stream>>>(qn, kn, U, lam, S0, (bf16*)out, T, Tp, Hk,
                                                                          Hv);
  }
  return cudaGetLastError();
}

}  // namespace rt_gdn_wy

// Workspace floats of the WY path (D = 64 or 128).
long rt_gdn_wy_workspace_floats(int B, int T, int Hk, int Hv, int D) {
  return D == 128 ? rt_gdn_wy::workspace<128>(B, T, Hk, Hv) : rt_gdn_wy::workspace<64>(B, T, Hk, Hv);
}

cudaError_t rt_gdn_wy_forward(const void* qkv, long row_stride, const void* a, const void* b, long ab_stride,
                              const float* A_log, const float* dt_bias, float* state, void* out, float* work, int B,
                              int T, int Hk, int Hv, int D, cudaStream_t stream) {
  switch (D) {
    case 128:
      return rt_gdn_wy::launch<128>(qkv, row_stride, a, b, ab_stride, A_log, dt_bias, state, out, work, B, T, Hk, Hv,
                                    stream);
    case 64:
      return rt_gdn_wy::launch<64>(qkv, row_stride, a, b, ab_stride, A_log, dt_bias, state, out, work, B, T, Hk, Hv,
                                   stream);
    default:
      return cudaErrorInvalidValue;
  }
}
