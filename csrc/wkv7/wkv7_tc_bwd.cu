// WKV7 backward on tcgen05 (head size 64, chunks of 64 steps), the adjoint of wkv7_tc_fwd.cu, sm_100a.
// The recurrence is RWKV7's (RWKV-LM, Apache-2.0; see NOTICE at the project root); this code is our own.
//
// With dS the gradient of a chunk's end state and dY of its outputs, the chunk-start gradient is
//     dS0 = dS G^T + dY^T Q                       (G, Q from the forward records),
// a serial scan over chunks (kernel 1). Per chunk, from the chunk-start state S0 (forward checkpoint) and dS,
// with T = (I - M_ab)^{-1} applied by an fp32 triangular solve (never formed):
//     U  = T (A~ S0^T + M_ak V) = W S0^T + U0      (the chunk's u_t = S_{t-1} a_t rows; W, U0 from the forward)
//     dU = M_rb^T dY + B^ dS^T,  dZ = T^T dU,  dV = M_rk^T dY + K^ dS^T + M_ak^T dZ          (kernel 2)
//     dM_ab = (dZ U^T) strict, dM_ak = (dZ V^T) strict, dM_rb = (dY U^T) incl, dM_rk = (dY V^T) incl
//     dA~ = dZ S0 + dM_ab B~ + dM_ak K~,   dR~ = dY S0 + dM_rb B~ + dM_rk K~
//     dB~ = dM_ab^T A~ + dM_rb^T R~ + E,   dK~ = dM_ak^T A~ + dM_rk^T R~ + F,   [E; F] = [U; V] dS diag(D_L)
//                                                                                          (kernel 3)
// and the raw gradients da = dA~ e^{Lambda_{t-1}}, dr = dR~ e^{Lambda_t}, db = dB~ e^{-Lambda_t},
// dk = dK~ e^{-Lambda_t}; the decay gradient is the reverse cumulative sum over the chunk of
//     dLambda_t = dr r - db b - dk k + (da a)_{t+1},   plus  sum_i dS S0 D_L + sum_s (E b~ + F k~)  at the end,
// times d log d / dw = -e^{-1/2} sigmoid(w) (1 - sigmoid(w)). Every product is a tf32 MMA into TMEM; the
// masks, transposes and the decay factors are applied by the threads that move tiles between TMEM and shared
// memory. No atomics, fixed summation order (deterministic). Every wait is bounded.
#include "wkv7_tc.cuh"
#include "../common/tmap.cuh"

namespace {

using namespace wtc;

// Optional phase timing (compile with -DWKV7_TC_TRACE): thread 0 of every CTA adds the %globaltimer time spent
// since the previous mark to a per-phase total; rt_wkv7_tc_trace_read copies the totals out. Off by default.
#ifdef WKV7_TC_TRACE
__device__ unsigned long long wkv7_trace_ns[64];
#define WKV_TRACE_BEGIN unsigned long long trace_t0_ = threadIdx.x == 0 ? sm100::globaltimer() : 0ull;
#define WKV_TRACE(slot)                                                       \
  if (threadIdx.x == 0) {                                                     \
    const unsigned long long trace_now_ = sm100::globaltimer();               \
    atomicAdd(&wkv7_trace_ns[(slot)], trace_now_ - trace_t0_);                \
    trace_t0_ = trace_now_;                                                   \
  }
#else
#define WKV_TRACE_BEGIN
#define WKV_TRACE(slot)
#endif

constexpr int KB = 1024;
constexpr int MAT = N * N;
enum { REC_G = 0, REC_H0 = 1, REC_Q = 2, REC_Y0 = 3, REC_W = 4, REC_U0 = 5, REC_MATS = 6 };  // forward record
enum { WK_DS = 0, WK_U = 1, WK_DZ = 2, WK_MATS = 3 };                             // backward work record

__device__ int wkv7_tc_bwd_fault_word = 0;

RT_DEVICE uint8_t* align1024(uint8_t* p) { return sm100::align_smem_1024(p); }
RT_DEVICE bool wait_all(uint64_t* bar, uint32_t parity) {
  const bool ok = sm100::mbar_wait_bounded(bar, parity);
  return __syncthreads_and(ok ? 1 : 0) != 0;
}

// ---------------------------------------------------------------- 1: reverse scan dS <- dS G^T + dY^T Q
// grid (B*H, 8 row blocks of 8 value rows), 128 threads: thread = column j and rows r0..r0+3 of the block.
constexpr int BS_ROWS = 8;
constexpr int GP = 68;  // padded row of G (conflict-free float4 reads of G[j][j'..j'+3] across j)
constexpr int BSCAN_SMEM = (2 * 64 * GP + 2 * MAT + BS_ROWS * 64) * 4 + 2 * 64 * BS_ROWS * 2;
__global__ void __launch_bounds__(128)
wkv7_tc_bscan_kernel(const float* __restrict__ rec, const __nv_bfloat16* __restrict__ dy,
                     const float* __restrict__ dend, float* __restrict__ work, float* __restrict__ ds0, int T, int H,
                     int chunks) {
  extern __shared__ __align__(16) float bsm[];
  float* Gs = bsm;                     // [2][64][GP]
  float* Qs = Gs + 2 * 64 * GP;        // [2][64][64]
  float* dS = Qs + 2 * MAT;            // [8][64]
  __nv_bfloat16* dYs = reinterpret_cast<__nv_bfloat16*>(dS + BS_ROWS * 64);  // [2][64 t][8 rows] raw bf16
  const int bh = blockIdx.x, rb = blockIdx.y * BS_ROWS, tid = threadIdx.x;
  const int b = bh / H, h = bh % H;
  const int j = tid & 63, r0 = (tid >> 6) * 4;
  const float* rec0 = rec + (long)bh * chunks * REC_MATS * MAT;
  auto prefetch = [&](int c) {  // G_c, Q_c and the chunk's dY rows (this block's 8 value columns), one group
    const float* g = rec0 + (long)c * REC_MATS * MAT + REC_G * MAT;
    const float* q = rec0 + (long)c * REC_MATS * MAT + REC_Q * MAT;
    float* gd = Gs + (c & 1) * 64 * GP;
    float* qd = Qs + (c & 1) * MAT;
    for (int e = tid; e < MAT / 4; e += 128) {
      rt::cp_async16(gd + (e >> 4) * GP + 4 * (e & 15), g + 4 * e, true);
      rt::cp_async16(qd + 4 * e, q + 4 * e, true);
    }
    if (tid < 64) {  // 16 bytes per step; past the sequence end the copy reads nothing and fills zeros
      const int tg = c * L + tid;
      const bool valid = tg < T;
      rt::cp_async16(dYs + ((c & 1) * 64 + tid) * BS_ROWS,
                     dy + (((long)b * T + (valid ? tg : 0)) * H + h) * N + rb, valid);
    }
    rt::cp_async_commit();
  };
  prefetch(chunks - 1);
  float s[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    s[q] = dend ? dend[((long)bh * N + rb + r0 + q) * N + j] : 0.f;  // null: zero end-state gradient
    dS[(r0 + q) * 64 + j] = s[q];
  }
#pragma unroll 1
  for (int c = chunks - 1; c >= 0; --c) {
    float* wk = work + ((long)bh * chunks + c) * WK_MATS * MAT + WK_DS * MAT;
#pragma unroll
    for (int q = 0; q < 4; ++q) wk[(rb + r0 + q) * N + j] = s[q];
    rt::cp_async_wait<0>();
    __syncthreads();  // G_c, Q_c, dY_c landed; dS visible; the other buffers are no longer read
    if (c > 0) prefetch(c - 1);
    const float* g = Gs + (c & 1) * 64 * GP;
    const float* qm = Qs + (c & 1) * MAT;
    const __nv_bfloat16* dyc = dYs + (c & 1) * 64 * BS_ROWS;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int jp = 0; jp < 64; jp += 4) {
      const float4 gv = *reinterpret_cast<const float4*>(g + j * GP + jp);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 sv = *reinterpret_cast<const float4*>(dS + (r0 + q) * 64 + jp);
        acc[q] += sv.x * gv.x + sv.y * gv.y + sv.z * gv.z + sv.w * gv.w;
      }
    }
#pragma unroll 8
    for (int t = 0; t < 64; ++t) {
      const float qv = qm[t * 64 + j];
      const uint2 raw4 = *reinterpret_cast<const uint2*>(dyc + t * BS_ROWS + r0);
      const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&raw4.x);
      const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&raw4.y);
      acc[0] += __low2float(lo) * qv;
      acc[1] += __high2float(lo) * qv;
      acc[2] += __low2float(hi) * qv;
      acc[3] += __high2float(hi) * qv;
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      s[q] = acc[q];
      dS[(r0 + q) * 64 + j] = s[q];
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) ds0[((long)bh * N + rb + r0 + q) * N + j] = s[q];
}

// ---------------------------------------------------------------- 2: U, dZ, dV per chunk
namespace ka {
constexpr int RAW = 0;          // r, w, k, v, a, b, dY (8 KB each)
constexpr int LAM = 56 * KB;
constexpr int MISC = 72 * KB;
constexpr int X1 = 73 * KB;     // [A~; R~]                     -> dU^T (89..105)
constexpr int X2 = 105 * KB;    // [B~; K~] -> [M_rb^T; M_rk^T]  -> T^T (105..121)
// 137..153: free until M_ak^T (129..145) is written after MMA-dU
constexpr int BKH = 153 * KB;   // [B^; K^] (128 rows)
constexpr int DYT = 185 * KB;   // dY^T (64 rows)
// after phase A (raw, Lambda dead): S0 (0..16), dS (16..32), M_ab plain (32..48)
constexpr int WT = 201 * KB;    // W (64 rows t, K = j) by TMA; read as 128 rows (the 8 KB after it stay in bounds)
constexpr int SMEM = 225 * KB + 1024;
}  // namespace ka

// 256 threads: the tile and epilogue phases split their rows or TMEM columns over two threads (warps w and w + 4
// share a TMEM lane quarter); the two triangular solves keep one right-hand-side column per thread on the first
// 128 threads.
constexpr int STATE_THREADS = 256;

__global__ void __launch_bounds__(STATE_THREADS, 1)
wkv7_tc_bwd_state_kernel(const __grid_constant__ CUtensorMap m_r, const __grid_constant__ CUtensorMap m_w,
                         const __grid_constant__ CUtensorMap m_k, const __grid_constant__ CUtensorMap m_v,
                         const __grid_constant__ CUtensorMap m_a, const __grid_constant__ CUtensorMap m_b,
                         const __grid_constant__ CUtensorMap m_dy, const __grid_constant__ CUtensorMap m_rec,
                         const float* __restrict__ rec, const float* __restrict__ ckpt,
                         float* __restrict__ work, float* __restrict__ dv, int T, int H, int chunks) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const int c = blockIdx.x, h = blockIdx.y, bb = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int quarter = warp & 3, colh = warp >> 2;
  uint8_t* Rr = sm + ka::RAW;
  uint8_t *Rw = Rr + 8 * KB, *Rk = Rr + 16 * KB, *Rv = Rr + 24 * KB, *Ra = Rr + 32 * KB, *Rb = Rr + 40 * KB;
  uint8_t* Rdy = Rr + 48 * KB;
  float* lam = reinterpret_cast<float*>(sm + ka::LAM);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + ka::MISC);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + ka::MISC + 32);
  uint8_t *X1 = sm + ka::X1, *X2 = sm + ka::X2, *BKH = sm + ka::BKH, *DYT = sm + ka::DYT;
  uint8_t *S0t = sm, *DSt = sm + 16 * KB;
  float* MPL = reinterpret_cast<float*>(sm + 32 * KB);
  float* DUP = reinterpret_cast<float*>(X1 + 16 * KB);  // dU^T, plain (row i = column i of dU)
  uint8_t* WT = sm + ka::WT;
  float* carry = reinterpret_cast<float*>(BKH);         // Lambda carries (before BKH is built)
  uint8_t *MRT = X2, *MAKT = sm + 129 * KB, *DZT = sm;
  const long bh = (long)bb * H + h, ch = bh * chunks + c;
  const float* S0g = ckpt + (bh * (chunks + 1) + c) * MAT;
  float* wk = work + ch * WK_MATS * MAT;
  const int nvalid = min(L, T - c * L);
  const uint32_t trow_off = (uint32_t)(32 * quarter) << 16;
  WKV_TRACE_BEGIN

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
    sm100::mbar_expect_tx(&bars[0], 7 * 8192 + 16 * KB);
    const int x = h * N, y = c * L;
    sm100::tma_load_3d(Rr, &m_r, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rw, &m_w, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rk, &m_k, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rv, &m_v, &bars[0], x, y, bb);
    sm100::tma_load_3d(Ra, &m_a, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rb, &m_b, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rdy, &m_dy, &bars[0], x, y, bb);
    const int wrow = (int)((ch * REC_MATS + REC_W) * N);
    sm100::tma_load_2d(WT, &m_rec, &bars[0], 0, wrow);
    sm100::tma_load_2d(WT + 8 * KB, &m_rec, &bars[0], 32, wrow);
  }
  int stage = 1;
  bool ok = wait_all(&bars[0], 0);
  uint32_t mph = 0;
  WKV_TRACE(16)
  if (ok) {
    float* DLs = reinterpret_cast<float*>(sm + ka::MISC + 64);
    build_lambda_nt<STATE_THREADS>(Rw, lam, carry, nvalid, tid);
    if (tid < 64) DLs[tid] = expf(lam[poff(63, tid)]);
    __syncthreads();
    {  // X1 (A~ / R~), X2 (B~ / K~), BKH (B^ = B~ D_L / K^ = K~ D_L): row tid % 128, 32 keys, eight at a time
      const int r = tid & 127, t = r & 63, j1 = 32 * (tid >> 7);
      const bool hi = r >= 64;
      const uint8_t* s1 = hi ? Rr : Ra;
      const uint8_t* s2 = hi ? Rk : Rb;
#pragma unroll 1
      for (int j0 = j1; j0 < j1 + 32; j0 += 8) {
        float x1[8], x2[8], lt[8], lp[8];
        raw8(s1, t, j0, x1);
        raw8(s2, t, j0, x2);
        *reinterpret_cast<float4*>(lt) = *reinterpret_cast<const float4*>(&lam[poff(t, j0)]);
        *reinterpret_cast<float4*>(lt + 4) = *reinterpret_cast<const float4*>(&lam[poff(t, j0 + 4)]);
        if (!hi && t > 0) {
          *reinterpret_cast<float4*>(lp) = *reinterpret_cast<const float4*>(&lam[poff(t - 1, j0)]);
          *reinterpret_cast<float4*>(lp + 4) = *reinterpret_cast<const float4*>(&lam[poff(t - 1, j0 + 4)]);
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) lp[q] = 0.f;
        }
        float xh[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          x1[q] *= expf(hi ? lt[q] : lp[q]);
          x2[q] *= expf(-lt[q]);
          xh[q] = x2[q] * DLs[j0 + q];
        }
#pragma unroll
        for (int q = 0; q < 8; q += 4) {
          put4(X1, 128, r, j0 + q, x1[q], x1[q + 1], x1[q + 2], x1[q + 3]);
          put4(X2, 128, r, j0 + q, x2[q], x2[q + 1], x2[q + 2], x2[q + 3]);
          put4(BKH, 128, r, j0 + q, xh[q], xh[q + 1], xh[q + 2], xh[q + 3]);
        }
      }
    }
    WKV_TRACE(17)
    {  // dY^T (row i): 16 steps per thread
      const int i = tid & 63, s1 = 16 * (tid >> 6);
      float x[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) x[q] = raw(Rdy, s1 + q, i);
#pragma unroll
      for (int q = 0; q < 16; q += 4) put4(DYT, 64, i, s1 + q, x[q], x[q + 1], x[q + 2], x[q + 3]);
    }
    tc_sync();
    WKV_TRACE(18)
    // ---- MMA1 (cols 0..127): chunk matrices
    if (tid == 0) {
      mma_tf32_tiles(tmem, sm100::smem_u32(X1), 128, sm100::smem_u32(X2), 128, 8, sm100::idesc_tf32(128, 128),
                     false);
      sm100::mma_commit(&bars[1]);
    }
    // raw tiles and Lambda are dead: S0 and dS rows (rounded) by the threads, half a row each
    {
      const int r = tid & 127, k0 = 32 * (tid >> 7);
      uint8_t* tile = r < 64 ? S0t : DSt;
      const float* src = (r < 64 ? S0g : wk + WK_DS * MAT) + (r & 63) * N;
#pragma unroll
      for (int k = k0; k < k0 + 32; k += 4) {
        const float4 v4 = __ldg(reinterpret_cast<const float4*>(src + k));
        put4(tile, 64, r & 63, k, v4.x, v4.y, v4.z, v4.w);
      }
    }
    stage = 2;
    ok = wait_all(&bars[1], mph);
    mph ^= 1;
    sm100::tc_fence_after();
  }
  if (ok) {
    WKV_TRACE(19)
    // ---- epilogue 1 (32 columns of each 64-column block per thread): M_ab (strict) -> MPL (plain);
    //      [M_rb^T; M_rk^T] -> MRT (transposed, from rows t >= 64)
    const int row = 32 * quarter + (tid & 31), t = row & 63, s0 = 32 * colh;
    float d[32];
    sm100::tmem_ld32(tmem + trow_off + s0, d);  // M_ab / M_rb
    sm100::tmem_wait_ld();
    if (row < 64) {
#pragma unroll
      for (int u = 0; u < 32; u += 4) {
        const int s = s0 + u;
        *reinterpret_cast<float4*>(&MPL[poff(t, s)]) =
            make_float4(s < t ? d[u] : 0.f, s + 1 < t ? d[u + 1] : 0.f, s + 2 < t ? d[u + 2] : 0.f,
                        s + 3 < t ? d[u + 3] : 0.f);
      }
    } else {
#pragma unroll
      for (int u = 0; u < 32; ++u) put1(MRT, 128, s0 + u, t, s0 + u <= t ? d[u] : 0.f);
    }
    if (row >= 64) {  // warp-uniform: lane quarters 2 and 3
      sm100::tmem_ld32(tmem + trow_off + 64 + s0, d);  // M_rk
      sm100::tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 32; ++u) put1(MRT, 128, 64 + s0 + u, t, s0 + u <= t ? d[u] : 0.f);
    }
    tc_sync();
    // ---- MMA-U (cols 128..191): [W S0^T; *];  MMA-dU (cols 192..255): [dU; dV'] =
    //      [M_rb^T; M_rk^T] dY + [B^; K^] dS^T
    if (tid == 0) {
      mma_tf32_tiles(tmem + 128, sm100::smem_u32(WT), 64, sm100::smem_u32(S0t), 64, 8, sm100::idesc_tf32(128, 64),
                     false);
      mma_tf32_tiles(tmem + 192, sm100::smem_u32(MRT), 128, sm100::smem_u32(DYT), 64, 8, sm100::idesc_tf32(128, 64),
                     false);
      mma_tf32_tiles(tmem + 192, sm100::smem_u32(BKH), 128, sm100::smem_u32(DSt), 64, 8, sm100::idesc_tf32(128, 64),
                     true);
      sm100::mma_commit(&bars[1]);
    }
    stage = 3;
    ok = wait_all(&bars[1], mph);
    mph ^= 1;
    sm100::tc_fence_after();
  }
  if (ok) {
    WKV_TRACE(20)
    // ---- epilogue 2 (lanes 0..63, 32 columns per thread): U = W S0^T + U0 rows t (tf32) to the work record; dU
    //      rows t -> columns t of the plain dU^T; M_ak row t -> column t of M_ak^T
    const int row = 32 * quarter + (tid & 31), s0 = 32 * colh;
    if (quarter < 2) {
      float e[32];
      sm100::tmem_ld32(tmem + trow_off + 128 + s0, e);  // (W S0^T) row t
      sm100::tmem_wait_ld();
      const float* u0 = rec + (ch * REC_MATS + REC_U0) * MAT + row * N + s0;
      float* gu = wk + WK_U * MAT + row * N + s0;
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float4 b4 = __ldg(reinterpret_cast<const float4*>(u0 + i));
        *reinterpret_cast<float4*>(gu + i) = make_float4(tf32r(e[i] + b4.x), tf32r(e[i + 1] + b4.y),
                                                         tf32r(e[i + 2] + b4.z), tf32r(e[i + 3] + b4.w));
      }
      sm100::tmem_ld32(tmem + trow_off + 192 + s0, e);  // dU row t
      sm100::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) DUP[poff(s0 + i, row)] = e[i];
      sm100::tmem_ld32(tmem + trow_off + 64 + s0, e);  // M_ak row t (still in TMEM)
      sm100::tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 32; ++u) put1(MAKT, 64, s0 + u, row, s0 + u < row ? e[u] : 0.f);
    }
    __syncthreads();
    WKV_TRACE(21)
    // ---- dZ = T^T dU (threads i < 64: column i, back substitution); dZ (tf32) to the work record and as the rows
    //      of dZ^T for dV
    if (tid < 64) {
      float d[64];
      const int i = tid;
#pragma unroll
      for (int s = 0; s < 64; s += 4) {
        const float4 z = *reinterpret_cast<const float4*>(&DUP[poff(i, s)]);
        d[s] = z.x;
        d[s + 1] = z.y;
        d[s + 2] = z.z;
        d[s + 3] = z.w;
      }
      solve_upper_t(MPL, d);
      WKV_TRACE(22)
      float* g = wk + WK_DZ * MAT + i;
#pragma unroll
      for (int s = 0; s < 64; ++s) g[s * N] = tf32r(d[s]);
#pragma unroll
      for (int s = 0; s < 64; s += 4) put4(DZT, 64, i, s, d[s], d[s + 1], d[s + 2], d[s + 3]);
    }
    tc_sync();
    WKV_TRACE(23)
    // ---- MMA-dV (cols 192..255, rows 64..127): dV += M_ak^T dZ  (M_ak^T read as the lower half of 128 rows)
    if (tid == 0) {
      mma_tf32_tiles(tmem + 192, sm100::smem_u32(MAKT) - 8192, 64, sm100::smem_u32(DZT), 64, 8,
                     sm100::idesc_tf32(128, 64), true);
      sm100::mma_commit(&bars[1]);
    }
    stage = 6;
    ok = wait_all(&bars[1], mph);
    mph ^= 1;
    sm100::tc_fence_after();
  }
  if (ok && quarter >= 2) {  // dV rows s (lanes 64..127, 32 columns per thread; the TMEM load is warp-collective)
    const int s = 32 * quarter + (tid & 31) - 64, tg = c * L + s, i0 = 32 * colh;
    float d[32];
    sm100::tmem_ld32(tmem + trow_off + 192 + i0, d);
    sm100::tmem_wait_ld();
    if (s < nvalid) {
      float* out = dv + (((long)bb * T + tg) * H + h) * N + i0;
#pragma unroll
      for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(out + i) = make_float4(d[i], d[i + 1], d[i + 2], d[i + 3]);
    }
  }
  WKV_TRACE(24)
  if (!ok && tid == 0) atomicCAS(&wkv7_tc_bwd_fault_word, 0, 0x200 | stage);  // state kernel, failing wait
  if (!ok && stage > 1) sm100::mbar_wait_bounded(&bars[1], mph);
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 256);
  }
}

// ---------------------------------------------------------------- 3: input gradients per chunk
namespace kb {
constexpr int RAW = 0;          // r, w, k, v, a, b, dY (8 KB each); r, w, k, a, b stay until the row epilogue,
                                // v and dY die once copied, and their slots hold the two atoms of (dS D_L)^T
constexpr int LAM = 56 * KB;
constexpr int MISC = 72 * KB;
constexpr int DZY = 73 * KB;    // [dZ; dY] (128 rows, K = i)  -> stage tile SA -> FW (73..89), QA (89..105)
constexpr int UV = 105 * KB;    // [U; V]   (128 rows, K = i)  -> stage tile SB -> PA (105..121), PB (121..137)
constexpr int X1T = 137 * KB;   // [A~^T | R~^T] (64 rows j, K = 128) -> E arrays
constexpr int X2T = 169 * KB;   // [B~^T | K~^T]
constexpr int S0T = 201 * KB;   // S0^T (64 rows j, K = i)
constexpr int DST0 = 24 * KB;   // (dS D_L)^T atom 0 (keys i < 32), over raw v
constexpr int DST1 = 48 * KB;   // atom 1 (i >= 32), over raw dY
constexpr int SMEM = 217 * KB + 1024;
}  // namespace kb

// 256 threads (8 warps): warps w and w + 4 read the same TMEM lane quarter (rows 32 (w % 4) ..) and split the
// columns between them; the SIMT phases split their row or column ranges the same way, so every phase has twice
// the warps of a 128-thread CTA to hide its latencies (the shared-memory map allows one CTA per SM).
constexpr int GRAD_THREADS = 256;

__global__ void __launch_bounds__(GRAD_THREADS, 1)
wkv7_tc_bwd_grad_kernel(const __grid_constant__ CUtensorMap m_r, const __grid_constant__ CUtensorMap m_w,
                        const __grid_constant__ CUtensorMap m_k, const __grid_constant__ CUtensorMap m_v,
                        const __grid_constant__ CUtensorMap m_a, const __grid_constant__ CUtensorMap m_b,
                        const __grid_constant__ CUtensorMap m_dy, const __grid_constant__ CUtensorMap m_wk,
                        const __nv_bfloat16* __restrict__ pr, const __nv_bfloat16* __restrict__ pw,
                        const __nv_bfloat16* __restrict__ pk, const __nv_bfloat16* __restrict__ pa,
                        const __nv_bfloat16* __restrict__ pb, const float* __restrict__ ckpt,
                        const float* __restrict__ work, float* __restrict__ dr, float* __restrict__ dw,
                        float* __restrict__ dk, float* __restrict__ da, float* __restrict__ db, int T, int H,
                        int chunks) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const int c = blockIdx.x, h = blockIdx.y, bb = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int quarter = warp & 3;  // TMEM lane quarter of this warp
  const int colh = warp >> 2;    // which 32 of a 64-column TMEM block this warp reads
  uint8_t* Rr = sm + kb::RAW;
  uint8_t *Rw = Rr + 8 * KB, *Rk = Rr + 16 * KB, *Rv = Rr + 24 * KB, *Ra = Rr + 32 * KB, *Rb = Rr + 40 * KB;
  uint8_t* Rdy = Rr + 48 * KB;
  float* lam = reinterpret_cast<float*>(sm + kb::LAM);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kb::MISC);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + kb::MISC + 32);
  float* DL = reinterpret_cast<float*>(sm + kb::MISC + 64);
  float* colsum = reinterpret_cast<float*>(sm + kb::X2T);  // [512] (after the stage MMAs): the chunk-end term
                                                           // in four parts, then each quarter's sum of g
  float* carry = reinterpret_cast<float*>(sm + kb::X2T);   // [256] Lambda carries (before X2T is built)
  uint8_t *DZY = sm + kb::DZY, *UV = sm + kb::UV, *X1T = sm + kb::X1T, *X2T = sm + kb::X2T;
  uint8_t *S0T = sm + kb::S0T, *DST0 = sm + kb::DST0, *DST1 = sm + kb::DST1;
  uint8_t *SA = DZY, *SB = UV;  // stage tiles (32 KB each)
  float* PA = reinterpret_cast<float*>(sm + kb::UV);             // dr r - dk k   (rows of the r~ / k~ half)
  float* PB = PA + MAT;                                           // -db b         (rows of the a~ / b~ half)
  float* QA = reinterpret_cast<float*>(sm + kb::DZY + 16 * KB);  // da a
  float* EA = reinterpret_cast<float*>(sm + kb::X1T);            // E b~
  float* EB = EA + MAT;                                           // F k~
  float* FW = reinterpret_cast<float*>(sm + kb::DZY);            // d log d / dw per element
  const long bh = (long)bb * H + h, ch = bh * chunks + c;
  const float* S0g = ckpt + (bh * (chunks + 1) + c) * MAT;

  const float* wk = work + ch * WK_MATS * MAT;
  WKV_TRACE_BEGIN
  const int nvalid = min(L, T - c * L);

  if (tid == 0) {
    for (int i = 0; i < 3; ++i) sm100::mbar_init(&bars[i], 1);
    sm100::fence_barrier_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tslot, 512);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    sm100::mbar_expect_tx(&bars[0], 7 * 8192 + 32 * KB);
    const int x = h * N, y = c * L;
    sm100::tma_load_3d(Rr, &m_r, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rw, &m_w, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rk, &m_k, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rv, &m_v, &bars[0], x, y, bb);
    sm100::tma_load_3d(Ra, &m_a, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rb, &m_b, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rdy, &m_dy, &bars[0], x, y, bb);
    const int zrow = (int)((ch * WK_MATS + WK_DZ) * N), urow = (int)((ch * WK_MATS + WK_U) * N);
    for (int a = 0; a < 2; ++a) {  // top halves (rows 0..63) of the two 128-row operands
      sm100::tma_load_2d(DZY + a * 16 * KB, &m_wk, &bars[0], 32 * a, zrow);
      sm100::tma_load_2d(UV + a * 16 * KB, &m_wk, &bars[0], 32 * a, urow);
    }
  }
  int stage = 1;
  bool ok = wait_all(&bars[0], 0);
  uint32_t mph = 0;
  bool second_issued = false;
  WKV_TRACE(32)
  if (ok) {
    // ---- dY and V rows into the lower halves (thread: one row, 32 columns); the dM product can start
    {
      const int r = tid & 127, t = r & 63, i0 = 32 * (tid >> 7);
      uint8_t* dst = r < 64 ? DZY : UV;
      const uint8_t* src = r < 64 ? Rdy : Rv;
#pragma unroll
      for (int i = i0; i < i0 + 32; i += 8) {
        float x[8];
        raw8(src, t, i, x);
        put4(dst, 128, 64 + t, i, x[0], x[1], x[2], x[3]);
        put4(dst, 128, 64 + t, i + 4, x[4], x[5], x[6], x[7]);
      }
    }
    tc_sync();
    if (tid == 0) {  // dM block (cols 0..127) = [dZ; dY] [U; V]^T
      mma_tf32_tiles(tmem, sm100::smem_u32(DZY), 128, sm100::smem_u32(UV), 128, 8, sm100::idesc_tf32(128, 128),
                     false);
      sm100::mma_commit(&bars[1]);
    }
    build_lambda_nt<GRAD_THREADS>(Rw, lam, carry, nvalid, tid);
    if (tid < 64) DL[tid] = expf(lam[poff(63, tid)]);
    WKV_TRACE(33)
    // X1T row j: A~[t][j] (k = t), R~[t][j] (k = 64 + t); X2T row j: B~ / K~ (column owners; a thread takes 32 steps)
    {
      const int j = tid & 63, second = (tid >> 6) & 1, tbase = 32 * (tid >> 7);
      uint8_t* dst = second ? X2T : X1T;
      const uint8_t* s1 = second ? Rb : Ra;
      const uint8_t* s2 = second ? Rk : Rr;
#pragma unroll 1
      for (int t0 = tbase; t0 < tbase + 32; t0 += 16) {  // 16 steps at a time: loads, exponentials, stores
        float x1[16], x2[16], lt[17];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          x1[q] = raw(s1, t0 + q, j);
          x2[q] = raw(s2, t0 + q, j);
          lt[q + 1] = lam[poff(t0 + q, j)];
        }
        lt[0] = t0 ? lam[poff(t0 - 1, j)] : 0.f;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          if (!second) {  // A~ = a e^{Lambda_{t-1}}, R~ = r e^{Lambda_t}
            x1[q] *= expf(lt[q]);
            x2[q] *= expf(lt[q + 1]);
          } else {        // B~ = b e^{-Lambda_t}, K~ = k e^{-Lambda_t}
            const float dn = expf(-lt[q + 1]);
            x1[q] *= dn;
            x2[q] *= dn;
          }
        }
#pragma unroll
        for (int q = 0; q < 16; q += 4) {
          put4(dst, 64, j, t0 + q, x1[q], x1[q + 1], x1[q + 2], x1[q + 3]);
          put4(dst, 64, j, 64 + t0 + q, x2[q], x2[q + 1], x2[q + 2], x2[q + 3]);
        }
      }
    }
    __syncthreads();  // raw v and dY dead from here on (r, w, k, a, b stay for the row epilogue)
    WKV_TRACE(34)
    {  // S0^T (row j, K = i) and (dS D_L)^T (row j; atom i / 32 in its own slot): column loads from global
      const int j = tid & 63, second = (tid >> 6) & 1, i0 = 32 * (tid >> 7);
      const float* src = second ? wk + WK_DS * MAT : S0g;
      const float sc = second ? DL[j] : 1.f;
      float col[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) col[i] = __ldg(src + (i0 + i) * N + j);
      if (second) {
        uint8_t* atom = i0 ? DST1 : DST0;
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          put4(atom, 64, j, i, col[i] * sc, col[i + 1] * sc, col[i + 2] * sc, col[i + 3] * sc);
      } else {
#pragma unroll
        for (int i = 0; i < 32; i += 4) put4(S0T, 64, j, i0 + i, col[i], col[i + 1], col[i + 2], col[i + 3]);
      }
    }
    tc_sync();
    if (tid == 0) {  // [dZ S0; dY S0] (cols 128..191) and [E; F] = [U; V] (dS D_L) (cols 256..319)
      mma_tf32_tiles(tmem + 128, sm100::smem_u32(DZY), 128, sm100::smem_u32(S0T), 64, 8, sm100::idesc_tf32(128, 64),
                     false);
      mma_tf32_tiles(tmem + 256, sm100::smem_u32(UV), 128, sm100::smem_u32(DST0), 64, 4, sm100::idesc_tf32(128, 64),
                     false);
      mma_tf32_tiles(tmem + 256, sm100::smem_u32(UV) + 128 * 128, 128, sm100::smem_u32(DST1), 64, 4,
                     sm100::idesc_tf32(128, 64), true);
      sm100::mma_commit(&bars[2]);  // own barrier: both commits may complete before either wait
    }
    second_issued = true;
    WKV_TRACE(35)
    stage = 2;
    ok = wait_all(&bars[1], mph);  // dM
    mph ^= 1;
    if (ok) {
      stage = 3;
      ok = wait_all(&bars[2], 0);  // S0 and dS products (DZY, UV, S0^T, dS^T free after this)
    }
    sm100::tc_fence_after();
  }
  WKV_TRACE(36)
  // dM stage tiles. Stage 1: SA = [dM_ab; dM_rb] (rows t, K = s), SB = [dM_ab^T; dM_ak^T] (rows s, K = t).
  //                 Stage 2: SA = [dM_ak; dM_rk],               SB = [dM_rb^T; dM_rk^T].
  // Thread: row 32 quarter + lane of the 128 rows, columns [32 colh, 32 colh + 32) of each 64-column block.
  const int row = 32 * quarter + (tid & 31), t = row & 63, s0 = 32 * colh;
  const uint32_t trow = tmem + ((uint32_t)(32 * quarter) << 16);
#pragma unroll 1
  for (int stage_ = 0; stage_ < 2 && ok; ++stage_) {
    {
      float d[32];
      const bool lo = row < 64;
      const int lim = lo ? t : t + 1;  // strict for the a~ rows, inclusive for the r~ rows
      sm100::tmem_ld32(trow + (stage_ ? 64 : 0) + s0, d);  // stage 0: dM_ab / dM_rb; stage 1: dM_ak / dM_rk
      sm100::tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 32; u += 4) {
        const int s = s0 + u;
        put4(SA, 128, row, s, s < lim ? d[u] : 0.f, s + 1 < lim ? d[u + 1] : 0.f, s + 2 < lim ? d[u + 2] : 0.f,
             s + 3 < lim ? d[u + 3] : 0.f);
      }
      // transposes: stage 0 from the a~ rows (dM_ab, then dM_ak), stage 1 from the r~ rows (dM_rk, then dM_rb)
      const bool owner = stage_ == 0 ? lo : !lo;
      if (owner) {
#pragma unroll
        for (int u = 0; u < 32; ++u) put1(SB, 128, (stage_ ? 64 : 0) + s0 + u, t, s0 + u < lim ? d[u] : 0.f);
      }
      // warp-collective TMEM load outside the per-row condition
      sm100::tmem_ld32(trow + (stage_ ? 0 : 64) + s0, d);
      sm100::tmem_wait_ld();
      if (owner) {
#pragma unroll
        for (int u = 0; u < 32; ++u) put1(SB, 128, (stage_ ? 0 : 64) + s0 + u, t, s0 + u < lim ? d[u] : 0.f);
      }
    }
    tc_sync();
    if (tid == 0) {
      // [dA~; dR~] += SA . (B~^T | K~^T);  [dB~; dK~] (cols 192..255) (+)= SB . (A~^T | R~^T)
      mma_tf32_tiles(tmem + 128, sm100::smem_u32(SA), 128, sm100::smem_u32(X2T) + stage_ * 16 * KB, 64, 8,
                     sm100::idesc_tf32(128, 64), true);
      mma_tf32_tiles(tmem + 192, sm100::smem_u32(SB), 128, sm100::smem_u32(X1T) + stage_ * 16 * KB, 64, 8,
                     sm100::idesc_tf32(128, 64), stage_ > 0);
      sm100::mma_commit(&bars[1]);
    }
    WKV_TRACE(37 + 2 * stage_)
    stage = 4 + stage_;
    ok = wait_all(&bars[1], mph);
    mph ^= 1;
    sm100::tc_fence_after();
    WKV_TRACE(38 + 2 * stage_)
  }
  if (ok) {
    WKV_TRACE(41)
    // ---- row epilogue: raw gradients and the dLambda terms (thread = row t of its half, 32 columns). The raw input
    // rows are read from the tiles TMA brought at the start (zero past the sequence end), the gradient rows leave
    // as 16-byte stores, and the decay-gradient factor of w is formed here (row-wise) for the column pass.
    const int tg = c * L + t;
    const bool lo = row < 64;  // rows of a~ / b~ (da, db) vs r~ / k~ (dr, dk)
    const bool valid = tg < T;
    const long go = (((long)bb * T + (valid ? tg : 0)) * H + h) * N;
    const uint8_t* src1 = lo ? Ra : Rr;  // a / r
    const uint8_t* src2 = lo ? Rb : Rk;  // b / k
    float* out1 = lo ? da : dr;
    float* out2 = lo ? db : dk;
    const int half = colh;
    {
      float d1[32], d2[32], d3[32], x1[32], x2[32];
      sm100::tmem_ld32(trow + 128 + 32 * half, d1);  // dA~ / dR~
      sm100::tmem_ld32(trow + 192 + 32 * half, d2);  // dB~' / dK~'
      sm100::tmem_ld32(trow + 256 + 32 * half, d3);  // E / F
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        raw8(src1, t, 32 * half + 8 * q, x1 + 8 * q);
        raw8(src2, t, 32 * half + 8 * q, x2 + 8 * q);
      }
      if (lo && valid) {  // w factor of this row: -e^{-1/2} sigmoid(w) (1 - sigmoid(w))
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float wv[8];
          raw8(Rw, t, 32 * half + 8 * q, wv);
#pragma unroll
          for (int u = 0; u < 8; u += 4) {
            float f[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float sg = rt::sigmoidf_(wv[u + e]);
              f[e] = -DECAY_SCALE * sg * (1.f - sg);
            }
            *reinterpret_cast<float4*>(&FW[poff(t, 32 * half + 8 * q + u)]) = make_float4(f[0], f[1], f[2], f[3]);
          }
        }
      }
      sm100::tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 32; u += 4) {
        const int j = 32 * half + u;
        const float4 lt4 = *reinterpret_cast<const float4*>(&lam[poff(t, j)]);
        const float lt[4] = {lt4.x, lt4.y, lt4.z, lt4.w};
        float lp[4] = {0.f, 0.f, 0.f, 0.f};
        if (lo && t > 0) {
          const float4 lp4 = *reinterpret_cast<const float4*>(&lam[poff(t - 1, j)]);
          lp[0] = lp4.x; lp[1] = lp4.y; lp[2] = lp4.z; lp[3] = lp4.w;
        }
        float g1[4], g2[4], pv[4], qv[4], ev[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float up = expf(lo ? lp[e] : lt[e]);  // e^{Lambda_{t-1}} (a) or e^{Lambda_t} (r)
          const float dn = expf(-lt[e]);              // e^{-Lambda_t} (b, k)
          g1[e] = d1[u + e] * up;                     // da / dr
          g2[e] = (d2[u + e] + d3[u + e]) * dn;       // db / dk
          ev[e] = d3[u + e] * x2[u + e] * dn;         // E b~ / F k~
          qv[e] = g1[e] * x1[u + e];                  // da a / dr r
          pv[e] = -g2[e] * x2[u + e];                 // -db b / -dk k
        }
        if (lo) {
          *reinterpret_cast<float4*>(&QA[poff(t, j)]) = make_float4(qv[0], qv[1], qv[2], qv[3]);
          *reinterpret_cast<float4*>(&PB[poff(t, j)]) = make_float4(pv[0], pv[1], pv[2], pv[3]);
          *reinterpret_cast<float4*>(&EA[poff(t, j)]) = make_float4(ev[0], ev[1], ev[2], ev[3]);
        } else {
          *reinterpret_cast<float4*>(&PA[poff(t, j)]) =
              make_float4(qv[0] + pv[0], qv[1] + pv[1], qv[2] + pv[2], qv[3] + pv[3]);
          *reinterpret_cast<float4*>(&EB[poff(t, j)]) = make_float4(ev[0], ev[1], ev[2], ev[3]);
        }
        if (valid) {
          *reinterpret_cast<float4*>(out1 + go + j) = make_float4(g1[0], g1[1], g1[2], g1[3]);
          *reinterpret_cast<float4*>(out2 + go + j) = make_float4(g2[0], g2[1], g2[2], g2[3]);
        }
      }
    }
    __syncthreads();
    WKV_TRACE(42)
    // ---- column pass, key j: threads j + 64 q split every column sum in four parts of 16 steps.
    {
      const int j = tid & 63, q = tid >> 6, r0 = 16 * q;
      const float* dS = wk + WK_DS * MAT;
      float ds[16], sv[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        ds[i] = __ldg(dS + (r0 + i) * N + j);
        sv[i] = __ldg(S0g + (r0 + i) * N + j);
      }
      float acc = 0.f, eacc = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) acc += ds[i] * sv[i];
#pragma unroll
      for (int s2 = 0; s2 < 16; ++s2) eacc += EA[poff(r0 + s2, j)] + EB[poff(r0 + s2, j)];
      // g_t = (dr r - dk k) + (-db b) + (da a)_{t+1} for this thread's 16 steps, as suffix sums
      float g[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int tt = r0 + u;
        g[u] = PA[poff(tt, j)] + PB[poff(tt, j)] + (tt < 63 ? QA[poff(tt + 1, j)] : 0.f);
      }
#pragma unroll
      for (int u = 14; u >= 0; --u) g[u] += g[u + 1];
      colsum[q * 64 + j] = acc * DL[j] + eacc;  // the chunk-end term, in four parts
      colsum[256 + q * 64 + j] = g[0];         // this part's total of g
      __syncthreads();
      // dLogd_t = (sum_i dS S0 D_L + sum_s (E b~ + F k~)) + sum_{t' >= t} g_t'
      float base = colsum[j] + colsum[64 + j] + colsum[128 + j] + colsum[192 + j];
      for (int p2 = q + 1; p2 < 4; ++p2) base += colsum[256 + p2 * 64 + j];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int tgg = c * L + r0 + u;
        if (tgg < T) dw[(((long)bb * T + tgg) * H + h) * N + j] = (g[u] + base) * FW[poff(r0 + u, j)];
      }
    }
  }
  WKV_TRACE(43)
  if (!ok && tid == 0) atomicCAS(&wkv7_tc_bwd_fault_word, 0, 0x400 | stage);  // gradient kernel, failing wait
  if (!ok) {
    if (stage > 1) sm100::mbar_wait_bounded(&bars[1], mph);
    if (second_issued && stage != 3) sm100::mbar_wait_bounded(&bars[2], 0);
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

bool input_map(CUtensorMap* m, const void* base, int B, int T, int H) {
  const uint64_t dims[3] = {(uint64_t)H * N, (uint64_t)T, (uint64_t)B};
  const uint64_t strides[2] = {(uint64_t)H * N * 2, (uint64_t)T * H * N * 2};
  const uint32_t box[3] = {64, 64, 1};
  return tmap::encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box);
}

bool fp32_rows_map(CUtensorMap* m, const float* base, long rows) {
  const uint64_t dims[2] = {64, (uint64_t)rows};
  const uint64_t strides[1] = {64 * 4};
  const uint32_t box[2] = {32, 64};
  return tmap::encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box);
}

}  // namespace

#ifdef WKV7_TC_TRACE
extern "C" void rt_wkv7_tc_bwd_trace(unsigned long long* out, int reset) {
  cudaMemcpyFromSymbol(out, wkv7_trace_ns, sizeof(unsigned long long) * 64);
  if (reset) {
    static unsigned long long zeros[64] = {};
    cudaMemcpyToSymbol(wkv7_trace_ns, zeros, sizeof(zeros));
  }
}
#endif

extern "C" long rt_wkv7_tc_backward_workspace_floats(int B, int T, int H) {
  const long chunks = (T + L - 1) / L;
  return chunks * B * H * WK_MATS * MAT;
}

// Nonzero if a backward kernel gave up a bounded wait since the last call (synchronizes the device):
// 0x200 | wait index for the U/dZ/dV kernel, 0x400 | wait index for the gradient kernel.
extern "C" int rt_wkv7_tc_bwd_fault() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, wkv7_tc_bwd_fault_word, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(wkv7_tc_bwd_fault_word, &zero, sizeof(int));
  return v;
}

// Gradients (fp32 [B, T, H, 64]) of the tcgen05 forward; ckpt and rec as written by rt_wkv7_tc_forward; dy bf16.
extern "C" cudaError_t rt_wkv7_tc_backward(int B, int T, int H, const void* r, const void* w, const void* k,
                                           const void* v, const void* a, const void* b, const float* ckpt,
                                           const float* rec, const void* dy, const float* dend, float* dr, float* dw,
                                           float* dk, float* dv, float* da, float* db, float* ds0, float* work,
                                           cudaStream_t stream) {
  if (B <= 0 || T <= 0 || H <= 0) return cudaErrorInvalidValue;
  const int chunks = (T + L - 1) / L;
  CUtensorMap mr, mw, mk, mv, ma, mb, mdy, mwk;
  bool ok = input_map(&mr, r, B, T, H) && input_map(&mw, w, B, T, H) && input_map(&mk, k, B, T, H) &&
            input_map(&mv, v, B, T, H) && input_map(&ma, a, B, T, H) && input_map(&mb, b, B, T, H) &&
            input_map(&mdy, dy, B, T, H);
  CUtensorMap mrec;
  ok = ok && fp32_rows_map(&mwk, work, (long)B * H * chunks * WK_MATS * N) &&
       fp32_rows_map(&mrec, rec, (long)B * H * chunks * REC_MATS * N);
  if (!ok) return cudaErrorInvalidValue;
  RT_CUDA_CHECK(cudaFuncSetAttribute(wkv7_tc_bscan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BSCAN_SMEM));
  wkv7_tc_bscan_kernel<<<dim3(B * H, N / BS_ROWS), 128, BSCAN_SMEM, stream>>>(
      rec, (const __nv_bfloat16*)dy, dend, work, ds0, T, H, chunks);
  RT_CUDA_CHECK(cudaGetLastError());
  RT_CUDA_CHECK(cudaFuncSetAttribute(wkv7_tc_bwd_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ka::SMEM));
  wkv7_tc_bwd_state_kernel<<<dim3(chunks, H, B), STATE_THREADS, ka::SMEM, stream>>>(mr, mw, mk, mv, ma, mb, mdy, mrec, rec, ckpt, work, dv,
                                                                          T, H, chunks);
  RT_CUDA_CHECK(cudaGetLastError());
  RT_CUDA_CHECK(cudaFuncSetAttribute(wkv7_tc_bwd_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kb::SMEM));
  wkv7_tc_bwd_grad_kernel<<<dim3(chunks, H, B), GRAD_THREADS, kb::SMEM, stream>>>(
      mr, mw, mk, mv, ma, mb, mdy, mwk, (const __nv_bfloat16*)r, (const __nv_bfloat16*)w, (const __nv_bfloat16*)k,
      (const __nv_bfloat16*)a, (const __nv_bfloat16*)b, ckpt, work, dr, dw, dk, da, db, T, H, chunks);
  return cudaGetLastError();
}

// Asynchronous form of the fault read: on `stream`, copy the fault word to `dst` and clear it.
extern "C" cudaError_t rt_wkv7_tc_bwd_fault_async(int* dst, cudaStream_t stream) {
  void* word = nullptr;
  RT_CUDA_CHECK(cudaGetSymbolAddress(&word, wkv7_tc_bwd_fault_word));
  RT_CUDA_CHECK(cudaMemcpyAsync(dst, word, sizeof(int), cudaMemcpyDefault, stream));
  return cudaMemsetAsync(word, 0, sizeof(int), stream);
}
