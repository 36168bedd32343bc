// WKV7 forward on tcgen05 (head size 64, chunks of 64 steps, bf16 inputs, fp32 state), sm_100a.
// The recurrence is RWKV7's (RWKV-LM, Apache-2.0; see NOTICE at the project root); this code is our own.
//
// Per chunk of L = 64 steps with Lambda_t = sum_{tau <= t} log d_tau (per key) and the decayed vectors
// a~ = a e^{Lambda_{t-1}}, r~ = r e^{Lambda_t}, b~ = b e^{-Lambda_s}, k~ = k e^{-Lambda_s}, the chunk matrices
// M_ab = a~.b~ (s < t), M_ak = a~.k~ (s < t), M_rb = r~.b~ (s <= t), M_rk = r~.k~ (s <= t) and
// T = (I - M_ab)^{-1}, the chunk maps its start state S0 (value i x key j) to
//     S_L = S0 G + H0,     y = Q S0^T + Y0,
// with the state-free terms (B^ = b e^{Lambda_L - Lambda_s}, K^ likewise, D_L = e^{Lambda_L})
//     W = T A~,  U0 = T (M_ak V),  G = diag(D_L) + W^T B^,  H0 = U0^T B^ + V^T K^,
//     Q = R~ + M_rb W,  Y0 = M_rk V + M_rb U0.
// Three kernels:
//   1. wkv7_tc_chunk (grid chunks x H x B, parallel): TMA brings the six raw input tiles; the chunk matrices, Z,
//      and the products for Q, Y0, G, H0 are tf32 MMAs into TMEM; W and U0 come from fp32 triangular solves
//      with I - M_ab on the CUDA cores (one right-hand-side column per thread, in registers; T itself is never
//      formed). Writes G, H0, Q, Y0 per chunk.
//   2. wkv7_tc_scan (grid B*H x 8 row blocks): S_{c+1} = S_c G_c + H0_c in fp32 on the CUDA cores, storing the
//      chunk-start states (checkpoints).
//   3. wkv7_tc_out (grid chunk pairs x H x B): y = Q S0^T + Y0, one M = 128 MMA per pair of chunks with Q and S0
//      brought by TMA.
// Every mbarrier wait is bounded; a wait that gives up records the fault word and the CTA unwinds.
#include "wkv7_tc.cuh"
#include "../common/tmap.cuh"

#include <algorithm>

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
constexpr int MAT = N * N;  // floats of one 64 x 64 matrix

// Workspace record per (batch, head, chunk): G, H0, Q, Y0, W, U0 (row-major 64 x 64 fp32 each; W and U0 rounded
// to tf32). The backward forms the chunk's u rows as U = W S0^T + U0 from the last two.
enum { REC_G = 0, REC_H0 = 1, REC_Q = 2, REC_Y0 = 3, REC_W = 4, REC_U0 = 5, REC_MATS = 6 };

// Shared-memory map of the chunk kernel (offsets from a 1024-byte aligned base; tiles are K-major SW128).
// Regions are reused once their last reader is done (noted per line).
constexpr int OFF_RAW = 0;           // six bf16 64 x 64 tiles r, w, k, v, a, b (8 KB each)
constexpr int OFF_LAM = 48 * KB;     // Lambda, plain swizzled 64 x 64 fp32
constexpr int OFF_MISC = 64 * KB;    // mbarriers, TMEM slot, D_L
constexpr int OFF_X1 = 65 * KB;      // [A~; R~] (128 rows) -> [W^T; U0^T]
constexpr int OFF_X2 = 97 * KB;      // [B~; K~] (128 rows) -> [M_ak; M_rk]
constexpr int OFF_VT = 129 * KB;     // V^T (64 rows)
constexpr int OFF_BT = 145 * KB;     // B^T (64 rows)
constexpr int OFF_KT = 161 * KB;     // K^T (64 rows)
constexpr int OFF_MRB = 177 * KB;    // M_rb (64 rows; read as the lower half of a 128-row operand)
constexpr int OFF_MPL = 193 * KB;    // M_ab, plain swizzled (the solves read its rows)
constexpr int OFF_ZT = 209 * KB;     // Z^T, plain swizzled (row i = column i of Z = M_ak V)
constexpr int CHUNK_SMEM = 225 * KB + 1024;
constexpr int CHUNK_TMEM = 512;      // [0,128) chunk matrices, then M_rb [W | U0]; [128,192) [W^T; U0^T] B^;
                                     // [192,256) V^T K^; [256,320) [Z; M_rk V]

__device__ int wkv7_tc_fault_word = 0;

RT_DEVICE uint8_t* align1024(uint8_t* p) { return sm100::align_smem_1024(p); }

// Bounded wait on an MMA/TMA barrier that every thread takes part in; false (uniformly) if it gave up.
RT_DEVICE bool wait_all(uint64_t* bar, uint32_t parity) {
  const bool ok = sm100::mbar_wait_bounded(bar, parity);
  return __syncthreads_and(ok ? 1 : 0) != 0;
}

// 256 threads: warps w and w + 4 share a TMEM lane quarter and split each 64-column block; tile phases split
// their rows or columns the same way. The solves keep one right-hand-side column per thread on the first 128
// threads (A~ columns on threads 64..127, Z columns on threads 0..63).
constexpr int CHUNK_THREADS = 256;

__global__ void __launch_bounds__(CHUNK_THREADS, 1)
wkv7_tc_chunk_kernel(const __grid_constant__ CUtensorMap m_r, const __grid_constant__ CUtensorMap m_w,
                     const __grid_constant__ CUtensorMap m_k, const __grid_constant__ CUtensorMap m_v,
                     const __grid_constant__ CUtensorMap m_a, const __grid_constant__ CUtensorMap m_b, int T,
                     int H, int chunks, float* __restrict__ ws) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const int c = blockIdx.x, h = blockIdx.y, bb = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int quarter = warp & 3, colh = warp >> 2;
  uint8_t* Rr = sm + OFF_RAW;
  uint8_t* Rw = Rr + 8 * KB;
  uint8_t* Rk = Rr + 16 * KB;
  uint8_t* Rv = Rr + 24 * KB;
  uint8_t* Ra = Rr + 32 * KB;
  uint8_t* Rb = Rr + 40 * KB;
  float* lam = reinterpret_cast<float*>(sm + OFF_LAM);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_MISC);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_MISC + 16);
  float* DL = reinterpret_cast<float*>(sm + OFF_MISC + 64);
  uint8_t *X1 = sm + OFF_X1, *X2 = sm + OFF_X2, *VT = sm + OFF_VT, *BT = sm + OFF_BT, *KT = sm + OFF_KT;
  uint8_t* MRB = sm + OFF_MRB;
  float* MPL = reinterpret_cast<float*>(sm + OFF_MPL);
  float* ZT = reinterpret_cast<float*>(sm + OFF_ZT);
  float* carry = ZT;  // Lambda carries (before Z^T is written)
  uint8_t* MAK = X2;
  uint8_t* WUT = X1;
  float* rec = ws + (((long)bb * H + h) * chunks + c) * (REC_MATS * MAT);
  const uint32_t trow = (uint32_t)(32 * quarter) << 16;  // this warp's TMEM lane quarter
  const int row = 32 * quarter + (tid & 31);             // its TMEM lane (row of a 128-row result)
  WKV_TRACE_BEGIN

  if (tid == 0) {
    sm100::mbar_init(&bars[0], 1);
    sm100::mbar_init(&bars[1], 1);
    sm100::fence_barrier_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tslot, CHUNK_TMEM);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    sm100::mbar_expect_tx(&bars[0], 6 * 8192);
    const int x = h * N, y = c * L;
    sm100::tma_load_3d(Rr, &m_r, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rw, &m_w, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rk, &m_k, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rv, &m_v, &bars[0], x, y, bb);
    sm100::tma_load_3d(Ra, &m_a, &bars[0], x, y, bb);
    sm100::tma_load_3d(Rb, &m_b, &bars[0], x, y, bb);
  }
  int stage = 1;  // which wait a failure happened at (recorded in the fault word)
  bool ok = wait_all(&bars[0], 0);
  WKV_TRACE(0)
  uint32_t mph = 0;  // parity of the next MMA-barrier completion
  const int nvalid = min(L, T - c * L);

  if (ok) {
    build_lambda_nt<CHUNK_THREADS>(Rw, lam, carry, nvalid, tid);
    if (tid < 64) DL[tid] = expf(lam[poff(63, tid)]);
    WKV_TRACE(1)
    // ---- phase-A tiles. X1 row r: A~ (r < 64) / R~; X2 row r: B~ / K~ (thread: row r = tid % 128, 32 keys).
    {
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
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          x1[q] *= expf(hi ? lt[q] : lp[q]);
          x2[q] *= expf(-lt[q]);
        }
        put4(X1, 128, r, j0, x1[0], x1[1], x1[2], x1[3]);
        put4(X1, 128, r, j0 + 4, x1[4], x1[5], x1[6], x1[7]);
        put4(X2, 128, r, j0, x2[0], x2[1], x2[2], x2[3]);
        put4(X2, 128, r, j0 + 4, x2[4], x2[5], x2[6], x2[7]);
      }
    }
    WKV_TRACE(2)
    // V^T rows i (16 steps per thread); B^T / K^T rows j: x[s][j] e^{Lambda_L - Lambda_s} (32 steps per thread)
    {
      const int j = tid & 63;
      {
        const int s0 = 16 * (tid >> 6);
        float x[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) x[q] = raw(Rv, s0 + q, j);
#pragma unroll
        for (int q = 0; q < 16; q += 4) put4(VT, 64, j, s0 + q, x[q], x[q + 1], x[q + 2], x[q + 3]);
      }
      const bool kt = (tid & 64) != 0;
      const uint8_t* src = kt ? Rk : Rb;
      uint8_t* dst = kt ? KT : BT;
      const float lL = lam[poff(63, j)];
      const int s1 = 32 * (tid >> 7);
#pragma unroll 1
      for (int s0 = s1; s0 < s1 + 32; s0 += 16) {  // loads first, then exponentials, then stores
        float x[16], ls[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          x[q] = raw(src, s0 + q, j);
          ls[q] = lam[poff(s0 + q, j)];
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) x[q] *= expf(lL - ls[q]);
#pragma unroll
        for (int q = 0; q < 16; q += 4) put4(dst, 64, j, s0 + q, x[q], x[q + 1], x[q + 2], x[q + 3]);
      }
    }
    tc_sync();
    WKV_TRACE(3)
    // ---- MMA1: [M_ab M_ak; M_rb M_rk] = [A~; R~] [B~; K~]^T  (TMEM cols 0..127)
    if (tid == 0) {
      mma_tf32_tiles(tmem, sm100::smem_u32(X1), 128, sm100::smem_u32(X2), 128, 8, sm100::idesc_tf32(128, 128),
                     false);
      sm100::mma_commit(&bars[1]);
    }
    stage = 2;
    ok = wait_all(&bars[1], mph);
    mph ^= 1;
    sm100::tc_fence_after();
  }
  if (ok) {
    WKV_TRACE(4)
    // ---- epilogue 1 (32 columns of each block per thread): masks; M_ab -> MPL (plain), [M_ak; M_rk] -> MAK,
    //      M_rb -> MRB
    {
      float d[32];
      const int t = row & 63, s0 = 32 * colh;
      sm100::tmem_ld32(tmem + trow + s0, d);
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
        for (int u = 0; u < 32; u += 4) {
          const int s = s0 + u;
          put4(MRB, 64, t, s, s <= t ? d[u] : 0.f, s + 1 <= t ? d[u + 1] : 0.f, s + 2 <= t ? d[u + 2] : 0.f,
               s + 3 <= t ? d[u + 3] : 0.f);
        }
      }
      sm100::tmem_ld32(tmem + trow + 64 + s0, d);
      sm100::tmem_wait_ld();
      const int lim = row < 64 ? t : t + 1;  // strict for M_ak, inclusive for M_rk
#pragma unroll
      for (int u = 0; u < 32; u += 4) {
        const int s = s0 + u;
        put4(MAK, 128, row, s, s < lim ? d[u] : 0.f, s + 1 < lim ? d[u + 1] : 0.f, s + 2 < lim ? d[u + 2] : 0.f,
             s + 3 < lim ? d[u + 3] : 0.f);
      }
    }
    tc_sync();
    // ---- MMA2: [Z; M_rk V] = [M_ak; M_rk] V  (cols 256..319)
    if (tid == 0) {
      mma_tf32_tiles(tmem + 256, sm100::smem_u32(MAK), 128, sm100::smem_u32(VT), 64, 8, sm100::idesc_tf32(128, 64),
                     false);
      sm100::mma_commit(&bars[1]);
    }
    WKV_TRACE(5)
  }
  // Right-hand sides of the solves, one column per thread: A~ column j (threads 64 + j, built while MMA2 runs)
  // and Z column i (threads i < 64, from Z^T after MMA2).
  float x[64];
  if (ok && tid >= 64 && tid < 128) {
    const int j = tid - 64;
#pragma unroll
    for (int t = 0; t < 64; ++t) x[t] = raw(Ra, t, j);
#pragma unroll
    for (int t = 1; t < 64; ++t) x[t] *= expf(lam[poff(t - 1, j)]);
  }
  if (ok) {
    stage = 3;
    ok = wait_all(&bars[1], mph);  // MMA2 done
    mph ^= 1;
    sm100::tc_fence_after();
  }
  if (ok) {
    WKV_TRACE(6)
    if (quarter < 2) {  // Z row t -> column t of Z^T (32 columns per thread)
      float d[32];
      sm100::tmem_ld32(tmem + trow + 256 + 32 * colh, d);
      sm100::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) ZT[poff(32 * colh + i, row)] = d[i];
    }
    __syncthreads();
    if (tid < 64) {
#pragma unroll
      for (int t = 0; t < 64; t += 4) {
        const float4 z = *reinterpret_cast<const float4*>(&ZT[poff(tid, t)]);
        x[t] = z.x;
        x[t + 1] = z.y;
        x[t + 2] = z.z;
        x[t + 3] = z.w;
      }
    }
    WKV_TRACE(7)
    // ---- W = T A~ (threads 64 + j: column j) and U0 = T Z (threads i: column i), T = (I - M_ab)^{-1}; the
    //      columns become the rows of [W^T; U0^T] (X1's [A~; R~] was last read by MMA1)
    if (tid < 128) {
      solve_lower(MPL, x);
      WKV_TRACE(11)
      const int wrow = tid < 64 ? 64 + tid : tid - 64;
#pragma unroll
      for (int t = 0; t < 64; t += 4) put4(WUT, 128, wrow, t, x[t], x[t + 1], x[t + 2], x[t + 3]);
    }
    tc_sync();
    WKV_TRACE(8)
    // ---- MMA3: M_rb [W | U0] (cols 0..127, rows 64..127 from M_rb read as the lower half of 128 rows),
    //      [W^T; U0^T] B^ (cols 128..191), V^T K^ (cols 192..255, rows 64..127 likewise)
    if (tid == 0) {
      mma_tf32_tiles(tmem, sm100::smem_u32(MRB) - 8192, 64, sm100::smem_u32(WUT), 128, 8,
                     sm100::idesc_tf32(128, 128), false);
      mma_tf32_tiles(tmem + 128, sm100::smem_u32(WUT), 128, sm100::smem_u32(BT), 64, 8, sm100::idesc_tf32(128, 64),
                     false);
      mma_tf32_tiles(tmem + 192, sm100::smem_u32(VT) - 8192, 64, sm100::smem_u32(KT), 64, 8,
                     sm100::idesc_tf32(128, 64), false);
      sm100::mma_commit(&bars[1]);
    }
    {  // while MMA3 runs: W and U0 rows to the record, read out of [W^T; U0^T] (row t, 32 columns per thread)
      const int t = tid & 63, part = tid >> 6;  // parts: W cols 0..31, 32..63, U0 cols 0..31, 32..63
      const int base = part < 2 ? 0 : 64, c0 = 32 * (part & 1);
      float* g = rec + (part < 2 ? REC_W : REC_U0) * MAT + t * 64 + c0;
#pragma unroll
      for (int u = 0; u < 32; u += 4)
        *reinterpret_cast<float4*>(g + u) =
            make_float4(get1(WUT, 128, base + c0 + u, t), get1(WUT, 128, base + c0 + u + 1, t),
                        get1(WUT, 128, base + c0 + u + 2, t), get1(WUT, 128, base + c0 + u + 3, t));
    }
    stage = 4;
    ok = wait_all(&bars[1], mph);
    mph ^= 1;
    sm100::tc_fence_after();
  }
  if (ok) {
    WKV_TRACE(9)
    const int half = colh;
    if (row < 64) {  // G = diag(D_L) + W^T B^ (row j = row; 32 columns per thread)
      const int r = row;
      float d[32];
      sm100::tmem_ld32(tmem + trow + 128 + 32 * half, d);
      sm100::tmem_wait_ld();
      float* g = rec + REC_G * MAT + r * 64 + 32 * half;
#pragma unroll
      for (int u = 0; u < 32; ++u) d[u] += 32 * half + u == r ? DL[r] : 0.f;
#pragma unroll
      for (int u = 0; u < 32; u += 4) *reinterpret_cast<float4*>(g + u) = make_float4(d[u], d[u + 1], d[u + 2], d[u + 3]);
    } else {  // row t = row - 64: Q = R~ + M_rb W (tf32: an MMA operand later), Y0 = M_rk V + M_rb U0,
              // H0 = U0^T B^ + V^T K^ (row i = t)
      const int t = row - 64;
      float d[32], e[32];
      sm100::tmem_ld32(tmem + trow + 32 * half, d);
      sm100::tmem_wait_ld();
      float* gq = rec + REC_Q * MAT + t * 64 + 32 * half;
#pragma unroll
      for (int j8 = 0; j8 < 32; j8 += 8) {
        float xr[8], lt[8], q[8];
        raw8(Rr, t, 32 * half + j8, xr);
        *reinterpret_cast<float4*>(lt) = *reinterpret_cast<const float4*>(&lam[poff(t, 32 * half + j8)]);
        *reinterpret_cast<float4*>(lt + 4) = *reinterpret_cast<const float4*>(&lam[poff(t, 32 * half + j8 + 4)]);
#pragma unroll
        for (int u = 0; u < 8; ++u) q[u] = tf32r(xr[u] * expf(lt[u]) + d[j8 + u]);
        *reinterpret_cast<float4*>(gq + j8) = make_float4(q[0], q[1], q[2], q[3]);
        *reinterpret_cast<float4*>(gq + j8 + 4) = make_float4(q[4], q[5], q[6], q[7]);
      }
      sm100::tmem_ld32(tmem + trow + 64 + 32 * half, d);
      sm100::tmem_ld32(tmem + trow + 256 + 32 * half, e);
      sm100::tmem_wait_ld();
      float* gy = rec + REC_Y0 * MAT + t * 64 + 32 * half;
#pragma unroll
      for (int u = 0; u < 32; u += 4)
        *reinterpret_cast<float4*>(gy + u) = make_float4(d[u] + e[u], d[u + 1] + e[u + 1], d[u + 2] + e[u + 2],
                                                         d[u + 3] + e[u + 3]);
      sm100::tmem_ld32(tmem + trow + 128 + 32 * half, d);
      sm100::tmem_ld32(tmem + trow + 192 + 32 * half, e);
      sm100::tmem_wait_ld();
      float* gh = rec + REC_H0 * MAT + t * 64 + 32 * half;
#pragma unroll
      for (int u = 0; u < 32; u += 4)
        *reinterpret_cast<float4*>(gh + u) = make_float4(d[u] + e[u], d[u + 1] + e[u + 1], d[u + 2] + e[u + 2],
                                                         d[u + 3] + e[u + 3]);
    }
  }
  WKV_TRACE(10)
  if (!ok && tid == 0) atomicCAS(&wkv7_tc_fault_word, 0, 0x100 | stage);  // kernel 1, failing wait
  if (!ok && stage > 1) sm100::mbar_wait_bounded(&bars[1], mph);  // an MMA may still be in flight
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, CHUNK_TMEM);
  }
}

// ---------------------------------------------------------------- 2: serial chunk scan S <- S G + H0
constexpr int SCAN_ROWS = 8;
__global__ void __launch_bounds__(128)
wkv7_tc_scan_kernel(const float* __restrict__ ws, const float* __restrict__ s0, float* __restrict__ ckpt,
                    float* __restrict__ s_end, int chunks) {
  __shared__ __align__(16) float G[2][MAT];
  __shared__ __align__(16) float H[2][SCAN_ROWS][N];
  __shared__ __align__(16) float S[SCAN_ROWS][N];
  const int bh = blockIdx.x, rb = blockIdx.y * SCAN_ROWS, tid = threadIdx.x;
  const int r = tid >> 4, j0 = 4 * (tid & 15);
  const float* rec0 = ws + (long)bh * chunks * REC_MATS * MAT;
  auto prefetch = [&](int c) {  // G_c and this block's rows of H0_c, one group
    const float* src = rec0 + (long)c * REC_MATS * MAT + REC_G * MAT;
    float* dst = G[c & 1];
    for (int e = tid; e < MAT / 4; e += 128) rt::cp_async16(dst + 4 * e, src + 4 * e, true);
    rt::cp_async16(&H[c & 1][r][j0], rec0 + (long)c * REC_MATS * MAT + REC_H0 * MAT + (long)(rb + r) * N + j0, true);
    rt::cp_async_commit();
  };
  prefetch(0);
  float4 s = *reinterpret_cast<const float4*>(s0 + ((long)bh * N + rb + r) * N + j0);
  *reinterpret_cast<float4*>(&S[r][j0]) = s;
  float* ck = ckpt + (long)bh * (chunks + 1) * MAT + (long)(rb + r) * N + j0;
#pragma unroll 1
  for (int c = 0; c < chunks; ++c) {
    *reinterpret_cast<float4*>(ck + (long)c * MAT) = s;
    rt::cp_async_wait<0>();
    __syncthreads();  // G_c and H0_c landed, S visible, buffers (c + 1) & 1 no longer read
    float4 acc = *reinterpret_cast<const float4*>(&H[c & 1][r][j0]);
    if (c + 1 < chunks) prefetch(c + 1);
    const float* g = G[c & 1];
#pragma unroll 8
    for (int j = 0; j < N; ++j) {
      const float sv = S[r][j];
      const float4 gv = *reinterpret_cast<const float4*>(g + j * N + j0);
      acc.x += sv * gv.x;
      acc.y += sv * gv.y;
      acc.z += sv * gv.z;
      acc.w += sv * gv.w;
    }
    __syncthreads();
    *reinterpret_cast<float4*>(&S[r][j0]) = acc;
    s = acc;
  }
  *reinterpret_cast<float4*>(ck + (long)chunks * MAT) = s;
  *reinterpret_cast<float4*>(s_end + ((long)bh * N + rb + r) * N + j0) = s;
}

// ---------------------------------------------------------------- 3: y = Q S0^T + Y0 for a pair of chunks
// A = [Q_c0; Q_c1] (rows t), B = [S0_c0; S0_c1] (rows i), both K = 64 keys, brought by TMA as K-major SW128 atoms
// (box 32 x 64 fp32). The diagonal 64 x 64 blocks of the 128 x 128 product are the two chunks' Q S0^T.
constexpr int OUT_SMEM = 64 * KB + 1024 + 1024;
__global__ void __launch_bounds__(128)
wkv7_tc_out_kernel(const __grid_constant__ CUtensorMap m_q, const __grid_constant__ CUtensorMap m_s,
                   const float* __restrict__ ws, __nv_bfloat16* __restrict__ y, int T, int H, int chunks) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* A = sm;
  uint8_t* Bt = sm + 32 * KB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + 64 * KB);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + 64 * KB + 16);
  const int h = blockIdx.y, bb = blockIdx.z, tid = threadIdx.x, warp = tid >> 5;
  const int c0 = 2 * blockIdx.x, c1 = min(c0 + 1, chunks - 1);
  const long bh = (long)bb * H + h;
  if (tid == 0) {
    sm100::mbar_init(&bars[0], 1);
    sm100::mbar_init(&bars[1], 1);
    sm100::fence_barrier_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tslot, 128);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    sm100::mbar_expect_tx(&bars[0], 64 * KB);
    const int cs[2] = {c0, c1};
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int qrow = (int)(((bh * chunks + cs[p]) * REC_MATS + REC_Q) * N);
      const int srow = (int)((bh * (chunks + 1) + cs[p]) * N);
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        sm100::tma_load_2d(A + a * 16 * KB + p * 8 * KB, &m_q, &bars[0], 32 * a, qrow);
        sm100::tma_load_2d(Bt + a * 16 * KB + p * 8 * KB, &m_s, &bars[0], 32 * a, srow);
      }
    }
  }
  bool ok = wait_all(&bars[0], 0);
  int stage = ok ? 2 : 1;
  if (ok && tid == 0) {
    sm100::tc_fence_after();
    mma_tf32_tiles(tmem, sm100::smem_u32(A), 128, sm100::smem_u32(Bt), 128, 8, sm100::idesc_tf32(128, 128), false);
    sm100::mma_commit(&bars[1]);
  }
  if (ok) ok = wait_all(&bars[1], 0);
  sm100::tc_fence_after();
  const int p = tid >> 6, t = tid & 63, cc = p ? c1 : c0, tg = cc * L + t;
  const bool store = !(p == 1 && c1 == c0) && tg < T;
  if (ok) {  // tcgen05.ld is warp-collective: every lane loads, only rows inside the sequence store
    const uint32_t row = tmem + ((uint32_t)(32 * warp) << 16) + 64 * p;
    const float* y0 = ws + ((bh * chunks + cc) * REC_MATS + REC_Y0) * MAT + t * N;
    __nv_bfloat16* out = y + (((long)bb * T + (store ? tg : 0)) * H + h) * N;
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      float d[32];
      sm100::tmem_ld32(row + 32 * half, d);
      sm100::tmem_wait_ld();
      if (!store) continue;
#pragma unroll
      for (int u = 0; u < 32; u += 8) {
        float v[8];
        const float4 a4 = __ldg(reinterpret_cast<const float4*>(y0 + 32 * half + u));
        const float4 b4 = __ldg(reinterpret_cast<const float4*>(y0 + 32 * half + u + 4));
        v[0] = d[u] + a4.x; v[1] = d[u + 1] + a4.y; v[2] = d[u + 2] + a4.z; v[3] = d[u + 3] + a4.w;
        v[4] = d[u + 4] + b4.x; v[5] = d[u + 5] + b4.y; v[6] = d[u + 6] + b4.z; v[7] = d[u + 7] + b4.w;
        *reinterpret_cast<uint4*>(out + 32 * half + u) = rt::pack8(v);
      }
    }
  }
  if (!ok && tid == 0) atomicCAS(&wkv7_tc_fault_word, 0, 0x300 | stage);  // kernel 3, failing wait
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 128);
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

// Floats of the per-chunk record workspace (G, H0, Q, Y0, W, U0 per chunk and head). The backward reads G, Q, W
// and U0.
#ifdef WKV7_TC_TRACE
extern "C" void rt_wkv7_tc_fwd_trace(unsigned long long* out, int reset) {
  cudaMemcpyFromSymbol(out, wkv7_trace_ns, sizeof(unsigned long long) * 64);
  if (reset) {
    static unsigned long long zeros[64] = {};
    cudaMemcpyToSymbol(wkv7_trace_ns, zeros, sizeof(zeros));
  }
}
#endif

extern "C" long rt_wkv7_tc_workspace_floats(int B, int T, int H) {
  const long chunks = (T + L - 1) / L;
  return chunks * B * H * REC_MATS * MAT;
}

extern "C" int rt_wkv7_tc_chunk_len() { return L; }

// Nonzero if a tcgen05 WKV7 forward kernel gave up a bounded wait since the last call (synchronizes the device):
// 0x100 | wait index for the chunk kernel, 0x300 | wait index for the output kernel (first failure recorded).
extern "C" int rt_wkv7_tc_fault() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, wkv7_tc_fault_word, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(wkv7_tc_fault_word, &zero, sizeof(int));
  return v;
}

// bf16 inputs [B, T, H, 64]; s0 [B, H, 64, 64] fp32; y [B, T, H, 64] bf16; s_end [B, H, 64, 64];
// ckpt [B, H, chunks + 1, 64, 64] (chunk-start states, then the final state); ws: rt_wkv7_tc_workspace_floats.
extern "C" cudaError_t rt_wkv7_tc_forward(int B, int T, int H, const void* r, const void* w, const void* k,
                                          const void* v, const void* a, const void* b, const float* s0, void* y,
                                          float* s_end, float* ckpt, float* ws, cudaStream_t stream) {
  if (B <= 0 || T <= 0 || H <= 0) return cudaErrorInvalidValue;
  const int chunks = (T + L - 1) / L;
  CUtensorMap mr, mw, mk, mv, ma, mb, mq, ms;
  bool ok = input_map(&mr, r, B, T, H) && input_map(&mw, w, B, T, H) && input_map(&mk, k, B, T, H) &&
            input_map(&mv, v, B, T, H) && input_map(&ma, a, B, T, H) && input_map(&mb, b, B, T, H);
  ok = ok && fp32_rows_map(&mq, ws, (long)B * H * chunks * REC_MATS * N) &&
       fp32_rows_map(&ms, ckpt, (long)B * H * (chunks + 1) * N);
  if (!ok) return cudaErrorInvalidValue;
  RT_CUDA_CHECK(cudaFuncSetAttribute(wkv7_tc_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CHUNK_SMEM));
  wkv7_tc_chunk_kernel<<<dim3(chunks, H, B), CHUNK_THREADS, CHUNK_SMEM, stream>>>(mr, mw, mk, mv, ma, mb, T, H, chunks, ws);
  RT_CUDA_CHECK(cudaGetLastError());
  wkv7_tc_scan_kernel<<<dim3(B * H, N / SCAN_ROWS), 128, 0, stream>>>(ws, s0, ckpt, s_end, chunks);
  RT_CUDA_CHECK(cudaGetLastError());
  RT_CUDA_CHECK(cudaFuncSetAttribute(wkv7_tc_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, OUT_SMEM));
  wkv7_tc_out_kernel<<<dim3((chunks + 1) / 2, H, B), 128, OUT_SMEM, stream>>>(mq, ms, ws, (__nv_bfloat16*)y, T, H,
                                                                             chunks);
  return cudaGetLastError();
}

// Asynchronous form of the fault read: on `stream`, copy the fault word to `dst` and clear it.
extern "C" cudaError_t rt_wkv7_tc_fault_async(int* dst, cudaStream_t stream) {
  void* word = nullptr;
  RT_CUDA_CHECK(cudaGetSymbolAddress(&word, wkv7_tc_fault_word));
  RT_CUDA_CHECK(cudaMemcpyAsync(dst, word, sizeof(int), cudaMemcpyDefault, stream));
  return cudaMemsetAsync(word, 0, sizeof(int), stream);
}
