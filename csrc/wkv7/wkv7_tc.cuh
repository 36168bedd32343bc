// Shared pieces of the tcgen05 WKV7 kernels (head size 64, chunks of 64 steps, bf16 inputs).
// The recurrence is RWKV7's (RWKV-LM, Apache-2.0; see NOTICE at the project root); this code is our own.
//
// Operand tiles are fp32 words in shared memory read by tcgen05.mma kind::tf32 (K = 8 per instruction):
// K-major with the 128-byte swizzle, i.e. for a tile of `rows` rows the K extent is split into atoms of 32
// words, atom a holds rows x 128 bytes, and the 16-byte chunk q of row r sits at chunk q ^ (r % 8). Values
// written by threads are rounded to tf32 (round to nearest) so that the tensor core's truncation of the low
// mantissa bits does not bias the products.
//
// Raw bf16 input tiles arrive by TMA (3-D map over [B][T][H * 64], box 64 x 64 x 1, 128-byte swizzle): element
// (t, j) of a tile sits at t * 128 + (((j / 8) ^ (t % 8)) * 16) + (j % 8) * 2. Rows past the sequence end are
// zero-filled by the TMA unit.
#pragma once
#include "../common/common.cuh"
#include "../common/sm100.cuh"

namespace wtc {

constexpr int N = 64;                           // head size
constexpr int L = 64;                           // chunk length
constexpr float DECAY_SCALE = 0.6065306597126334f;  // log d = -e^{-1/2} sigmoid(w)

RT_DEVICE float tf32r(float x) {
  uint32_t u;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u) : "f"(x));
  return __uint_as_float(u);
}

// Byte offset of element (r, k) in a K-major SW128 fp32 tile of `rows` rows.
RT_DEVICE uint32_t koff(int rows, int r, int k) {
  return (uint32_t)((k >> 5) * rows * 128 + r * 128 + ((((k & 31) >> 2) ^ (r & 7)) << 4) + ((k & 3) << 2));
}
RT_DEVICE void put1(uint8_t* tile, int rows, int r, int k, float v) {
  *reinterpret_cast<float*>(tile + koff(rows, r, k)) = tf32r(v);
}
// Four consecutive k (k % 4 == 0) of row r.
RT_DEVICE void put4(uint8_t* tile, int rows, int r, int k, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(tile + koff(rows, r, k)) = make_float4(tf32r(a), tf32r(b), tf32r(c), tf32r(d));
}
RT_DEVICE float get1(const uint8_t* tile, int rows, int r, int k) {
  return *reinterpret_cast<const float*>(tile + koff(rows, r, k));
}

// Element (t, j) of a raw bf16 64 x 64 tile loaded by TMA with the 128-byte swizzle.
RT_DEVICE float raw(const uint8_t* tile, int t, int j) {
  const uint32_t off = t * 128 + ((((j >> 3) ^ (t & 7))) << 4) + ((j & 7) << 1);
  return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(tile + off));
}
// Eight consecutive j (j % 8 == 0) of row t.
RT_DEVICE void raw8(const uint8_t* tile, int t, int j, float* out) {
  const uint32_t off = t * 128 + ((((j >> 3) ^ (t & 7))) << 4);
  rt::unpack8(*reinterpret_cast<const uint4*>(tile + off), out);
}

// Plain 64 x 64 fp32 matrix with 16-byte chunks swizzled by row (chunk q of row t at q ^ (t % 16)): row-wise
// float4 access by one thread per row and column-wise scalar access by one thread per column are both free of
// bank conflicts.
RT_DEVICE int poff(int t, int j) { return t * 64 + ((((j >> 2) ^ (t & 15))) << 2) + (j & 3); }

// D (+)= A . B^T over `ksteps` K-steps of 8 (tf32), A of a_rows rows and B of b_rows rows (tile layouts above).
// Issued by one thread.
RT_DEVICE void mma_tf32_tiles(uint32_t tmem_d, uint32_t a, int a_rows, uint32_t b, int b_rows, int ksteps,
                              uint32_t idesc, bool accumulate) {
#pragma unroll 1
  for (int ks = 0; ks < ksteps; ++ks) {
    const uint32_t ao = a + (ks >> 2) * a_rows * 128 + (ks & 3) * 32;
    const uint32_t bo = b + (ks >> 2) * b_rows * 128 + (ks & 3) * 32;
    sm100::mma_tf32(tmem_d, sm100::smem_desc(ao, 16, 1024), sm100::smem_desc(bo, 16, 1024), idesc,
                    (accumulate || ks > 0) ? 1u : 0u);
  }
}

RT_DEVICE void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Make this thread's shared-memory writes visible to the tensor core and order TMEM accesses around a barrier.
RT_DEVICE void tc_sync() {
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
}

// 64 columns [col, col + 64) of this warp's TMEM lane (thread = lane) into v.
RT_DEVICE void tmem_row64(uint32_t tmem, int warp, int col, float (&v)[64]) {
  const uint32_t addr = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + col;
  sm100::tmem_ld32(addr, *reinterpret_cast<float(*)[32]>(v));
  sm100::tmem_ld32(addr + 32, *reinterpret_cast<float(*)[32]>(v + 32));
  sm100::tmem_wait_ld();
}

// Lambda_t[j] = sum_{tau <= t} log d_tau[j] (plain swizzled 64 x 64 in `lam`) from the raw w tile, 128 threads:
// thread j and 64 + j take steps [0, 32) and [32, 64) of column j. Loads and sigmoids are independent (staged in
// registers); only the running sum is serial. Steps at or past `nvalid` have log d = 0. Ends with a barrier.
RT_DEVICE void build_lambda(const uint8_t* Rw, float* lam, float* carry, int nvalid, int tid) {
  const int j = tid & 63, half = tid >> 6, t0 = 32 * half;
  float v[32];
#pragma unroll
  for (int u = 0; u < 32; ++u) v[u] = raw(Rw, t0 + u, j);
#pragma unroll
  for (int u = 0; u < 32; ++u) v[u] = t0 + u < nvalid ? -DECAY_SCALE * rt::sigmoidf_(v[u]) : 0.f;
#pragma unroll
  for (int u = 1; u < 32; ++u) v[u] += v[u - 1];
  if (half == 0) carry[j] = v[31];
  __syncthreads();
  const float base = half ? carry[j] : 0.f;
#pragma unroll
  for (int u = 0; u < 32; ++u) lam[poff(t0 + u, j)] = v[u] + base;
  __syncthreads();
}

// build_lambda for NT threads (NT = 128 or 256): thread j + 64 p takes steps [S p, S p + S), S = 4096 / NT, of
// column j. `carry` holds NT floats (the parts' totals). Ends with a barrier.
template <int NT>
RT_DEVICE void build_lambda_nt(const uint8_t* Rw, float* lam, float* carry, int nvalid, int tid) {
  constexpr int S = 64 * 64 / NT;
  const int j = tid & 63, part = tid >> 6, t0 = S * part;
  float v[S];
#pragma unroll
  for (int u = 0; u < S; ++u) v[u] = raw(Rw, t0 + u, j);
#pragma unroll
  for (int u = 0; u < S; ++u) v[u] = t0 + u < nvalid ? -DECAY_SCALE * rt::sigmoidf_(v[u]) : 0.f;
#pragma unroll
  for (int u = 1; u < S; ++u) v[u] += v[u - 1];
  carry[part * 64 + j] = v[S - 1];
  __syncthreads();
  float base = 0.f;
  for (int q = 0; q < part; ++q) base += carry[q * 64 + j];
#pragma unroll
  for (int u = 0; u < S; ++u) lam[poff(t0 + u, j)] = v[u] + base;
  __syncthreads();
}

// Triangular solves with the strictly lower 64 x 64 chunk matrix M (plain swizzled rows in `mpl`, zero on and
// above the diagonal), one right-hand side per thread held in registers. Every thread reads the same M entries
// (broadcast float4 loads). With one warp per scheduler the loads' latency is not hidden by other warps, so the
// row needed next is loaded into registers while the current row's products run (explicit double buffer); all
// loops unroll, so x and the buffers stay in registers.
// Shared-space address of M for the solves. The empty volatile asm pins the point where the address is taken
// (after the barrier that published M), so the loads below, which depend on it, cannot be hoisted above it.
RT_DEVICE uint32_t shared_base(const float* p) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("" : "+r"(a));
  return a;
}
// 16-byte shared load of M[t][4g .. 4g+3] (an explicit ld.shared: the plain pointer reaches here through integer
// alignment arithmetic, which hides its address space from the compiler).
RT_DEVICE float4 mrow4(uint32_t mpl, int t, int g) {
  float4 v;
  asm("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "r"(mpl + 4u * (uint32_t)poff(t, 4 * g)));
  return v;
}

// x <- (I - M)^{-1} x: forward substitution, left-looking: x_t += sum_{s < t} M[t][s] x_s (four partial sums).
RT_DEVICE void solve_lower(const float* mpl_ptr, float (&x)[64]) {
  const uint32_t mpl = shared_base(mpl_ptr);
  float4 cur[16], nxt[16];
  cur[0] = mrow4(mpl, 1, 0);
#pragma unroll
  for (int t = 1; t < 64; ++t) {
    const int n = (t + 3) >> 2;  // float4 groups holding M[t][0..t-1]
    if (t + 1 < 64) {
#pragma unroll
      for (int g = 0; g < ((t + 4) >> 2); ++g) nxt[g] = mrow4(mpl, t + 1, g);
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int g = 0; g < n; ++g) {
      const int s = 4 * g;
      acc[0] += cur[g].x * x[s];
      if (s + 1 < t) acc[1] += cur[g].y * x[s + 1];
      if (s + 2 < t) acc[2] += cur[g].z * x[s + 2];
      if (s + 3 < t) acc[3] += cur[g].w * x[s + 3];
    }
    x[t] += (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
    for (int g = 0; g < 16; ++g) cur[g] = nxt[g];
  }
}

// x <- (I - M)^{-T} x: back substitution, right-looking from the last row: once x_t is final,
// x_s += M[t][s] x_t for every s < t (independent updates).
RT_DEVICE void solve_upper_t(const float* mpl_ptr, float (&x)[64]) {
  const uint32_t mpl = shared_base(mpl_ptr);
  float4 cur[16], nxt[16];
#pragma unroll
  for (int g = 0; g < 16; ++g) cur[g] = mrow4(mpl, 63, g);
#pragma unroll
  for (int t = 63; t >= 1; --t) {
    if (t > 1) {
#pragma unroll
      for (int g = 0; g < ((t + 2) >> 2); ++g) nxt[g] = mrow4(mpl, t - 1, g);  // M[t-1][0..t-2]
    }
    const float xt = x[t];
#pragma unroll
    for (int g = 0; g < ((t + 3) >> 2); ++g) {
      const int s = 4 * g;
      x[s] += cur[g].x * xt;
      if (s + 1 < t) x[s + 1] += cur[g].y * xt;
      if (s + 2 < t) x[s + 2] += cur[g].z * xt;
      if (s + 3 < t) x[s + 3] += cur[g].w * xt;
    }
#pragma unroll
    for (int g = 0; g < 16; ++g) cur[g] = nxt[g];
  }
}

}  // namespace wtc
