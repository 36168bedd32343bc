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

// One 16 x 16 block (bi, bj) of the inverse being built: diagonal blocks from `td`, the others from `mpl`.
RT_DEVICE float tblock(const float* mpl, const float* td, int bi, int bj, int r, int c) {
  return bi == bj ? td[bi * 256 + r * 16 + c] : mpl[poff(16 * bi + r, 16 * bj + c)];
}

// T = (I - M)^{-1} for the strictly lower 64 x 64 M in `mpl` (plain swizzled), in place; 128 threads.
//  1. the four diagonal 16 x 16 blocks by right-looking substitution (thread = column; after x[s] is final every
//     later row's sum takes its term, so the updates of one step are independent);
//  2. the off-diagonal blocks by distance d = i - j = 1, 2, 3:  R_j = sum_{k=j}^{i-1} M_ik T_kj, then T_ij = T_ii R_j,
//     each a batch of independent 16 x 16 block products spread over all threads (up to six outputs per thread).
// Scratch: rtmp >= 768 floats, td >= 1024 floats.
RT_DEVICE void invert_unit_lower(float* mpl, float* rtmp, float* td, int tid) {
  if (tid < 64) {
    const int kb = tid >> 4, cc = tid & 15, base = 16 * kb;
    float acc[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) acc[r] = r == cc ? 1.f : 0.f;
#pragma unroll
    for (int s = 0; s < 16; ++s) {
      const float xs = s >= cc ? acc[s] : 0.f;
      acc[s] = xs;
#pragma unroll
      for (int r = s + 1; r < 16; ++r) acc[r] += mpl[poff(base + r, base + s)] * xs;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) td[kb * 256 + r * 16 + cc] = acc[r];
  }
  __syncthreads();
#pragma unroll 1
  for (int d = 1; d < 4; ++d) {
    const int nb = 4 - d;  // blocks (j + d, j), j = 0 .. nb - 1
    float acc[6];
#pragma unroll
    for (int q = 0; q < 6; ++q) acc[q] = 0.f;
#pragma unroll 1
    for (int kk = 0; kk < d; ++kk) {
#pragma unroll 4
      for (int m = 0; m < 16; ++m) {
#pragma unroll
        for (int q = 0; q < 6; ++q) {
          const int e = tid + 128 * q, j = e >> 8, r = (e >> 4) & 15, c = e & 15;
          if (q < 2 * nb) {
            const int k = j + kk;
            acc[q] += mpl[poff(16 * (j + d) + r, 16 * k + m)] * tblock(mpl, td, k, j, m, c);
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 6; ++q)
      if (q < 2 * nb) rtmp[tid + 128 * q] = acc[q];
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 6; ++q) acc[q] = 0.f;
#pragma unroll 4
    for (int m = 0; m < 16; ++m) {
#pragma unroll
      for (int q = 0; q < 6; ++q) {
        const int e = tid + 128 * q, j = e >> 8, r = (e >> 4) & 15, c = e & 15;
        if (q < 2 * nb) acc[q] += td[(j + d) * 256 + r * 16 + m] * rtmp[j * 256 + m * 16 + c];
      }
    }
#pragma unroll
    for (int q = 0; q < 6; ++q) {
      const int e = tid + 128 * q, j = e >> 8, r = (e >> 4) & 15, c = e & 15;
      if (q < 2 * nb) mpl[poff(16 * (j + d) + r, 16 * j + c)] = acc[q];
    }
    __syncthreads();
  }
  for (int e = tid; e < 4 * 256; e += 128) {
    const int kb = e >> 8, r = (e >> 4) & 15, c = e & 15;
    mpl[poff(16 * kb + r, 16 * kb + c)] = td[e];
  }
  __syncthreads();
}

}  // namespace wtc
