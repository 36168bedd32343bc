// Fused element-wise stages of the RWKV7 TimeMix student (forward and
// hand-written backward) and the flat-buffer optimizer, sm_100a.
//
// Layout: activations are row-major [M = B*T tokens, C] bf16 unless noted;
// head h covers columns [h*N, (h+1)*N). Parameter vectors are fp32 [C].
//
// Forward (reference math: theseus/timemix.py:66-89 of the reference project)
//   mix      x, shift -> mixed_{r,w,k,v,a,g} = x + (shift(x) - x) * x_*
//   pre_wkv  w = w0 + lw ; a = sigmoid(a0 + la) ; kk = normalize(k * k_k) per head ;
//            k' = k (1 + (a - 1) k_a)  ->  WKV inputs (w, k', -kk, kk * a)
//   post_wkv u = GroupNorm_h(y) + (sum_n r k' r_k) v ;  out = u * g
//   loss     per-token NMSE / cosine sums and d(sum NMSE)/d prediction
// Backward stages mirror these; parameter-vector gradients (x_*, w0, a0, k_k,
// k_a, r_k, ln_x.weight/bias) are summed over the rows of a block in
// registers/shared memory and added to the flat fp32 gradient buffer with one
// atomicAdd per block and channel.
//
// Optimizer: gradients are scaled by 1/count (count read from device memory),
// the global L2 norm over the layer's flat buffer is formed by a partial-sum
// kernel, then one update kernel applies the clip coefficient
// min(1, clip / (norm + 1e-6)), decoupled weight decay on the decay prefix,
// Adam moments with bias correction, refreshes the bf16 copy used by the
// GEMMs, clears the gradient and writes the step report
// [sum nmse, sum cos, count, norm, error].
#include <algorithm>
#include "../common/common.cuh"

namespace {

using bf16 = __nv_bfloat16;
constexpr float GN_EPS = 64e-5f;

RT_DEVICE float bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// ---------------------------------------------------------------- token shift / mix
// grid (ceil(C/256), M); out: [6][M][C]
__global__ void mix_kernel(const bf16* __restrict__ x, const bf16* __restrict__ shift, const float* __restrict__ coef,
                           bf16* __restrict__ out, int T, int C, long M) {
  const long row = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int t = row % T;
  const long b = row / T;
  const float xv = rt::to_f(x[row * C + c]);
  const float prev = t ? rt::to_f(x[(row - 1) * C + c]) : rt::to_f(shift[b * C + c]);
  const float delta = bf(prev - xv);
#pragma unroll
  for (int n = 0; n < 6; ++n) out[(long)n * M * C + row * C + c] = __float2bfloat16_rn(xv + delta * coef[n * C + c]);
}

// d x_n[c] += sum_rows dmix_n[row][c] * delta[row][c]; grid (ceil(C/256), ceil(M/ROWS))
constexpr int MIX_ROWS = 64;
__global__ void mix_bwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ shift,
                               const bf16* __restrict__ dmix, float* __restrict__ dcoef, int T, int C, long M) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const long r0 = (long)blockIdx.y * MIX_ROWS;
  const long r1 = min(M, r0 + MIX_ROWS);
  float acc[6] = {0, 0, 0, 0, 0, 0};
  for (long row = r0; row < r1; ++row) {
    const int t = row % T;
    const long b = row / T;
    const float xv = rt::to_f(x[row * C + c]);
    const float prev = t ? rt::to_f(x[(row - 1) * C + c]) : rt::to_f(shift[b * C + c]);
    const float delta = bf(prev - xv);
#pragma unroll
    for (int n = 0; n < 6; ++n) acc[n] += rt::to_f(dmix[(long)n * M * C + row * C + c]) * delta;
  }
#pragma unroll
  for (int n = 0; n < 6; ++n) atomicAdd(&dcoef[n * C + c], acc[n]);
}

// Vectorised forms (C % 8 == 0, 16-byte aligned rows): a thread takes eight columns of a row with 16-byte loads
// and stores. The backward sums each band of MIXV_ROWS rows into a partial row (no atomics), and a second kernel
// adds the partials in band order, so dcoef does not depend on scheduling.
constexpr int MIXV_ROWS = 16;

__global__ void mix_vec_kernel(const bf16* __restrict__ x, const bf16* __restrict__ shift,
                               const float* __restrict__ coef, bf16* __restrict__ out, int T, int C, long M) {
  const int C8 = C / 8;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= M * C8) return;
  const long row = idx / C8;
  const int c = (int)(idx % C8) * 8;
  const int t = row % T;
  const long b = row / T;
  float xv[8], pv[8], delta[8];
  rt::unpack8(__ldg(reinterpret_cast<const uint4*>(x + row * C + c)), xv);
  rt::unpack8(__ldg(reinterpret_cast<const uint4*>(t ? x + (row - 1) * C + c : shift + b * C + c)), pv);
#pragma unroll
  for (int u = 0; u < 8; ++u) delta[u] = bf(pv[u] - xv[u]);
#pragma unroll
  for (int n = 0; n < 6; ++n) {
    const float4 c0 = __ldg(reinterpret_cast<const float4*>(coef + n * C + c));
    const float4 c1 = __ldg(reinterpret_cast<const float4*>(coef + n * C + c + 4));
    const float cf[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    float o[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) o[u] = xv[u] + delta[u] * cf[u];
    *reinterpret_cast<uint4*>(out + (long)n * M * C + row * C + c) = rt::pack8(o);
  }
}

// partial[band][n][c] = sum over the band's rows of dmix_n[row][c] * delta[row][c]; grid (ceil(C/8/128), bands)
__global__ void mix_bwd_part_kernel(const bf16* __restrict__ x, const bf16* __restrict__ shift,
                                    const bf16* __restrict__ dmix, float* __restrict__ partial, int T, int C, long M) {
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= C) return;
  const long r0 = (long)blockIdx.y * MIXV_ROWS;
  const long r1 = min(M, r0 + MIXV_ROWS);
  float acc[6][8];
#pragma unroll
  for (int n = 0; n < 6; ++n)
#pragma unroll
    for (int u = 0; u < 8; ++u) acc[n][u] = 0.f;
#pragma unroll 2
  for (long row = r0; row < r1; ++row) {
    const int t = row % T;
    const long b = row / T;
    float xv[8], pv[8], dm[6][8];
    rt::unpack8(__ldg(reinterpret_cast<const uint4*>(x + row * C + c)), xv);
    rt::unpack8(__ldg(reinterpret_cast<const uint4*>(t ? x + (row - 1) * C + c : shift + b * C + c)), pv);
#pragma unroll
    for (int n = 0; n < 6; ++n)
      rt::unpack8(__ldcs(reinterpret_cast<const uint4*>(dmix + (long)n * M * C + row * C + c)), dm[n]);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float delta = bf(pv[u] - xv[u]);
#pragma unroll
      for (int n = 0; n < 6; ++n) acc[n][u] += dm[n][u] * delta;
    }
  }
  float* dst = partial + (long)blockIdx.y * 6 * C;
#pragma unroll
  for (int n = 0; n < 6; ++n) {
    *reinterpret_cast<float4*>(dst + n * C + c) = make_float4(acc[n][0], acc[n][1], acc[n][2], acc[n][3]);
    *reinterpret_cast<float4*>(dst + n * C + c + 4) = make_float4(acc[n][4], acc[n][5], acc[n][6], acc[n][7]);
  }
}

__global__ void mix_bwd_sum_kernel(const float* __restrict__ partial, float* __restrict__ dcoef, int bands,
                                   int C6) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= C6) return;
  float s = 0.f;
  for (int b = 0; b < bands; ++b) s += partial[(long)b * C6 + i];
  dcoef[i] += s;
}

// ---------------------------------------------------------------- pre-WKV
// One warp per (row, head); N <= 128 (4 values per lane).
struct PreParams {
  const float *w0, *a0, *k_k, *k_a;
};

__global__ void pre_wkv_kernel(const bf16* __restrict__ k, const bf16* __restrict__ lw, const bf16* __restrict__ la,
                               PreParams p, bf16* __restrict__ w_in, bf16* __restrict__ k_in, bf16* __restrict__ a_in,
                               bf16* __restrict__ b_in, long rows, int H, int N) {
  const long wid = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= rows * H) return;
  const long row = wid / H;
  const int h = wid % H;
  const int C = H * N;
  float kv[4], z[4], av[4];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = lane + 32 * j;
    if (n < N) {
      const int c = h * N + n;
      kv[j] = rt::to_f(k[row * C + c]);
      z[j] = kv[j] * p.k_k[c];
      ss += z[j] * z[j];
    } else {
      kv[j] = z[j] = 0.f;
    }
  }
  ss = rt::warp_sum(ss);
  const float inv = 1.f / fmaxf(sqrtf(ss), 1e-12f);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = lane + 32 * j;
    if (n >= N) continue;
    const int c = h * N + n;
    const long o = row * C + c;
    const float w = p.w0[c] + rt::to_f(lw[o]);
    av[j] = rt::sigmoidf_(p.a0[c] + rt::to_f(la[o]));
    const float kk = z[j] * inv;
    const float kp = kv[j] * (1.f + (av[j] - 1.f) * p.k_a[c]);
    w_in[o] = __float2bfloat16_rn(w);
    k_in[o] = __float2bfloat16_rn(kp);
    a_in[o] = __float2bfloat16_rn(-kk);
    b_in[o] = __float2bfloat16_rn(kk * av[j]);
  }
}

// ---------------------------------------------------------------- post-WKV
// One warp per (row, head): u = GN(y) + s v, out = u * g; saves mean, rstd and s for backward.
__global__ void post_wkv_kernel(const bf16* __restrict__ y, const bf16* __restrict__ r, const bf16* __restrict__ kp,
                                const bf16* __restrict__ v, const bf16* __restrict__ g, const float* __restrict__ ln_w,
                                const float* __restrict__ ln_b, const float* __restrict__ r_k, bf16* __restrict__ out,
                                float* __restrict__ stats, long rows, int H, int N) {
  const long wid = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= rows * H) return;
  const long row = wid / H;
  const int h = wid % H;
  const int C = H * N;
  float yv[4], sum = 0.f, bonus = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = lane + 32 * j;
    yv[j] = 0.f;
    if (n < N) {
      const long o = row * C + h * N + n;
      yv[j] = rt::to_f(y[o]);
      sum += yv[j];
      bonus += rt::to_f(r[o]) * rt::to_f(kp[o]) * r_k[h * N + n];
    }
  }
  sum = rt::warp_sum(sum);
  bonus = rt::warp_sum(bonus);
  const float mean = sum / N;
  float var = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = lane + 32 * j;
    if (n < N) var += (yv[j] - mean) * (yv[j] - mean);
  }
  var = rt::warp_sum(var) / N;
  const float rstd = rsqrtf(var + GN_EPS);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = lane + 32 * j;
    if (n >= N) continue;
    const int c = h * N + n;
    const long o = row * C + c;
    const float u = (yv[j] - mean) * rstd * ln_w[c] + ln_b[c] + bonus * rt::to_f(v[o]);
    out[o] = __float2bfloat16_rn(u * rt::to_f(g[o]));
  }
  if (lane == 0) {
    stats[wid * 3 + 0] = mean;
    stats[wid * 3 + 1] = rstd;
    stats[wid * 3 + 2] = bonus;
  }
}

// Backward of post-WKV. Outputs dy (bf16, WKV output grad), dg (bf16), the bonus-term gradients of r, k',
// v (fp32, written), and parameter partials for ln_w, ln_b, r_k.
// Block = 8 warps = 8 (row, head) items of the same head group; params reduced per block in smem.
constexpr int PW_WARPS = 8;
__global__ void post_wkv_bwd_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ y,
                                    const bf16* __restrict__ r, const bf16* __restrict__ kp,
                                    const bf16* __restrict__ v, const bf16* __restrict__ g,
                                    const float* __restrict__ ln_w, const float* __restrict__ ln_b,
                                    const float* __restrict__ r_k, const float* __restrict__ stats,
                                    bf16* __restrict__ dy, bf16* __restrict__ dg, float* __restrict__ dr,
                                    float* __restrict__ dk, float* __restrict__ dv, float* __restrict__ dln_w,
                                    float* __restrict__ dln_b, float* __restrict__ dr_k, long rows, int H, int N,
                                    int rows_per_block) {
  // blockIdx.x: head, blockIdx.y: row block. Each warp walks rows of this head.
  const int h = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = H * N;
  const long r0 = (long)blockIdx.y * rows_per_block;
  const long r1 = min(rows, r0 + rows_per_block);
  float pw[4] = {0, 0, 0, 0}, pb[4] = {0, 0, 0, 0}, pk[4] = {0, 0, 0, 0};
  for (long row = r0 + warp; row < r1; row += PW_WARPS) {
    const long item = row * H + h;
    const float mean = stats[item * 3], rstd = stats[item * 3 + 1], s = stats[item * 3 + 2];
    float du[4], xh[4], vv[4], rr[4], kk[4];
    float sum_dxh = 0.f, sum_dxh_xh = 0.f, ds = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = lane + 32 * j;
      du[j] = xh[j] = vv[j] = rr[j] = kk[j] = 0.f;
      if (n < N) {
        const int c = h * N + n;
        const long o = row * C + c;
        const float gv = rt::to_f(g[o]);
        const float d = rt::to_f(dout[o]);
        xh[j] = (rt::to_f(y[o]) - mean) * rstd;
        vv[j] = rt::to_f(v[o]);
        rr[j] = rt::to_f(r[o]);
        kk[j] = rt::to_f(kp[o]);
        const float u = xh[j] * ln_w[c] + ln_b[c] + s * vv[j];
        dg[o] = __float2bfloat16_rn(d * u);
        du[j] = d * gv;
        const float dxh = du[j] * ln_w[c];
        sum_dxh += dxh;
        sum_dxh_xh += dxh * xh[j];
        ds += du[j] * vv[j];
        pw[j] += du[j] * xh[j];
        pb[j] += du[j];
      }
    }
    sum_dxh = rt::warp_sum(sum_dxh) / N;
    sum_dxh_xh = rt::warp_sum(sum_dxh_xh) / N;
    ds = rt::warp_sum(ds);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = lane + 32 * j;
      if (n >= N) continue;
      const int c = h * N + n;
      const long o = row * C + c;
      const float dxh = du[j] * ln_w[c];
      dy[o] = __float2bfloat16_rn(rstd * (dxh - sum_dxh - xh[j] * sum_dxh_xh));
      dv[o] = du[j] * s;
      const float rkv = r_k[c];
      dr[o] = ds * kk[j] * rkv;
      dk[o] = ds * rr[j] * rkv;
      pk[j] += ds * rr[j] * kk[j];
    }
  }
  __shared__ float red[3][PW_WARPS][128];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = lane + 32 * j;
    if (n < 128) {
      red[0][warp][n] = pw[j];
      red[1][warp][n] = pb[j];
      red[2][warp][n] = pk[j];
    }
  }
  __syncthreads();
  for (int n = threadIdx.x; n < N; n += blockDim.x) {
    float a = 0, b = 0, k = 0;
    for (int w = 0; w < PW_WARPS; ++w) { a += red[0][w][n]; b += red[1][w][n]; k += red[2][w][n]; }
    atomicAdd(&dln_w[h * N + n], a);
    atomicAdd(&dln_b[h * N + n], b);
    atomicAdd(&dr_k[h * N + n], k);
  }
}

// Backward of pre-WKV: consumes the fp32 WKV-input gradients plus the bonus-term gradients, produces bf16
// gradients of the projections r, k, v, lw (decay LoRA output), la (ICL LoRA pre-activation) and
// parameter partials for w0, a0, k_k, k_a.
__global__ void pre_wkv_bwd_kernel(const float* __restrict__ g_r, const float* __restrict__ g_w,
                                   const float* __restrict__ g_kp, const float* __restrict__ g_v,
                                   const float* __restrict__ g_a, const float* __restrict__ g_b,
                                   const float* __restrict__ b_r, const float* __restrict__ b_kp,
                                   const float* __restrict__ b_v,
                                   const bf16* __restrict__ k, const bf16* __restrict__ la, PreParams p,
                                   bf16* __restrict__ dr, bf16* __restrict__ dk, bf16* __restrict__ dv,
                                   bf16* __restrict__ dlw, bf16* __restrict__ dla, float* __restrict__ dw0,
                                   float* __restrict__ da0, float* __restrict__ dk_k, float* __restrict__ dk_a,
                                   long rows, int H, int N, int rows_per_block) {
  const int h = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = H * N;
  const long r0 = (long)blockIdx.y * rows_per_block;
  const long r1 = min(rows, r0 + rows_per_block);
  float s_w0[4] = {0, 0, 0, 0}, s_a0[4] = {0, 0, 0, 0}, s_kk[4] = {0, 0, 0, 0}, s_ka[4] = {0, 0, 0, 0};
  for (long row = r0 + warp; row < r1; row += PW_WARPS) {
    float kv[4], z[4], av[4], dkk[4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = lane + 32 * j;
      kv[j] = z[j] = av[j] = dkk[j] = 0.f;
      if (n < N) {
        const int c = h * N + n;
        const long o = row * C + c;
        kv[j] = rt::to_f(k[o]);
        z[j] = kv[j] * p.k_k[c];
        ss += z[j] * z[j];
        av[j] = rt::sigmoidf_(p.a0[c] + rt::to_f(la[o]));
      }
    }
    ss = rt::warp_sum(ss);
    const float norm = fmaxf(sqrtf(ss), 1e-12f);
    const float inv = 1.f / norm;
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = lane + 32 * j;
      if (n >= N) continue;
      const long o = row * C + h * N + n;
      const float kk = z[j] * inv;
      // b_in = kk * a, a_in = -kk
      dkk[j] = g_b[o] * av[j] - g_a[o];
      dot += dkk[j] * kk;
    }
    dot = rt::warp_sum(dot);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = lane + 32 * j;
      if (n >= N) continue;
      const int c = h * N + n;
      const long o = row * C + c;
      const float kk = z[j] * inv;
      const float gkp = g_kp[o] + b_kp[o];
      const float ka = p.k_a[c];
      // a: from b_in (kk) and from k' = k (1 + (a - 1) k_a)
      const float da = g_b[o] * kk + gkp * kv[j] * ka;
      const float dpre_a = da * av[j] * (1.f - av[j]);
      // normalisation backward (active branch ss > eps^2)
      const float dz = norm > 1e-12f ? (dkk[j] - kk * dot) * inv : dkk[j] * inv;
      const float dkv = gkp * (1.f + (av[j] - 1.f) * ka) + dz * p.k_k[c];
      dr[o] = __float2bfloat16_rn(g_r[o] + b_r[o]);
      dk[o] = __float2bfloat16_rn(dkv);
      dv[o] = __float2bfloat16_rn(g_v[o] + b_v[o]);
      dlw[o] = __float2bfloat16_rn(g_w[o]);
      dla[o] = __float2bfloat16_rn(dpre_a);
      s_w0[j] += g_w[o];
      s_a0[j] += dpre_a;
      s_kk[j] += dz * kv[j];
      s_ka[j] += gkp * kv[j] * (av[j] - 1.f);
    }
  }
  __shared__ float red[4][PW_WARPS][128];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = lane + 32 * j;
    if (n < 128) {
      red[0][warp][n] = s_w0[j];
      red[1][warp][n] = s_a0[j];
      red[2][warp][n] = s_kk[j];
      red[3][warp][n] = s_ka[j];
    }
  }
  __syncthreads();
  for (int n = threadIdx.x; n < N; n += blockDim.x) {
    float a = 0, b = 0, c2 = 0, d = 0;
    for (int w = 0; w < PW_WARPS; ++w) { a += red[0][w][n]; b += red[1][w][n]; c2 += red[2][w][n]; d += red[3][w][n]; }
    atomicAdd(&dw0[h * N + n], a);
    atomicAdd(&da0[h * N + n], b);
    atomicAdd(&dk_k[h * N + n], c2);
    atomicAdd(&dk_a[h * N + n], d);
  }
}

// Head size 64, vectorised: a half-warp per (row, head), lane l of it takes n = 4l .. 4l + 3 with 16-byte fp32 loads
// and 8-byte bf16 stores; a warp takes two rows at a time. Same arithmetic and the same per-block reductions as
// pre_wkv_bwd_kernel.
RT_DEVICE float half_warp_sum(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
RT_DEVICE void load4_bf16(const bf16* p, float* f) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
  const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
  f[0] = __low2float(lo); f[1] = __high2float(lo); f[2] = __low2float(hi); f[3] = __high2float(hi);
}
RT_DEVICE void store4_bf16(bf16* p, float a, float b, float c, float d) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  uint2 u;
  u.x = *reinterpret_cast<const unsigned*>(&lo);
  u.y = *reinterpret_cast<const unsigned*>(&hi);
  *reinterpret_cast<uint2*>(p) = u;
}
RT_DEVICE float4 ld4(const float* p) { return __ldcs(reinterpret_cast<const float4*>(p)); }

__global__ void pre_wkv_bwd64_kernel(const float* __restrict__ g_r, const float* __restrict__ g_w,
                                     const float* __restrict__ g_kp, const float* __restrict__ g_v,
                                     const float* __restrict__ g_a, const float* __restrict__ g_b,
                                     const float* __restrict__ b_r, const float* __restrict__ b_kp,
                                     const float* __restrict__ b_v, const bf16* __restrict__ k,
                                     const bf16* __restrict__ la, PreParams p, bf16* __restrict__ dr,
                                     bf16* __restrict__ dk, bf16* __restrict__ dv, bf16* __restrict__ dlw,
                                     bf16* __restrict__ dla, float* __restrict__ dw0, float* __restrict__ da0,
                                     float* __restrict__ dk_k, float* __restrict__ dk_a, long rows, int H,
                                     int rows_per_block) {
  constexpr int N = 64;
  const int h = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane >> 4, n0 = 4 * (lane & 15);
  const int C = H * N, c0 = h * N + n0;
  const long r0 = (long)blockIdx.y * rows_per_block;
  const long r1 = min(rows, r0 + rows_per_block);
  float kkp[4], a0p[4], kap[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    kkp[j] = p.k_k[c0 + j];
    a0p[j] = p.a0[c0 + j];
    kap[j] = p.k_a[c0 + j];
  }
  float s_w0[4] = {0, 0, 0, 0}, s_a0[4] = {0, 0, 0, 0}, s_kk[4] = {0, 0, 0, 0}, s_ka[4] = {0, 0, 0, 0};
  for (long base = r0 + 2 * warp; base < r1; base += 2 * PW_WARPS) {  // uniform per warp (shuffles below)
    const long row = base + sub;
    const bool valid = row < r1;
    const long o = (valid ? row : r0) * C + c0;
    float kv[4], lav[4], z[4], av[4];
    load4_bf16(k + o, kv);
    load4_bf16(la + o, lav);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      z[j] = kv[j] * kkp[j];
      ss += z[j] * z[j];
      av[j] = rt::sigmoidf_(a0p[j] + lav[j]);
    }
    ss = half_warp_sum(ss);
    const float norm = fmaxf(sqrtf(ss), 1e-12f);
    const float inv = 1.f / norm;
    const float4 gb = ld4(g_b + o), ga = ld4(g_a + o);
    const float gbv[4] = {gb.x, gb.y, gb.z, gb.w}, gav[4] = {ga.x, ga.y, ga.z, ga.w};
    float dkk[4], kk[4], dot = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      kk[j] = z[j] * inv;
      dkk[j] = gbv[j] * av[j] - gav[j];  // b_in = kk * a, a_in = -kk
      dot += dkk[j] * kk[j];
    }
    dot = half_warp_sum(dot);
    const float4 gkp4 = ld4(g_kp + o), bkp4 = ld4(b_kp + o);
    const float4 gr4 = ld4(g_r + o), br4 = ld4(b_r + o), gv4 = ld4(g_v + o), bv4 = ld4(b_v + o), gw4 = ld4(g_w + o);
    const float gkp[4] = {gkp4.x + bkp4.x, gkp4.y + bkp4.y, gkp4.z + bkp4.z, gkp4.w + bkp4.w};
    const float gwv[4] = {gw4.x, gw4.y, gw4.z, gw4.w};
    float dkv[4], dpa[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float da = gbv[j] * kk[j] + gkp[j] * kv[j] * kap[j];  // a: from b_in (kk) and from k'
      dpa[j] = da * av[j] * (1.f - av[j]);
      const float dz = norm > 1e-12f ? (dkk[j] - kk[j] * dot) * inv : dkk[j] * inv;
      dkv[j] = gkp[j] * (1.f + (av[j] - 1.f) * kap[j]) + dz * kkp[j];
      if (valid) {
        s_w0[j] += gwv[j];
        s_a0[j] += dpa[j];
        s_kk[j] += dz * kv[j];
        s_ka[j] += gkp[j] * kv[j] * (av[j] - 1.f);
      }
    }
    if (valid) {
      store4_bf16(dr + o, gr4.x + br4.x, gr4.y + br4.y, gr4.z + br4.z, gr4.w + br4.w);
      store4_bf16(dk + o, dkv[0], dkv[1], dkv[2], dkv[3]);
      store4_bf16(dv + o, gv4.x + bv4.x, gv4.y + bv4.y, gv4.z + bv4.z, gv4.w + bv4.w);
      store4_bf16(dlw + o, gwv[0], gwv[1], gwv[2], gwv[3]);
      store4_bf16(dla + o, dpa[0], dpa[1], dpa[2], dpa[3]);
    }
  }
  __shared__ float red[4][2 * PW_WARPS][N];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    red[0][2 * warp + sub][n0 + j] = s_w0[j];
    red[1][2 * warp + sub][n0 + j] = s_a0[j];
    red[2][2 * warp + sub][n0 + j] = s_kk[j];
    red[3][2 * warp + sub][n0 + j] = s_ka[j];
  }
  __syncthreads();
  for (int n = threadIdx.x; n < N; n += blockDim.x) {
    float a = 0, b = 0, c2 = 0, d = 0;
    for (int w = 0; w < 2 * PW_WARPS; ++w) { a += red[0][w][n]; b += red[1][w][n]; c2 += red[2][w][n]; d += red[3][w][n]; }
    atomicAdd(&dw0[h * N + n], a);
    atomicAdd(&da0[h * N + n], b);
    atomicAdd(&dk_k[h * N + n], c2);
    atomicAdd(&dk_a[h * N + n], d);
  }
}

// ---------------------------------------------------------------- LoRA activations
// mode 0: out = tanh(x); 1: out = sigmoid(x)  (forward, in place allowed)
__global__ void act_kernel(bf16* __restrict__ x, long n, int mode) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = rt::to_f(x[i]);
  x[i] = __float2bfloat16_rn(mode == 0 ? tanhf(v) : rt::sigmoidf_(v));
}
// d pre = dh * f'(pre) given the saved activation h: tanh -> 1 - h^2, sigmoid -> h (1 - h)
__global__ void act_bwd_kernel(const bf16* __restrict__ h, bf16* __restrict__ dh, long n, int mode) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float hv = rt::to_f(h[i]), d = rt::to_f(dh[i]);
  dh[i] = __float2bfloat16_rn(mode == 0 ? d * (1.f - hv * hv) : d * hv * (1.f - hv));
}

// ---------------------------------------------------------------- loss
// One block per token row. stats += [nmse, cos, 1]; dpred = scale * 2 (p - t) / (C max(mean(t^2), eps)).
__global__ void nmse_loss_kernel(const bf16* __restrict__ pred, const bf16* __restrict__ target,
                                 float* __restrict__ stats, bf16* __restrict__ dpred, int C, float eps) {
  __shared__ float scratch[32];
  const long row = blockIdx.x;
  float se = 0.f, tt = 0.f, pp = 0.f, pt = 0.f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float p = rt::to_f(pred[row * C + c]), t = rt::to_f(target[row * C + c]);
    se += (p - t) * (p - t);
    tt += t * t;
    pp += p * p;
    pt += p * t;
  }
  se = rt::block_sum(se, scratch);
  tt = rt::block_sum(tt, scratch);
  pp = rt::block_sum(pp, scratch);
  pt = rt::block_sum(pt, scratch);
  const float denom = fmaxf(tt / C, eps);
  if (threadIdx.x == 0) {
    atomicAdd(&stats[0], (se / C) / denom);
    atomicAdd(&stats[1], pt / sqrtf(fmaxf(pp * tt, eps * eps)));
    atomicAdd(&stats[2], 1.f);
  }
  if (dpred) {
    const float k = 2.f / (C * denom);
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
      const float p = rt::to_f(pred[row * C + c]), t = rt::to_f(target[row * C + c]);
      dpred[row * C + c] = __float2bfloat16_rn(k * (p - t));
    }
  }
}

// Fused-loss path (output GEMM epilogue computes dpred and the row sums): rowsum [rows, 4] = {sum t^2, 0, 0, 0}
// before the GEMM; after it, one block turns the rows' sums into stats += [sum nmse, sum cos, rows] in a fixed
// order (deterministic).
__global__ void loss_rows_prep_kernel(const bf16* __restrict__ target, float* __restrict__ rowsum, int C) {
  __shared__ float scratch[32];
  const long row = blockIdx.x;
  float tt = 0.f;
  if (C % 8 == 0 && (reinterpret_cast<uintptr_t>(target) & 15) == 0) {
    const uint4* t8 = reinterpret_cast<const uint4*>(target + row * C);
    for (int c = threadIdx.x; c < C / 8; c += blockDim.x) {
      float t[8];
      rt::unpack8(__ldg(t8 + c), t);
#pragma unroll
      for (int u = 0; u < 8; ++u) tt += t[u] * t[u];
    }
  } else {
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
      const float t = rt::to_f(target[row * C + c]);
      tt += t * t;
    }
  }
  tt = rt::block_sum(tt, scratch);
  if (threadIdx.x < 4) rowsum[4 * row + threadIdx.x] = threadIdx.x == 0 ? tt : 0.f;
}

__global__ void loss_rows_finish_kernel(const float4* __restrict__ rowsum, float* __restrict__ stats, long rows, int C,
                                        float eps) {
  __shared__ float scratch[32];
  float nmse = 0.f, cosv = 0.f;
  for (long r = threadIdx.x; r < rows; r += blockDim.x) {
    const float4 q = rowsum[r];  // {tt, se, pp, pt}
    nmse += (q.y / C) / fmaxf(q.x / C, eps);
    cosv += q.w / sqrtf(fmaxf(q.z * q.x, eps * eps));
  }
  nmse = rt::block_sum(nmse, scratch);
  cosv = rt::block_sum(cosv, scratch);
  if (threadIdx.x == 0) {
    stats[0] += nmse;
    stats[1] += cosv;
    stats[2] += (float)rows;
  }
}

// ---------------------------------------------------------------- optimizer
// The gradient buffer is read, never written: the next micro-step's GEMMs store the four big matrices' gradients
// and the rest of the buffer is cleared when that micro-step starts (StudentStep in bindings.cpp).
// Per-block partial sums of g^2 (raw sums; the 1/count scale is applied later), one slot per block: the report
// kernel adds them in block order, so the norm does not depend on the order blocks finish in.
constexpr int NORM_BLOCKS = 1024;
__global__ void norm2_kernel(const float4* __restrict__ g, long n4, const float* __restrict__ g_tail, long tail,
                             float* __restrict__ partial) {
  __shared__ float scratch[32];
  float acc = 0.f;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    const float4 v = __ldcs(g + i);
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  if (blockIdx.x == 0)
    for (long i = threadIdx.x; i < tail; i += blockDim.x) acc += g_tail[i] * g_tail[i];
  acc = rt::block_sum(acc, scratch);
  if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

struct AdamArgs {
  float lr, beta1, beta2, eps, weight_decay, clip, bias1, bias2_sqrt;
  long decay_numel;
};

RT_DEVICE void adam_elem(float g, float& p, float& m, float& v, long i, const AdamArgs& a, float step) {
  if (i < a.decay_numel) p *= 1.f - a.lr * a.weight_decay;
  m = m + (1.f - a.beta1) * (g - m);
  v = a.beta2 * v + (1.f - a.beta2) * g * g;
  p -= step * m / (sqrtf(v) / a.bias2_sqrt + a.eps);
}

// One block: the norm from the partial sums (fixed order), the report [nmse, cos, count, norm, error], the
// gradient scale for adamw_kernel in scale[0], and the update's statistics cleared for the next update.
__global__ void report_kernel(float* __restrict__ stats, const float* __restrict__ partial, int nblocks,
                              float* __restrict__ scale, float* __restrict__ report, float clip) {
  __shared__ float scratch[32];
  float acc = 0.f;
  for (int b = threadIdx.x; b < nblocks; b += blockDim.x) acc += partial[b];
  acc = rt::block_sum(acc, scratch);
  if (threadIdx.x == 0) {
    const float count = stats[2];
    const float inv = count > 0.f ? 1.f / count : 0.f;
    const float norm = sqrtf(acc) * inv;
    report[0] = stats[0];
    report[1] = stats[1];
    report[2] = count;
    report[3] = norm;
    report[4] = (!isfinite(norm) || count <= 0.f) ? 1.f : 0.f;
    scale[0] = inv * fminf(1.f, clip / (norm + 1e-6f));
    stats[0] = stats[1] = stats[2] = 0.f;
  }
}

// g is scaled by (1/count) * min(1, clip / (|g| / count + 1e-6)): the reference's division by the token count
// followed by clip_grad_norm_ on the divided gradients (the factor comes from report_kernel).
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, bf16* __restrict__ shadow, long n, const float* __restrict__ scale,
                             AdamArgs a) {
  const float gscale = scale[0];
  const float step = a.lr / a.bias1;
  const long n4 = n / 4;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    const float4 g4 = __ldcs(reinterpret_cast<const float4*>(g) + i);
    float4 p4 = reinterpret_cast<const float4*>(p)[i];
    float4 m4 = __ldcs(reinterpret_cast<const float4*>(m) + i);
    float4 v4 = __ldcs(reinterpret_cast<const float4*>(v) + i);
    const long e = 4 * i;
    adam_elem(g4.x * gscale, p4.x, m4.x, v4.x, e + 0, a, step);
    adam_elem(g4.y * gscale, p4.y, m4.y, v4.y, e + 1, a, step);
    adam_elem(g4.z * gscale, p4.z, m4.z, v4.z, e + 2, a, step);
    adam_elem(g4.w * gscale, p4.w, m4.w, v4.w, e + 3, a, step);
    reinterpret_cast<float4*>(p)[i] = p4;
    __stcs(reinterpret_cast<float4*>(m) + i, m4);
    __stcs(reinterpret_cast<float4*>(v) + i, v4);
    if (shadow) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(p4.x, p4.y), hi = __floats2bfloat162_rn(p4.z, p4.w);
      uint2 packed;
      packed.x = *reinterpret_cast<unsigned*>(&lo);
      packed.y = *reinterpret_cast<unsigned*>(&hi);
      reinterpret_cast<uint2*>(shadow)[i] = packed;
    }
  }
  if (blockIdx.x == 0) {
    for (long i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) {
      float pv = p[i], mv = m[i], vv = v[i];
      adam_elem(g[i] * gscale, pv, mv, vv, i, a, step);
      p[i] = pv;
      m[i] = mv;
      v[i] = vv;
      if (shadow) shadow[i] = __float2bfloat16_rn(pv);
    }
  }
}

__global__ void zero_f32_kernel(float4* __restrict__ p, long n4, float* __restrict__ tail, long ntail) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x)
    p[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (blockIdx.x == 0)
    for (long i = threadIdx.x; i < ntail; i += blockDim.x) tail[i] = 0.f;
}

__global__ void to_bf16_kernel(const float* __restrict__ src, bf16* __restrict__ dst, long n) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

int grid_for(long n, int threads, int cap = 148 * 8) {
  const long g = (n + threads - 1) / threads;
  return (int)(g < cap ? g : cap);
}

}  // namespace

namespace {
bool mix_vectorizable(const void* x, const void* shift, const void* other, const float* coef, int C) {
  return C % 8 == 0 &&
         ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(shift) | reinterpret_cast<uintptr_t>(other) |
           reinterpret_cast<uintptr_t>(coef)) & 15) == 0;
}
}  // namespace

extern "C" cudaError_t rt_tm_mix(const void* x, const void* shift, const float* coef, void* out, int B, int T, int C,
                                 cudaStream_t s) {
  const long M = (long)B * T;
  if (mix_vectorizable(x, shift, out, coef, C)) {
    const long items = M * (C / 8);
    mix_vec_kernel<<<(items + 255) / 256, 256, 0, s>>>((const bf16*)x, (const bf16*)shift, coef, (bf16*)out, T, C,
                                                        M);
    return cudaGetLastError();
  }
  mix_kernel<<<dim3((C + 255) / 256, M), 256, 0, s>>>((const bf16*)x, (const bf16*)shift, coef, (bf16*)out, T, C, M);
  return cudaGetLastError();
}

// Floats of scratch rt_tm_mix_bwd needs for its partial sums (0: the atomic fallback needs none).
extern "C" long rt_tm_mix_bwd_scratch(int B, int T, int C) {
  const long M = (long)B * T;
  return C % 8 == 0 ? ((M + MIXV_ROWS - 1) / MIXV_ROWS) * 6L * C : 0;
}

extern "C" cudaError_t rt_tm_mix_bwd(const void* x, const void* shift, const void* dmix, float* dcoef, int B, int T,
                                     int C, float* scratch, cudaStream_t s) {
  const long M = (long)B * T;
  if (scratch && mix_vectorizable(x, shift, dmix, dcoef, C) && (reinterpret_cast<uintptr_t>(scratch) & 15) == 0) {
    const int bands = (int)((M + MIXV_ROWS - 1) / MIXV_ROWS);
    mix_bwd_part_kernel<<<dim3((C / 8 + 127) / 128, bands), 128, 0, s>>>((const bf16*)x, (const bf16*)shift,
                                                                        (const bf16*)dmix, scratch, T, C, M);
    RT_CUDA_CHECK(cudaGetLastError());
    mix_bwd_sum_kernel<<<(6 * C + 255) / 256, 256, 0, s>>>(scratch, dcoef, bands, 6 * C);
    return cudaGetLastError();
  }
  mix_bwd_kernel<<<dim3((C + 255) / 256, (M + MIX_ROWS - 1) / MIX_ROWS), 256, 0, s>>>(
      (const bf16*)x, (const bf16*)shift, (const bf16*)dmix, dcoef, T, C, M);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_tm_pre_wkv(const void* k, const void* lw, const void* la, const float* w0, const float* a0,
                                     const float* k_k, const float* k_a, void* w_in, void* k_in, void* a_in,
                                     void* b_in, long rows, int H, int N, cudaStream_t s) {
  if (N > 128) return cudaErrorInvalidValue;
  PreParams p{w0, a0, k_k, k_a};
  const long items = rows * H;
  pre_wkv_kernel<<<(items + 7) / 8, 256, 0, s>>>((const bf16*)k, (const bf16*)lw, (const bf16*)la, p, (bf16*)w_in,
                                                 (bf16*)k_in, (bf16*)a_in, (bf16*)b_in, rows, H, N);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_tm_post_wkv(const void* y, const void* r, const void* kp, const void* v, const void* g,
                                      const float* ln_w, const float* ln_b, const float* r_k, void* out, float* stats,
                                      long rows, int H, int N, cudaStream_t s) {
  if (N > 128) return cudaErrorInvalidValue;
  const long items = rows * H;
  post_wkv_kernel<<<(items + 7) / 8, 256, 0, s>>>((const bf16*)y, (const bf16*)r, (const bf16*)kp, (const bf16*)v,
                                                  (const bf16*)g, ln_w, ln_b, r_k, (bf16*)out, stats, rows, H, N);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_tm_post_wkv_bwd(const void* dout, const void* y, const void* r, const void* kp,
                                          const void* v, const void* g, const float* ln_w, const float* ln_b,
                                          const float* r_k, const float* stats, void* dy, void* dg, float* dr,
                                          float* dk, float* dv, float* dln_w, float* dln_b, float* dr_k, long rows,
                                          int H, int N, cudaStream_t s) {
  if (N > 128) return cudaErrorInvalidValue;
  const int rpb = 64;
  dim3 grid(H, (rows + rpb - 1) / rpb);
  post_wkv_bwd_kernel<<<grid, PW_WARPS * 32, 0, s>>>((const bf16*)dout, (const bf16*)y, (const bf16*)r,
                                                     (const bf16*)kp, (const bf16*)v, (const bf16*)g, ln_w, ln_b, r_k,
                                                     stats, (bf16*)dy, (bf16*)dg, dr, dk, dv, dln_w, dln_b, dr_k,
                                                     rows, H, N, rpb);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_tm_pre_wkv_bwd(const float* g_r, const float* g_w, const float* g_kp, const float* g_v,
                                         const float* g_a, const float* g_b, const float* b_r, const float* b_kp,
                                         const float* b_v, const void* k, const void* la,
                                         const float* w0, const float* a0, const float* k_k, const float* k_a,
                                         void* dr, void* dk, void* dv, void* dlw, void* dla, float* dw0, float* da0,
                                         float* dk_k, float* dk_a, long rows, int H, int N, cudaStream_t s) {
  if (N > 128) return cudaErrorInvalidValue;
  PreParams p{w0, a0, k_k, k_a};
  const int rpb = 64;
  dim3 grid(H, (rows + rpb - 1) / rpb);
  const uintptr_t align = reinterpret_cast<uintptr_t>(g_r) | reinterpret_cast<uintptr_t>(g_w) |
                          reinterpret_cast<uintptr_t>(g_kp) | reinterpret_cast<uintptr_t>(g_v) |
                          reinterpret_cast<uintptr_t>(g_a) | reinterpret_cast<uintptr_t>(g_b) |
                          reinterpret_cast<uintptr_t>(b_r) | reinterpret_cast<uintptr_t>(b_kp) |
                          reinterpret_cast<uintptr_t>(b_v) | reinterpret_cast<uintptr_t>(k) |
                          reinterpret_cast<uintptr_t>(la) | reinterpret_cast<uintptr_t>(dr) |
                          reinterpret_cast<uintptr_t>(dk) | reinterpret_cast<uintptr_t>(dv) |
                          reinterpret_cast<uintptr_t>(dlw) | reinterpret_cast<uintptr_t>(dla);
  if (N == 64 && (align & 15) == 0) {
    pre_wkv_bwd64_kernel<<<grid, PW_WARPS * 32, 0, s>>>(g_r, g_w, g_kp, g_v, g_a, g_b, b_r, b_kp, b_v,
                                                        (const bf16*)k, (const bf16*)la, p, (bf16*)dr, (bf16*)dk,
                                                        (bf16*)dv, (bf16*)dlw, (bf16*)dla, dw0, da0, dk_k, dk_a,
                                                        rows, H, rpb);
    return cudaGetLastError();
  }
  pre_wkv_bwd_kernel<<<grid, PW_WARPS * 32, 0, s>>>(g_r, g_w, g_kp, g_v, g_a, g_b, b_r, b_kp, b_v, (const bf16*)k,
                                                    (const bf16*)la,
                                                    p, (bf16*)dr, (bf16*)dk, (bf16*)dv, (bf16*)dlw, (bf16*)dla, dw0,
                                                    da0, dk_k, dk_a, rows, H, N, rpb);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_act(void* x, long n, int mode, cudaStream_t s) {
  act_kernel<<<(n + 255) / 256, 256, 0, s>>>((bf16*)x, n, mode);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_act_bwd(const void* h, void* dh, long n, int mode, cudaStream_t s) {
  act_bwd_kernel<<<(n + 255) / 256, 256, 0, s>>>((const bf16*)h, (bf16*)dh, n, mode);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_loss_rows_prep(const void* target, float* rowsum, long rows, int C, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  loss_rows_prep_kernel<<<rows, 128, 0, s>>>((const bf16*)target, rowsum, C);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_loss_rows_finish(const float* rowsum, float* stats, long rows, int C, float eps,
                                           cudaStream_t s) {
  if (reinterpret_cast<uintptr_t>(rowsum) & 15) return cudaErrorInvalidValue;
  loss_rows_finish_kernel<<<1, 1024, 0, s>>>((const float4*)rowsum, stats, rows, C, eps);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_nmse_loss(const void* pred, const void* target, float* stats, void* dpred, long rows, int C,
                                    float eps, cudaStream_t s) {
  nmse_loss_kernel<<<rows, 256, 0, s>>>((const bf16*)pred, (const bf16*)target, stats, (bf16*)dpred, C, eps);
  return cudaGetLastError();
}

// Reduces the flat gradient's norm, scales by 1/count, clips, applies AdamW, refreshes the bf16 shadow, writes
// the report and clears `stats`; the gradient itself is left untouched. `scratch` holds >= rt_flat_adamw_scratch()
// floats (per-block partial norms and the scale). p, g, m, v and shadow must be 16-byte aligned (flat buffers
// from the caching allocator are).
extern "C" int rt_flat_adamw_scratch() { return NORM_BLOCKS + 4; }

extern "C" cudaError_t rt_flat_adamw(float* p, float* g, float* m, float* v, void* shadow, long n, long decay_numel,
                                     float* stats, float* scratch, float* report, float lr, float beta1, float beta2,
                                     float eps, float weight_decay, float clip, int step, cudaStream_t s) {
  if ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(m) |
       reinterpret_cast<uintptr_t>(v)) & 15 || reinterpret_cast<uintptr_t>(shadow) & 7)
    return cudaErrorMisalignedAddress;
  const long n4 = n / 4;
  const int nblocks = (int)std::min<long>(grid_for(n4, 512), NORM_BLOCKS);
  norm2_kernel<<<nblocks, 512, 0, s>>>(reinterpret_cast<const float4*>(g), n4, g + 4 * n4, n - 4 * n4, scratch);
  RT_CUDA_CHECK(cudaGetLastError());
  float* scale = scratch + NORM_BLOCKS;
  report_kernel<<<1, 256, 0, s>>>(stats, scratch, nblocks, scale, report, clip);
  RT_CUDA_CHECK(cudaGetLastError());
  AdamArgs a;
  a.lr = lr; a.beta1 = beta1; a.beta2 = beta2; a.eps = eps; a.weight_decay = weight_decay; a.clip = clip;
  a.bias1 = (float)(1.0 - pow((double)beta1, (double)step));
  a.bias2_sqrt = (float)sqrt(1.0 - pow((double)beta2, (double)step));
  a.decay_numel = decay_numel;
  adamw_kernel<<<grid_for(n4, 256, 148 * 12), 256, 0, s>>>(p, g, m, v, (bf16*)shadow, n, scale, a);
  return cudaGetLastError();
}

__global__ void copy_bytes_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src, long n16,
                                  uint8_t* __restrict__ dtail, const uint8_t* __restrict__ stail, long ntail) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (long)gridDim.x * blockDim.x)
    dst[i] = __ldcs(src + i);
  if (blockIdx.x == 0)
    for (long i = threadIdx.x; i < ntail; i += blockDim.x) dtail[i] = stail[i];
}

// dst[0 .. nbytes) = src[0 .. nbytes) on the device (own kernel: 16-byte moves when both are 16-byte aligned).
extern "C" cudaError_t rt_copy_bytes(void* dst, const void* src, long nbytes, cudaStream_t s) {
  if (nbytes <= 0) return cudaSuccess;
  const bool aligned = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0;
  const long n16 = aligned ? nbytes / 16 : 0;
  copy_bytes_kernel<<<grid_for(std::max<long>(n16, 1), 256, 148 * 4), 256, 0, s>>>(
      reinterpret_cast<uint4*>(dst), reinterpret_cast<const uint4*>(src), n16,
      reinterpret_cast<uint8_t*>(dst) + 16 * n16, reinterpret_cast<const uint8_t*>(src) + 16 * n16,
      nbytes - 16 * n16);
  return cudaGetLastError();
}

// p[0 .. n) = 0 (own kernel, so that the step's launches stay this package's).
extern "C" cudaError_t rt_zero_f32(float* p, long n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const bool aligned = (reinterpret_cast<uintptr_t>(p) & 15) == 0;
  const long n4 = aligned ? n / 4 : 0;
  zero_f32_kernel<<<grid_for(std::max<long>(n4, 1), 256, 148 * 4), 256, 0, s>>>(reinterpret_cast<float4*>(p), n4,
                                                                                 p + 4 * n4, n - 4 * n4);
  return cudaGetLastError();
}

extern "C" cudaError_t rt_to_bf16(const float* src, void* dst, long n, cudaStream_t s) {
  to_bf16_kernel<<<grid_for(n, 512), 512, 0, s>>>(src, (bf16*)dst, n);
  return cudaGetLastError();
}
