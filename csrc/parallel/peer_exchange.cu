// Per-layer gradient exchange + clip + AdamW over NVLink peer memory (one node, up to 8 ranks).
//
// The reference sums each layer's gradients with an NCCL all-reduce, then runs
// clip_grad_norm_ and torch AdamW on every rank over the whole layer
// (theseus/stage.py:27-44, train.py:170-211). Here one rank owns 1/N of the
// layer's flat buffer and three kernels do the whole update:
//
//   A  reduce-scatter: every rank announces "gradients ready", waits for all
//      ranks, then sums its shard from every rank's gradient buffer with plain
//      peer loads, keeps the sum locally and reduces its squared norm
//      (per-block partials summed in a fixed order by the last block, which
//      publishes the rank's partial norm and loss statistics into every
//      rank's slot array and raises its flag there);
//   B  update: after every rank's norm is published, each rank forms the
//      same global norm (fixed summation order), clips, applies AdamW to its
//      shard (fp32 master, moments, bf16 weight copy; local memory only),
//      clears its loss statistics, writes the report and raises its "shard
//      updated" flag everywhere (the gradient buffer is not cleared: the next
//      micro-step overwrites it);
//   C  all-gather: after every rank's flag, each rank pulls the other shards
//      of the bf16 weight copy and of the fp32 non-decay parameters (read in
//      fp32 by the forward) with peer loads. The fp32 masters of the four
//      decay matrices stay sharded (only the bf16 copy is used for compute)
//      and are gathered for checkpoints. NVLink bytes per rank and direction:
//      (N-1)/N * (4 + 2) bytes per parameter.
//
// Flags are epoch numbers (monotonic per exchange, no reset). Every wait is
// bounded by %globaltimer; on expiry the kernel records a status word that
// the host reads and skips the remaining work (no trap, the context stays
// usable). No TMA or bulk copy touches peer memory: only ld/st.global.
#include "../common/common.cuh"

namespace {

using bf16 = __nv_bfloat16;
constexpr int MAXR = 8;
// Small blocks with capped registers: every exchange kernel fits on an SM beside one persistent tcgen05 GEMM CTA
// (192 threads, <= 152 registers, <= 195 KB of shared memory), so an exchange running on the side stream under the
// next layer's GEMMs never holds an SM that a GEMM CTA waits for.
constexpr int THREADS = 128;
constexpr int THREADS_B = 256;  // update kernel: 4x the grid of the copy kernels

// Signal-buffer layout (32-bit words) of every rank.
constexpr int ARRIVE = 0;      // [MAXR] epoch of rank q's "gradients ready"
constexpr int NORMF = 8;       // [MAXR] epoch of rank q's published partial norm
constexpr int DONE = 16;       // [MAXR] epoch of rank q's updated shard
constexpr int STATUS = 24;     // nonzero after a timed-out wait: 1 = arrive, 2 = norm, 3 = updated shard
constexpr int COUNT_A = 25;    // block completion counters (local)
constexpr int COUNT_B = 26;
constexpr int WAITED = 27;     // rank whose flag was missing at the timeout
constexpr int NORM_SLOT = 32;  // [MAXR] float partial norm^2 of rank q
constexpr int STAT_SLOT = 40;  // [MAXR][3] float loss statistics of rank q
constexpr int PARTIAL = 64;    // [grid] float per-block partial norm^2 (local)
constexpr int SLICE = 1024;    // [update blocks] epoch of this rank's updated slice b (polled by peers)
constexpr int MAX_SLICES = 1024;
constexpr int SIG_WORDS = SLICE + MAX_SLICES;

struct Peers {
  float* grad[MAXR];
  float* param[MAXR];
  bf16* shadow[MAXR];
  unsigned* sig[MAXR];
};

struct Adam {
  float lr, beta1, beta2, eps, weight_decay, clip, bias1, bias2_sqrt;
  long decay_numel;
};

RT_DEVICE unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
RT_DEVICE void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
RT_DEVICE unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Thread-level bounded wait until sig[base + q] >= epoch for every q < world.
RT_DEVICE bool wait_all(unsigned* sig, int base, int world, unsigned epoch, unsigned long long limit_ns, int code) {
  const unsigned long long t0 = now_ns();
  for (int q = 0; q < world; ++q) {
    unsigned spins = 0;
    while ((int)(ld_acquire_sys(sig + base + q) - epoch) < 0) {
      if ((++spins & 63u) == 0 && now_ns() - t0 > limit_ns) {
        if (atomicCAS(sig + STATUS, 0u, (unsigned)code) == 0u) sig[WAITED] = (unsigned)q;  // first expiry only
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

RT_DEVICE float block_sum(float v, float* scratch) { return rt::block_sum(v, scratch); }

// ---------------------------------------------------------------- A: reduce-scatter + norm
template <int W>
__global__ void __launch_bounds__(THREADS, 4)
exchange_reduce_kernel(Peers peers, int rank, long lo4, long hi4, long tail_lo, long tail_hi,
                       const float* __restrict__ stats, unsigned epoch, unsigned long long limit_ns) {
  constexpr int world = W;
  constexpr int UNROLL = W <= 2 ? 8 : (W <= 4 ? 4 : 2);
  __shared__ float scratch[32];
  __shared__ int ok;
  unsigned* sig = peers.sig[rank];
  if (blockIdx.x == 0 && threadIdx.x < world) st_release_sys(peers.sig[threadIdx.x] + ARRIVE + rank, epoch);
  if (threadIdx.x == 0) ok = wait_all(sig, ARRIVE, world, epoch, limit_ns, 1);
  __syncthreads();
  if (!ok) return;
  float acc = 0.f;
  float4* mine = reinterpret_cast<float4*>(peers.grad[rank]);
  // UNROLL independent float4 per thread and rank in flight: NVLink loads need ~1-2 us of latency hidden.
  const long stride = (long)gridDim.x * THREADS;
  for (long i0 = lo4 + (long)blockIdx.x * THREADS + threadIdx.x; i0 < hi4; i0 += UNROLL * stride) {
    float4 v[UNROLL][W];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const long i = i0 + u * stride;
#pragma unroll
      for (int q = 0; q < W; ++q)
        if (i < hi4) v[u][q] = __ldcg(reinterpret_cast<const float4*>(peers.grad[q]) + i);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const long i = i0 + u * stride;
      if (i < hi4) {
        float4 s = v[u][0];
#pragma unroll
        for (int q = 1; q < W; ++q) { s.x += v[u][q].x; s.y += v[u][q].y; s.z += v[u][q].z; s.w += v[u][q].w; }
        mine[i] = s;
        acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
      }
    }
  }
  for (long i = tail_lo + (long)blockIdx.x * THREADS + threadIdx.x; i < tail_hi; i += (long)gridDim.x * THREADS) {
    float s = 0.f;
    for (int q = 0; q < world; ++q) s += peers.grad[q][i];
    peers.grad[rank][i] = s;
    acc += s * s;
  }
  acc = block_sum(acc, scratch);
  if (threadIdx.x == 0) {
    float* partial = reinterpret_cast<float*>(sig + PARTIAL);
    partial[blockIdx.x] = acc;
    __threadfence();
    const unsigned done = atomicAdd(sig + COUNT_A, 1u);
    if (done == gridDim.x - 1) {  // last block: publish this rank's norm^2 and statistics everywhere
      __threadfence();
      float total = 0.f;
      for (int b = 0; b < (int)gridDim.x; ++b) total += __ldcg(partial + b);
      const float s0 = stats[0], s1 = stats[1], s2 = stats[2];
      for (int q = 0; q < world; ++q) {
        float* slots = reinterpret_cast<float*>(peers.sig[q]);
        slots[NORM_SLOT + rank] = total;
        slots[STAT_SLOT + 3 * rank + 0] = s0;
        slots[STAT_SLOT + 3 * rank + 1] = s1;
        slots[STAT_SLOT + 3 * rank + 2] = s2;
      }
      __threadfence_system();
      for (int q = 0; q < world; ++q) st_release_sys(peers.sig[q] + NORMF + rank, epoch);
      sig[COUNT_A] = 0;
    }
  }
}

// ---------------------------------------------------------------- B: clip + AdamW + all-gather
RT_DEVICE float adam_one(float g, float& p, float& m, float& v, long i, const Adam& a, float step) {
  if (i < a.decay_numel) p *= 1.f - a.lr * a.weight_decay;
  m = m + (1.f - a.beta1) * (g - m);
  v = a.beta2 * v + (1.f - a.beta2) * g * g;
  p -= step * m / (sqrtf(v) / a.bias2_sqrt + a.eps);
  return p;
}

template <int W>
__global__ void __launch_bounds__(THREADS_B, 2)
exchange_update_kernel(Peers peers, int rank, long n, long lo4, long hi4, long tail_lo, long tail_hi,
                       float* __restrict__ m, float* __restrict__ v, float* __restrict__ stats,
                       float* __restrict__ report, Adam a, unsigned epoch, unsigned long long limit_ns) {
  constexpr int world = W;
  constexpr int UNROLL = 2;  // 8 independent 16-byte loads in flight per thread
  __shared__ int ok;
  unsigned* sig = peers.sig[rank];
  if (threadIdx.x == 0) ok = wait_all(sig, NORMF, world, epoch, limit_ns, 2);
  __syncthreads();
  if (!ok) return;
  const float* slots = reinterpret_cast<const float*>(sig);
  float norm2 = 0.f, s0 = 0.f, s1 = 0.f, count = 0.f;
  for (int q = 0; q < world; ++q) {  // same order on every rank: identical clip coefficient everywhere
    norm2 += __ldcg(slots + NORM_SLOT + q);
    s0 += __ldcg(slots + STAT_SLOT + 3 * q + 0);
    s1 += __ldcg(slots + STAT_SLOT + 3 * q + 1);
    count += __ldcg(slots + STAT_SLOT + 3 * q + 2);
  }
  const float inv = count > 0.f ? 1.f / count : 0.f;
  const float norm = sqrtf(norm2) * inv;
  const float gscale = inv * fminf(1.f, a.clip / (norm + 1e-6f));
  const float step = a.lr / a.bias1;
  float4* __restrict__ p4s = reinterpret_cast<float4*>(peers.param[rank]);
  float4* __restrict__ g4s = reinterpret_cast<float4*>(peers.grad[rank]);
  float4* __restrict__ m4s = reinterpret_cast<float4*>(m);
  float4* __restrict__ v4s = reinterpret_cast<float4*>(v);
  uint2* __restrict__ sh2 = reinterpret_cast<uint2*>(peers.shadow[rank]);
  const long stride = (long)gridDim.x * THREADS_B;
  for (long i0 = lo4 + (long)blockIdx.x * THREADS_B + threadIdx.x; i0 < hi4; i0 += UNROLL * stride) {
    float4 g4[UNROLL], p4[UNROLL], m4[UNROLL], v4[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const long i = i0 + u * stride;
      if (i < hi4) {
        g4[u] = __ldcs(g4s + i);
        p4[u] = p4s[i];
        m4[u] = __ldcs(m4s + i);
        v4[u] = __ldcs(v4s + i);
      }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const long i = i0 + u * stride;
      if (i < hi4) {
        const long e = 4 * i;
        adam_one(g4[u].x * gscale, p4[u].x, m4[u].x, v4[u].x, e + 0, a, step);
        adam_one(g4[u].y * gscale, p4[u].y, m4[u].y, v4[u].y, e + 1, a, step);
        adam_one(g4[u].z * gscale, p4[u].z, m4[u].z, v4[u].z, e + 2, a, step);
        adam_one(g4[u].w * gscale, p4[u].w, m4[u].w, v4[u].w, e + 3, a, step);
        __stcs(m4s + i, m4[u]);
        __stcs(v4s + i, v4[u]);
        p4s[i] = p4[u];
        __nv_bfloat162 lo = __floats2bfloat162_rn(p4[u].x, p4[u].y), hi = __floats2bfloat162_rn(p4[u].z, p4[u].w);
        uint2 packed;
        packed.x = *reinterpret_cast<unsigned*>(&lo);
        packed.y = *reinterpret_cast<unsigned*>(&hi);
        sh2[i] = packed;
      }
    }
  }
  float* p = peers.param[rank];
  float* g = peers.grad[rank];
  bf16* sh = peers.shadow[rank];
  for (long i = tail_lo + (long)blockIdx.x * THREADS_B + threadIdx.x; i < tail_hi; i += stride) {
    float pv = p[i], mv = m[i], vv = v[i];
    adam_one(g[i] * gscale, pv, mv, vv, i, a, step);
    m[i] = mv;
    v[i] = vv;
    p[i] = pv;
    sh[i] = __float2bfloat16_rn(pv);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    report[0] = s0;
    report[1] = s1;
    report[2] = count;
    report[3] = norm;
    report[4] = (!isfinite(norm) || count <= 0.f) ? 1.f : 0.f;
    stats[0] = stats[1] = stats[2] = 0.f;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned done = atomicAdd(sig + COUNT_B, 1u);
    if (done == gridDim.x - 1) {  // last block: this rank's shard is final; peers may pull it
      __threadfence_system();
      for (int q = 0; q < world; ++q) st_release_sys(peers.sig[q] + DONE + rank, epoch);
      sig[COUNT_B] = 0;
    }
  }
}

// ---------------------------------------------------------------- C: all-gather by pulling peers' shards
// Pulls every other rank's updated shard of the bf16 weight copy (16-byte loads, UNROLL in flight per thread)
// and the fp32 parameters of the non-decay range [decay4 * 4, n) (small vectors and LoRA factors read in fp32 by
// the forward). The decay-group fp32 masters stay sharded until gather_state. No completion flags are needed:
// a peer changes its shard again only in its next update of this layer, which waits for this rank's next norm.
template <int W>
__global__ void __launch_bounds__(THREADS, 4)
exchange_gather_kernel(Peers peers, int rank, long n, long n8, long decay4, unsigned epoch,
                       unsigned long long limit_ns) {
  constexpr int UNROLL = 8;
  __shared__ int ok;
  unsigned* sig = peers.sig[rank];
  if (threadIdx.x == 0) ok = wait_all(sig, DONE, W, epoch, limit_ns, 3);
  __syncthreads();
  if (!ok) return;
  const long stride = (long)gridDim.x * THREADS;
  const long t0 = (long)blockIdx.x * THREADS + threadIdx.x;
  // bf16 copy: concatenated index space over the W-1 peer shards (units of 8 elements)
#pragma unroll 1
  for (int k = 1; k < W; ++k) {
    const int q = (rank + k) % W;
    const long lo = n8 * q / W, hi = n8 * (q + 1) / W;
    const uint4* src = reinterpret_cast<const uint4*>(peers.shadow[q]);
    uint4* dst = reinterpret_cast<uint4*>(peers.shadow[rank]);
    for (long i0 = lo + t0; i0 < hi; i0 += UNROLL * stride) {
      uint4 r[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u)
        if (i0 + u * stride < hi) r[u] = __ldcg(src + i0 + u * stride);
#pragma unroll
      for (int u = 0; u < UNROLL; ++u)
        if (i0 + u * stride < hi) dst[i0 + u * stride] = r[u];
    }
    // fp32 parameters of the non-decay range inside shard q (units of 4 elements)
    const long flo = lo * 2 > decay4 ? lo * 2 : decay4, fhi = hi * 2;
    const float4* fsrc = reinterpret_cast<const float4*>(peers.param[q]);
    float4* fdst = reinterpret_cast<float4*>(peers.param[rank]);
    for (long i0 = flo + t0; i0 < fhi; i0 += UNROLL * stride) {
      float4 r[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u)
        if (i0 + u * stride < fhi) r[u] = __ldcg(fsrc + i0 + u * stride);
#pragma unroll
      for (int u = 0; u < UNROLL; ++u)
        if (i0 + u * stride < fhi) fdst[i0 + u * stride] = r[u];
    }
  }
  if (rank != W - 1) {  // scalar tail [8 * n8, n), owned by the last rank
    for (long i = 8 * n8 + t0; i < n; i += stride) {
      peers.shadow[rank][i] = peers.shadow[W - 1][i];
      peers.param[rank][i] = peers.param[W - 1][i];
    }
  }
}

// ---------------------------------------------------------------- B+C fused: slice updates and slice pulls at once
// One kernel with two roles. Blocks [0, U) update this rank's shard slice by slice (S slices, slice s by block
// s mod U, in increasing s): clip + AdamW into the fp32 master, moments and bf16 copy, then raise the slice's flag.
// Blocks [U, U + P) pull: slice s of every peer's shard (bf16 copy and fp32 non-decay parameters), each as soon
// as that peer's flag for it is up. Local HBM-bound updates and NVLink pulls run at the same time, and no grid-wide
// barrier separates them. Update blocks have the lower indices, so they are dispatched before any pull block can
// occupy an SM; pull waits only ever point at other ranks' update blocks. Slices are contiguous ranges of 8-element
// units; the scalar tail [8 n8, n) belongs to the last rank's last slice.
RT_DEVICE void slice_of(long n8, int q, int W, int sl, int S, long& lo, long& hi) {
  const long slo = n8 * q / W, shi = n8 * (q + 1) / W;
  lo = slo + (shi - slo) * sl / S;
  hi = slo + (shi - slo) * (sl + 1) / S;
}

template <int W>
__global__ void __launch_bounds__(THREADS_B, 2)
exchange_update_pull_kernel(Peers peers, int rank, long n, long n8, long decay4, int U, int S, float* __restrict__ m,
                            float* __restrict__ v, float* __restrict__ stats, float* __restrict__ report, Adam a,
                            unsigned epoch, unsigned long long limit_ns) {
  constexpr int world = W;
  constexpr int UNROLL = 2;
  __shared__ int ok;
  unsigned* sig = peers.sig[rank];
  const int b = blockIdx.x;
  if (b < U) {
    // ---------------- update role
    if (threadIdx.x == 0) ok = wait_all(sig, NORMF, world, epoch, limit_ns, 2);
    __syncthreads();
    if (!ok) return;
    const float* slots = reinterpret_cast<const float*>(sig);
    float norm2 = 0.f, s0 = 0.f, s1 = 0.f, count = 0.f;
    for (int q = 0; q < world; ++q) {  // same order on every rank: identical clip coefficient everywhere
      norm2 += __ldcg(slots + NORM_SLOT + q);
      s0 += __ldcg(slots + STAT_SLOT + 3 * q + 0);
      s1 += __ldcg(slots + STAT_SLOT + 3 * q + 1);
      count += __ldcg(slots + STAT_SLOT + 3 * q + 2);
    }
    const float inv = count > 0.f ? 1.f / count : 0.f;
    const float norm = sqrtf(norm2) * inv;
    const float gscale = inv * fminf(1.f, a.clip / (norm + 1e-6f));
    const float step = a.lr / a.bias1;
    float4* __restrict__ p4s = reinterpret_cast<float4*>(peers.param[rank]);
    const float4* __restrict__ g4s = reinterpret_cast<const float4*>(peers.grad[rank]);
    float4* __restrict__ m4s = reinterpret_cast<float4*>(m);
    float4* __restrict__ v4s = reinterpret_cast<float4*>(v);
    uint2* __restrict__ sh2 = reinterpret_cast<uint2*>(peers.shadow[rank]);
#pragma unroll 1
    for (int sl = b; sl < S; sl += U) {
      long lo, hi;
      slice_of(n8, rank, W, sl, S, lo, hi);
      const long lo4 = 2 * lo, hi4 = 2 * hi;
      for (long i0 = lo4 + threadIdx.x; i0 < hi4; i0 += UNROLL * THREADS_B) {
        float4 g4[UNROLL], p4[UNROLL], m4[UNROLL], v4[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
          const long i = i0 + u * THREADS_B;
          if (i < hi4) {
            g4[u] = __ldcs(g4s + i);
            p4[u] = p4s[i];
            m4[u] = __ldcs(m4s + i);
            v4[u] = __ldcs(v4s + i);
          }
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
          const long i = i0 + u * THREADS_B;
          if (i < hi4) {
            const long e = 4 * i;
            adam_one(g4[u].x * gscale, p4[u].x, m4[u].x, v4[u].x, e + 0, a, step);
            adam_one(g4[u].y * gscale, p4[u].y, m4[u].y, v4[u].y, e + 1, a, step);
            adam_one(g4[u].z * gscale, p4[u].z, m4[u].z, v4[u].z, e + 2, a, step);
            adam_one(g4[u].w * gscale, p4[u].w, m4[u].w, v4[u].w, e + 3, a, step);
            __stcs(m4s + i, m4[u]);
            __stcs(v4s + i, v4[u]);
            p4s[i] = p4[u];
            __nv_bfloat162 l2 = __floats2bfloat162_rn(p4[u].x, p4[u].y);
            __nv_bfloat162 h2 = __floats2bfloat162_rn(p4[u].z, p4[u].w);
            uint2 packed;
            packed.x = *reinterpret_cast<unsigned*>(&l2);
            packed.y = *reinterpret_cast<unsigned*>(&h2);
            sh2[i] = packed;
          }
        }
      }
      if (rank == W - 1 && sl == S - 1) {  // scalar tail
        float* p = peers.param[rank];
        const float* g = peers.grad[rank];
        bf16* sh = peers.shadow[rank];
        for (long i = 8 * n8 + threadIdx.x; i < n; i += THREADS_B) {
          float pv = p[i], mv = m[i], vv = v[i];
          adam_one(g[i] * gscale, pv, mv, vv, i, a, step);
          m[i] = mv;
          v[i] = vv;
          p[i] = pv;
          sh[i] = __float2bfloat16_rn(pv);
        }
      }
      __threadfence_system();
      __syncthreads();
      if (threadIdx.x == 0) st_release_sys(sig + SLICE + sl, epoch);  // peers poll this word
    }
    if (b == 0 && threadIdx.x == 0) {
      report[0] = s0;
      report[1] = s1;
      report[2] = count;
      report[3] = norm;
      report[4] = (!isfinite(norm) || count <= 0.f) ? 1.f : 0.f;
      stats[0] = stats[1] = stats[2] = 0.f;
    }
    return;
  }
  // ---------------- pull role
  const int P = gridDim.x - U;
  constexpr int PU = 4;
#pragma unroll 1
  for (int sl = b - U; sl < S; sl += P) {
#pragma unroll 1
    for (int k = 1; k < W; ++k) {
      const int q = (rank + k) % W;
      if (threadIdx.x == 0) {
        const unsigned long long t0 = now_ns();
        unsigned spins = 0;
        ok = 1;
        while ((int)(ld_acquire_sys(peers.sig[q] + SLICE + sl) - epoch) < 0) {
          if ((++spins & 63u) == 0 && now_ns() - t0 > limit_ns) {
            if (atomicCAS(sig + STATUS, 0u, 3u) == 0u) sig[WAITED] = (unsigned)q;
            ok = 0;
            break;
          }
          __nanosleep(128);
        }
      }
      __syncthreads();
      if (!ok) return;
      long qlo, qhi;
      slice_of(n8, q, W, sl, S, qlo, qhi);
      const uint4* src = reinterpret_cast<const uint4*>(peers.shadow[q]);
      uint4* dst = reinterpret_cast<uint4*>(peers.shadow[rank]);
      for (long i0 = qlo + threadIdx.x; i0 < qhi; i0 += PU * THREADS_B) {
        uint4 r[PU];
#pragma unroll
        for (int u = 0; u < PU; ++u)
          if (i0 + u * THREADS_B < qhi) r[u] = __ldcg(src + i0 + u * THREADS_B);
#pragma unroll
        for (int u = 0; u < PU; ++u)
          if (i0 + u * THREADS_B < qhi) dst[i0 + u * THREADS_B] = r[u];
      }
      const long flo = 2 * qlo > decay4 ? 2 * qlo : decay4, fhi = 2 * qhi;  // fp32 non-decay parameters
      const float4* fsrc = reinterpret_cast<const float4*>(peers.param[q]);
      float4* fdst = reinterpret_cast<float4*>(peers.param[rank]);
      for (long i0 = flo + threadIdx.x; i0 < fhi; i0 += PU * THREADS_B) {
        float4 r[PU];
#pragma unroll
        for (int u = 0; u < PU; ++u)
          if (i0 + u * THREADS_B < fhi) r[u] = __ldcg(fsrc + i0 + u * THREADS_B);
#pragma unroll
        for (int u = 0; u < PU; ++u)
          if (i0 + u * THREADS_B < fhi) fdst[i0 + u * THREADS_B] = r[u];
      }
      if (q == W - 1 && sl == S - 1) {  // scalar tail of the last rank
        for (long i = 8 * n8 + threadIdx.x; i < n; i += THREADS_B) {
          peers.shadow[rank][i] = peers.shadow[q][i];
          peers.param[rank][i] = peers.param[q][i];
        }
      }
      __syncthreads();  // `ok` is reused by the next wait
    }
  }
}

// Shard of rank r: float4 body [lo4, hi4) in units of 8 elements, plus the scalar tail (owned by the last rank).
void shard(long n, int rank, int world, long& lo4, long& hi4, long& tail_lo, long& tail_hi) {
  const long n8 = n / 8;
  lo4 = 2 * (n8 * rank / world);
  hi4 = 2 * (n8 * (rank + 1) / world);
  tail_lo = rank == world - 1 ? n8 * 8 : n;
  tail_hi = n;
}

}  // namespace

extern "C" int rt_exchange_signal_words() { return SIG_WORDS; }

// grads/params/shadows/sigs: `world` device pointers each (index = rank; peers mapped into this process).
// m, v: this rank's moment buffers; stats: this rank's [3] loss sums (cleared); report: [5].
// All pointers 16-byte aligned. `blocks` <= SLICE - PARTIAL. mode 0: reduce kernel + update/pull kernel; 1: reduce,
// update and all-gather kernels.
extern "C" cudaError_t rt_exchange_update(float* const* grads, float* const* params, void* const* shadows,
                                          unsigned* const* sigs, int rank, int world, long n, float* m, float* v,
                                          float* stats, float* report, float lr, float beta1, float beta2, float eps,
                                          float weight_decay, float clip, int step, long decay_numel,
                                          unsigned epoch, double limit_s, int blocks, int mode, cudaStream_t s) {
  if (world < 1 || world > MAXR || rank < 0 || rank >= world || blocks < 1 || blocks > SLICE - PARTIAL)
    return cudaErrorInvalidValue;
  Peers peers = {};
  for (int q = 0; q < world; ++q) {
    peers.grad[q] = grads[q];
    peers.param[q] = params[q];
    peers.shadow[q] = reinterpret_cast<bf16*>(shadows[q]);
    peers.sig[q] = sigs[q];
    if ((reinterpret_cast<uintptr_t>(grads[q]) | reinterpret_cast<uintptr_t>(params[q])) & 15 ||
        reinterpret_cast<uintptr_t>(shadows[q]) & 15)
      return cudaErrorMisalignedAddress;
  }
  long lo4, hi4, tail_lo, tail_hi;
  shard(n, rank, world, lo4, hi4, tail_lo, tail_hi);
  const unsigned long long limit_ns = (unsigned long long)(limit_s * 1e9);
  Adam a;
  a.lr = lr; a.beta1 = beta1; a.beta2 = beta2; a.eps = eps; a.weight_decay = weight_decay; a.clip = clip;
  a.bias1 = (float)(1.0 - pow((double)beta1, (double)step));
  a.bias2_sqrt = (float)sqrt(1.0 - pow((double)beta2, (double)step));
  a.decay_numel = decay_numel;
  const long n8 = n / 8, decay4 = decay_numel / 4;
  // fused update + pull (default): `slices` blocks, each one slice of every shard; else three-phase kernels
  const bool fused = mode == 0;
  const int upd = 2 * blocks;                      // update blocks (as many pull blocks)
  const int slices = 8 * blocks < MAX_SLICES ? 8 * blocks : MAX_SLICES;  // 4 slices per update block
  switch (world) {
#define RT_EXCHANGE_CASE(W)                                                                                        \
  case W:                                                                                                          \
    exchange_reduce_kernel<W><<<blocks, THREADS, 0, s>>>(peers, rank, lo4, hi4, tail_lo, tail_hi, stats, epoch,   \
                                                         limit_ns);                                                \
    RT_CUDA_CHECK(cudaGetLastError());                                                                             \
    if (fused) {                                                                                                   \
      exchange_update_pull_kernel<W><<<2 * upd, THREADS_B, 0, s>>>(peers, rank, n, n8, decay4, upd, slices, m, v,    \
                                                                   stats, report, a, epoch, limit_ns);             \
    } else {                                                                                                       \
      exchange_update_kernel<W><<<4 * blocks, THREADS_B, 0, s>>>(peers, rank, n, lo4, hi4, tail_lo, tail_hi, m, v,  \
                                                                 stats, report, a, epoch, limit_ns);               \
      RT_CUDA_CHECK(cudaGetLastError());                                                                           \
      exchange_gather_kernel<W><<<blocks, THREADS, 0, s>>>(peers, rank, n, n8, decay4, epoch, limit_ns);           \
    }                                                                                                              \
    break;
    RT_EXCHANGE_CASE(1)
    RT_EXCHANGE_CASE(2)
    RT_EXCHANGE_CASE(3)
    RT_EXCHANGE_CASE(4)
    RT_EXCHANGE_CASE(5)
    RT_EXCHANGE_CASE(6)
    RT_EXCHANGE_CASE(7)
    RT_EXCHANGE_CASE(8)
#undef RT_EXCHANGE_CASE
  }
  return cudaGetLastError();
}

// Shard bounds (elements) of `rank`: [lo, hi) in the float4 body plus the scalar tail.
extern "C" void rt_exchange_shard(long n, int rank, int world, long* out4) {
  long lo4, hi4, tail_lo, tail_hi;
  shard(n, rank, world, lo4, hi4, tail_lo, tail_hi);
  out4[0] = lo4 * 4;
  out4[1] = hi4 * 4;
  out4[2] = tail_lo;
  out4[3] = tail_hi;
}

// ---------------------------------------------------------------- IPC mapping of caching-allocator blocks
// Exports the allocation that contains `ptr`: its IPC handle and the offset of `ptr` inside it.
typedef int (*GetRangeFn)(unsigned long long*, size_t*, unsigned long long);

extern "C" cudaError_t rt_ipc_export(const void* ptr, void* handle64, long* offset) {
  static GetRangeFn fn = nullptr;
  if (!fn) {
    void* sym = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &sym, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return cudaErrorNotSupported;
    fn = reinterpret_cast<GetRangeFn>(sym);
  }
  unsigned long long base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<unsigned long long>(ptr)) != 0) return cudaErrorInvalidDevicePointer;
  cudaIpcMemHandle_t h;
  RT_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  memcpy(handle64, &h, sizeof(h));
  *offset = (long)(reinterpret_cast<unsigned long long>(ptr) - base);
  return cudaSuccess;
}

extern "C" cudaError_t rt_ipc_open(const void* handle64, void** base) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  return cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
}

extern "C" cudaError_t rt_ipc_close(void* base) { return cudaIpcCloseMemHandle(base); }
