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
//   B  update + all-gather: after every rank's norm is published, each rank
//      forms the same global norm (fixed summation order), clips, applies
//      AdamW to its shard, and stores the new fp32 parameters and their bf16
//      copy into every rank's buffers (peer stores); it then clears its whole
//      local gradient (all peers have finished reading it) and its loss
//      statistics, writes the report and raises its "done" flag everywhere;
//   C  one warp waits until every rank is done, so later work on the stream
//      sees the complete parameters.
//
// Flags are epoch numbers (monotonic per exchange, no reset). Every wait is
// bounded by %globaltimer; on expiry the kernel records a status word that
// the host reads and skips the remaining work (no trap, the context stays
// usable). No TMA or bulk copy touches peer memory: only ld/st.global.
#include "../common/common.cuh"

namespace {

using bf16 = __nv_bfloat16;
constexpr int MAXR = 8;
constexpr int THREADS = 512;

// Signal-buffer layout (32-bit words) of every rank.
constexpr int ARRIVE = 0;      // [MAXR] epoch of rank q's "gradients ready"
constexpr int NORMF = 8;       // [MAXR] epoch of rank q's published partial norm
constexpr int DONE = 16;       // [MAXR] epoch of rank q's finished parameter stores
constexpr int STATUS = 24;     // nonzero after a timed-out wait: 1 = arrive, 2 = norm, 3 = done
constexpr int COUNT_A = 25;    // block completion counters (local)
constexpr int COUNT_B = 26;
constexpr int WAITED = 27;     // rank whose flag was missing at the timeout
constexpr int NORM_SLOT = 32;  // [MAXR] float partial norm^2 of rank q
constexpr int STAT_SLOT = 40;  // [MAXR][3] float loss statistics of rank q
constexpr int PARTIAL = 64;    // [grid] float per-block partial norm^2 (local)
constexpr int SIG_WORDS = 1024;

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
        atomicCAS(sig + STATUS, 0u, (unsigned)code);
        sig[WAITED] = (unsigned)q;
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

RT_DEVICE float block_sum(float v, float* scratch) { return rt::block_sum(v, scratch); }

// ---------------------------------------------------------------- A: reduce-scatter + norm
__global__ void __launch_bounds__(THREADS)
exchange_reduce_kernel(Peers peers, int rank, int world, long lo4, long hi4, long tail_lo, long tail_hi,
                       const float* __restrict__ stats, unsigned epoch, unsigned long long limit_ns) {
  __shared__ float scratch[32];
  __shared__ int ok;
  unsigned* sig = peers.sig[rank];
  if (blockIdx.x == 0 && threadIdx.x < world) st_release_sys(peers.sig[threadIdx.x] + ARRIVE + rank, epoch);
  if (threadIdx.x == 0) ok = wait_all(sig, ARRIVE, world, epoch, limit_ns, 1);
  __syncthreads();
  if (!ok) return;
  float acc = 0.f;
  float4* mine = reinterpret_cast<float4*>(peers.grad[rank]);
  for (long i = lo4 + (long)blockIdx.x * THREADS + threadIdx.x; i < hi4; i += (long)gridDim.x * THREADS) {
    float4 v[MAXR];
#pragma unroll
    for (int q = 0; q < MAXR; ++q)
      if (q < world) v[q] = reinterpret_cast<const float4*>(peers.grad[q])[i];
    float4 s = v[0];
#pragma unroll
    for (int q = 1; q < MAXR; ++q)
      if (q < world) { s.x += v[q].x; s.y += v[q].y; s.z += v[q].z; s.w += v[q].w; }
    mine[i] = s;
    acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
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

__global__ void __launch_bounds__(THREADS)
exchange_update_kernel(Peers peers, int rank, int world, long n, long lo4, long hi4, long tail_lo, long tail_hi,
                       float* __restrict__ m, float* __restrict__ v, float* __restrict__ stats,
                       float* __restrict__ report, Adam a, unsigned epoch, unsigned long long limit_ns) {
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
  float* p = peers.param[rank];
  float* g = peers.grad[rank];
  for (long i = lo4 + (long)blockIdx.x * THREADS + threadIdx.x; i < hi4; i += (long)gridDim.x * THREADS) {
    const float4 g4 = reinterpret_cast<const float4*>(g)[i];
    reinterpret_cast<float4*>(g)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 p4 = reinterpret_cast<const float4*>(p)[i];
    float4 m4 = reinterpret_cast<const float4*>(m)[i];
    float4 v4 = reinterpret_cast<const float4*>(v)[i];
    const long e = 4 * i;
    adam_one(g4.x * gscale, p4.x, m4.x, v4.x, e + 0, a, step);
    adam_one(g4.y * gscale, p4.y, m4.y, v4.y, e + 1, a, step);
    adam_one(g4.z * gscale, p4.z, m4.z, v4.z, e + 2, a, step);
    adam_one(g4.w * gscale, p4.w, m4.w, v4.w, e + 3, a, step);
    reinterpret_cast<float4*>(m)[i] = m4;
    reinterpret_cast<float4*>(v)[i] = v4;
    __nv_bfloat162 lo = __floats2bfloat162_rn(p4.x, p4.y), hi = __floats2bfloat162_rn(p4.z, p4.w);
    uint2 packed;
    packed.x = *reinterpret_cast<unsigned*>(&lo);
    packed.y = *reinterpret_cast<unsigned*>(&hi);
#pragma unroll
    for (int q = 0; q < MAXR; ++q) {
      if (q < world) {
        reinterpret_cast<float4*>(peers.param[q])[i] = p4;
        reinterpret_cast<uint2*>(peers.shadow[q])[i] = packed;
      }
    }
  }
  for (long i = tail_lo + (long)blockIdx.x * THREADS + threadIdx.x; i < tail_hi; i += (long)gridDim.x * THREADS) {
    float pv = p[i], mv = m[i], vv = v[i];
    adam_one(g[i] * gscale, pv, mv, vv, i, a, step);
    g[i] = 0.f;
    m[i] = mv;
    v[i] = vv;
    for (int q = 0; q < world; ++q) {
      peers.param[q][i] = pv;
      peers.shadow[q][i] = __float2bfloat16_rn(pv);
    }
  }
  // Clear the rest of the local gradient: every peer has finished reading it (their norms are published).
  for (long i = (long)blockIdx.x * THREADS + threadIdx.x; i < n / 4; i += (long)gridDim.x * THREADS)
    if (i < lo4 || i >= hi4) reinterpret_cast<float4*>(g)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (long i = (n / 4) * 4 + (long)blockIdx.x * THREADS + threadIdx.x; i < tail_lo; i += (long)gridDim.x * THREADS)
    g[i] = 0.f;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    report[0] = s0;
    report[1] = s1;
    report[2] = count;
    report[3] = norm;
    report[4] = (!isfinite(norm) || count <= 0.f) ? 1.f : 0.f;
    stats[0] = stats[1] = stats[2] = 0.f;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned done = atomicAdd(sig + COUNT_B, 1u);
    if (done == gridDim.x - 1) {
      __threadfence_system();
      for (int q = 0; q < world; ++q) st_release_sys(peers.sig[q] + DONE + rank, epoch);
      sig[COUNT_B] = 0;
    }
  }
}

// ---------------------------------------------------------------- C: wait for every rank's stores
__global__ void exchange_wait_kernel(unsigned* sig, int world, unsigned epoch, unsigned long long limit_ns) {
  if (threadIdx.x == 0) wait_all(sig, DONE, world, epoch, limit_ns, 3);
}

// Shard of rank r in float4 units plus the scalar tail (owned by the last rank).
void shard(long n, int rank, int world, long& lo4, long& hi4, long& tail_lo, long& tail_hi) {
  const long n4 = n / 4;
  lo4 = n4 * rank / world;
  hi4 = n4 * (rank + 1) / world;
  tail_lo = rank == world - 1 ? n4 * 4 : n;
  tail_hi = n;
}

}  // namespace

extern "C" int rt_exchange_signal_words() { return SIG_WORDS; }

// grads/params/shadows/sigs: `world` device pointers each (index = rank; peers mapped into this process).
// m, v: this rank's moment buffers; stats: this rank's [3] loss sums (cleared); report: [5].
// All pointers 16-byte aligned. `blocks` <= SIG_WORDS - PARTIAL.
extern "C" cudaError_t rt_exchange_update(float* const* grads, float* const* params, void* const* shadows,
                                          unsigned* const* sigs, int rank, int world, long n, float* m, float* v,
                                          float* stats, float* report, float lr, float beta1, float beta2, float eps,
                                          float weight_decay, float clip, int step, long decay_numel,
                                          unsigned epoch, double limit_s, int blocks, cudaStream_t s) {
  if (world < 1 || world > MAXR || rank < 0 || rank >= world || blocks < 1 || blocks > SIG_WORDS - PARTIAL)
    return cudaErrorInvalidValue;
  Peers peers = {};
  for (int q = 0; q < world; ++q) {
    peers.grad[q] = grads[q];
    peers.param[q] = params[q];
    peers.shadow[q] = reinterpret_cast<bf16*>(shadows[q]);
    peers.sig[q] = sigs[q];
    if ((reinterpret_cast<uintptr_t>(grads[q]) | reinterpret_cast<uintptr_t>(params[q])) & 15 ||
        reinterpret_cast<uintptr_t>(shadows[q]) & 7)
      return cudaErrorMisalignedAddress;
  }
  long lo4, hi4, tail_lo, tail_hi;
  shard(n, rank, world, lo4, hi4, tail_lo, tail_hi);
  const unsigned long long limit_ns = (unsigned long long)(limit_s * 1e9);
  exchange_reduce_kernel<<<blocks, THREADS, 0, s>>>(peers, rank, world, lo4, hi4, tail_lo, tail_hi, stats, epoch,
                                                     limit_ns);
  RT_CUDA_CHECK(cudaGetLastError());
  Adam a;
  a.lr = lr; a.beta1 = beta1; a.beta2 = beta2; a.eps = eps; a.weight_decay = weight_decay; a.clip = clip;
  a.bias1 = (float)(1.0 - pow((double)beta1, (double)step));
  a.bias2_sqrt = (float)sqrt(1.0 - pow((double)beta2, (double)step));
  a.decay_numel = decay_numel;
  exchange_update_kernel<<<blocks, THREADS, 0, s>>>(peers, rank, world, n, lo4, hi4, tail_lo, tail_hi, m, v, stats,
                                                     report, a, epoch, limit_ns);
  RT_CUDA_CHECK(cudaGetLastError());
  exchange_wait_kernel<<<1, 32, 0, s>>>(sigs[rank], world, epoch, limit_ns);
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
