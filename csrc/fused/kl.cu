// KL(teacher || student) over the vocabulary in one pass over both logit rows: each row is split into segments
// (enough blocks to fill the GPU), each segment reduces to an online triple, a second kernel merges a row's triples.
//
// Each thread keeps an online triple over its slice of the row:
//   m_t = max t,  Z_t = sum exp(t - m_t),  A = sum exp(t - m_t) (t - s),  and m_s, Z_s for the student,
// and triples merge by rescaling with exp(m_old - m_new) (threads, then warps, then segments). Then
//   KL = sum_v p_t (log p_t - log p_s) = A / Z_t - (m_t + log Z_t) + (m_s + log Z_s).
// Replaces two full log_softmax passes and the elementwise product of the reference's kl_sum
// (theseus/losses.py:27-30) on the validation path (theseus/validation.py:135-141).
#include "../common/common.cuh"

namespace {

struct Online {
  float mt, zt, a, ms, zs;
};

__device__ __forceinline__ void push(Online& o, float t, float s) {
  if (t > o.mt) {
    const float r = expf(o.mt - t);  // exp(-inf) = 0 on the first element
    o.zt *= r;
    o.a *= r;
    o.mt = t;
  }
  const float e = expf(t - o.mt);
  o.zt += e;
  o.a += e * (t - s);
  if (s > o.ms) {
    o.zs *= expf(o.ms - s);
    o.ms = s;
  }
  o.zs += expf(s - o.ms);
}

__device__ __forceinline__ Online merge(const Online& x, const Online& y) {
  Online o;
  o.mt = fmaxf(x.mt, y.mt);
  const float rx = x.zt > 0.f ? expf(x.mt - o.mt) : 0.f, ry = y.zt > 0.f ? expf(y.mt - o.mt) : 0.f;
  o.zt = x.zt * rx + y.zt * ry;
  o.a = x.a * rx + y.a * ry;
  o.ms = fmaxf(x.ms, y.ms);
  o.zs = (x.zs > 0.f ? x.zs * expf(x.ms - o.ms) : 0.f) + (y.zs > 0.f ? y.zs * expf(y.ms - o.ms) : 0.f);
  return o;
}

__device__ __forceinline__ Online block_merge(Online o, Online* part) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    Online y;
    y.mt = __shfl_down_sync(0xffffffffu, o.mt, off);
    y.zt = __shfl_down_sync(0xffffffffu, o.zt, off);
    y.a = __shfl_down_sync(0xffffffffu, o.a, off);
    y.ms = __shfl_down_sync(0xffffffffu, o.ms, off);
    y.zs = __shfl_down_sync(0xffffffffu, o.zs, off);
    o = merge(o, y);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) part[warp] = o;
  __syncthreads();
  Online r = part[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) r = merge(r, part[w]);
  return r;
}

// Block (row, seg) reduces elements [seg V / S, (seg + 1) V / S) of a row to one triple. Each thread first loads
// BATCH elements of both rows (independent loads in flight), then folds them into its triple.
template <typename T>
__global__ void __launch_bounds__(256) kl_partial_kernel(const T* __restrict__ student, const T* __restrict__ teacher,
                                                         long V, long ld_s, long ld_t, int S, Online* __restrict__ out) {
  constexpr int BATCH = 8;
  __shared__ Online part[8];
  const long row = blockIdx.x;
  const int seg = blockIdx.y;
  const long lo = V * seg / S, hi = V * (seg + 1) / S;
  const T* s = student + row * ld_s;
  const T* t = teacher + row * ld_t;
  Online o{-INFINITY, 0.f, 0.f, -INFINITY, 0.f};
  for (long v0 = lo + threadIdx.x; v0 < hi; v0 += (long)BATCH * blockDim.x) {
    float tv[BATCH], sv[BATCH];
#pragma unroll
    for (int k = 0; k < BATCH; ++k) {
      const long v = v0 + (long)k * blockDim.x;
      tv[k] = v < hi ? rt::to_f<T>(__ldg(t + v)) : -INFINITY;
      sv[k] = v < hi ? rt::to_f<T>(__ldg(s + v)) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < BATCH; ++k)
      if (v0 + (long)k * blockDim.x < hi) push(o, tv[k], sv[k]);
  }
  const Online r = block_merge(o, part);
  if (threadIdx.x == 0) out[row * S + seg] = r;
}

// out[row] from the row's S partial triples (fixed order: deterministic).
__global__ void kl_finish_kernel(const Online* __restrict__ part, long rows, int S, float* __restrict__ out) {
  const long row = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  Online r = part[row * S];
  for (int k = 1; k < S; ++k) r = merge(r, part[row * S + k]);
  out[row] = r.a / r.zt - (r.mt + logf(r.zt)) + (r.ms + logf(r.zs));
}

}  // namespace

// Segments per row so that rows x segments fills the GPU about twice (one to 64 per row).
extern "C" int rt_kl_segments(long rows, long V) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  long seg = (2L * sms + rows - 1) / (rows > 0 ? rows : 1);
  seg = seg < 1 ? 1 : (seg > 64 ? 64 : seg);
  while (seg > 1 && V / seg < 2048) --seg;  // keep a few thousand elements per block
  return (int)seg;
}

// Floats of scratch rt_kl_rows needs for `rows` rows split into `segments` (five per partial triple).
extern "C" long rt_kl_workspace_floats(long rows, int segments) { return rows * segments * 5; }

// out[r] = KL(softmax(teacher[r]) || softmax(student[r])) for rows r < rows; dtype 1 = bf16, 0 = fp32.
// work: rt_kl_workspace_floats(rows, segments) floats (4-byte aligned) for the per-segment partial triples.
extern "C" cudaError_t rt_kl_rows(int dtype, const void* student, const void* teacher, long rows, long V, long ld_s,
                                  long ld_t, int segments, float* work, float* out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if (V <= 0 || segments < 1) return cudaErrorInvalidValue;
  Online* part = reinterpret_cast<Online*>(work);
  const dim3 grid((unsigned)rows, (unsigned)segments);
  if (dtype == 1)
    kl_partial_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>((const __nv_bfloat16*)student,
                                                              (const __nv_bfloat16*)teacher, V, ld_s, ld_t, segments,
                                                              part);
  else
    kl_partial_kernel<float><<<grid, 256, 0, stream>>>((const float*)student, (const float*)teacher, V, ld_s, ld_t,
                                                      segments, part);
  kl_finish_kernel<<<(unsigned)((rows + 127) / 128), 128, 0, stream>>>(part, rows, segments, out);
  return cudaGetLastError();
}
