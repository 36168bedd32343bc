// KL(teacher || student) over the vocabulary, one block per token row, one pass over both logit rows.
//
// Each thread keeps an online triple over its slice of the row:
//   m_t = max t,  Z_t = sum exp(t - m_t),  A = sum exp(t - m_t) (t - s),  and m_s, Z_s for the student,
// and the block merges the triples (rescaling by exp(m_old - m_new)). Then
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

template <typename T>
__global__ void __launch_bounds__(512) kl_rows_kernel(const T* __restrict__ student, const T* __restrict__ teacher,
                                                      long V, long ld_s, long ld_t, float* __restrict__ out) {
  __shared__ Online part[16];
  const long row = blockIdx.x;
  const T* s = student + row * ld_s;
  const T* t = teacher + row * ld_t;
  Online o{-INFINITY, 0.f, 0.f, -INFINITY, 0.f};
  for (long v = threadIdx.x; v < V; v += blockDim.x) push(o, rt::to_f<T>(__ldg(t + v)), rt::to_f<T>(__ldg(s + v)));
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
  if (threadIdx.x == 0) {
    Online r = part[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) r = merge(r, part[w]);
    out[row] = r.a / r.zt - (r.mt + logf(r.zt)) + (r.ms + logf(r.zs));
  }
}

}  // namespace

// out[r] = KL(softmax(teacher[r]) || softmax(student[r])) for rows r < rows; dtype 1 = bf16, 0 = fp32.
extern "C" cudaError_t rt_kl_rows(int dtype, const void* student, const void* teacher, long rows, long V, long ld_s,
                                  long ld_t, float* out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if (V <= 0) return cudaErrorInvalidValue;
  if (dtype == 1)
    kl_rows_kernel<__nv_bfloat16><<<rows, 512, 0, stream>>>((const __nv_bfloat16*)student,
                                                            (const __nv_bfloat16*)teacher, V, ld_s, ld_t, out);
  else
    kl_rows_kernel<float><<<rows, 512, 0, stream>>>((const float*)student, (const float*)teacher, V, ld_s, ld_t, out);
  return cudaGetLastError();
}
