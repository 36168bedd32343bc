// C entry points of the sm_100a kernels (one per op family). Every function
// launches on the given stream and returns the launch status; none of them
// allocates device memory.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

int rt_wkv7_chunk_len();
cudaError_t rt_wkv7_forward(int dtype, int B, int T, int H, int N, const void* r, const void* w, const void* k,
                            const void* v, const void* a, const void* b, const float* s0, void* y, float* s_end,
                            float* checkpoints, cudaStream_t stream);
cudaError_t rt_wkv7_backward(int dtype, int B, int T, int H, int N, const void* r, const void* w, const void* k,
                             const void* v, const void* a, const void* b, const float* checkpoints, const void* dy,
                             const float* dend, float* dr, float* dw, float* dk, float* dv, float* da, float* db,
                             float* ds0, cudaStream_t stream);

// GEMM: C = epi(A . B^T). a_mn / b_mn select MN-major operands (see gemm.cu).
// epi: 0 bf16 store, 1 fp32 store, 2 fp32 accumulate (C += alpha * A.B^T).
cudaError_t rt_gemm_bf16(const void* A, long lda, int a_mn, const void* B, long ldb, int b_mn, void* C, long ldc,
                         int M, int N, int K, int epi, float alpha, int* status, cudaStream_t stream);
cudaError_t rt_gemm_swiglu_bf16(const void* A, long lda, const void* Bg, const void* Bu, long ldb, void* C, long ldc,
                                int M, int N, int K, int* status, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
