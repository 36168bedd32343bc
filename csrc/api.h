// C entry points of the sm_100a kernels (one per op family). Every function
// launches on the given stream and returns the launch status; none of them
// allocates device memory.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

int rt_wkv7_chunk_len();
long rt_wkv7_scan_workspace_floats(int B, int T, int H, int N);
cudaError_t rt_wkv7_scan_forward(int dtype, int B, int T, int H, int N, const void* r, const void* w, const void* k,
                                 const void* v, const void* a, const void* b, const float* s0, void* y, float* s_end,
                                 float* checkpoints, float* work, cudaStream_t stream);
cudaError_t rt_wkv7_forward(int dtype, int B, int T, int H, int N, const void* r, const void* w, const void* k,
                            const void* v, const void* a, const void* b, const float* s0, void* y, float* s_end,
                            float* checkpoints, cudaStream_t stream);
// tcgen05 path (bf16, head size 64, chunks of 64 steps): wkv7_tc_fwd.cu / wkv7_tc_bwd.cu.
int rt_wkv7_tc_chunk_len();
long rt_wkv7_tc_workspace_floats(int B, int T, int H);
long rt_wkv7_tc_backward_workspace_floats(int B, int T, int H);
int rt_wkv7_tc_fault();
int rt_wkv7_tc_bwd_fault();
cudaError_t rt_wkv7_tc_fault_async(int* dst, cudaStream_t stream);
cudaError_t rt_wkv7_tc_bwd_fault_async(int* dst, cudaStream_t stream);
cudaError_t rt_wkv7_tc_forward(int B, int T, int H, const void* r, const void* w, const void* k, const void* v,
                               const void* a, const void* b, const float* s0, void* y, float* s_end, float* ckpt,
                               float* ws, cudaStream_t stream);
cudaError_t rt_wkv7_tc_backward(int B, int T, int H, const void* r, const void* w, const void* k, const void* v,
                                const void* a, const void* b, const float* ckpt, const float* rec, const void* dy,
                                const float* dend, float* dr, float* dw, float* dk, float* dv, float* da, float* db,
                                float* ds0, float* work, cudaStream_t stream);
long rt_wkv7_backward_workspace_floats(int B, int T, int H, int N);
cudaError_t rt_wkv7_backward(int dtype, int B, int T, int H, int N, const void* r, const void* w, const void* k,
                             const void* v, const void* a, const void* b, const float* checkpoints, const void* dy,
                             const float* dend, float* dr, float* dw, float* dk, float* dv, float* da, float* db,
                             float* ds0, float* work, cudaStream_t stream);

// GEMM: C = epi(A . B^T). a_mn / b_mn select MN-major operands (see gemm.cu).
// epi: 0 bf16 store, 1 fp32 store, 2 fp32 accumulate (C += alpha * A.B^T).
cudaError_t rt_gemm_bf16(const void* A, long lda, int a_mn, const void* B, long ldb, int b_mn, void* C, long ldc,
                         int M, int N, int K, int epi, float alpha, int* status, cudaStream_t stream);
// G (1..3) GEMMs of one shape, layout and epilogue in one launch: C[g] = epi(A[g] . B[g]^T); choice < 0 picks the
// measured tile schedule of the shape, else a fixed one (width | 1 << 16 for stream-K).
cudaError_t rt_gemm_bf16_group(int G, const void* const* A, long lda, int a_mn, const void* const* B, long ldb,
                               int b_mn, void* const* C, long ldc, int M, int N, int K, int epi, float alpha,
                               int choice, int* status, cudaStream_t stream);
cudaError_t rt_gemm_set_lane(int lane);
void rt_gemm_set_concurrent(int on);
int rt_gemm_fault();
cudaError_t rt_gemm_fault_async(int* dst, cudaStream_t stream);
int rt_kl_segments(long rows, long V);
long rt_kl_workspace_floats(long rows, int segments);
cudaError_t rt_kl_rows(int dtype, const void* student, const void* teacher, long rows, long V, long ld_s, long ld_t,
                       int segments, float* work, float* out, cudaStream_t stream);
cudaError_t rt_gemm_nmse_bf16(const void* A, long lda, const void* B, long ldb, void* dpred, long ldc, const void* target,
                              float* rowsum, int M, int N, int K, float eps, int* status, cudaStream_t stream);
cudaError_t rt_loss_rows_prep(const void* target, float* rowsum, long rows, int C, cudaStream_t stream);
cudaError_t rt_loss_rows_finish(const float* rowsum, float* stats, long rows, int C, float eps, cudaStream_t stream);
cudaError_t rt_gemm_bf16_tile(const void* A, long lda, int a_mn, const void* B, long ldb, int b_mn, void* C, long ldc,
                              int M, int N, int K, int epi, float alpha, int choice, int* status, cudaStream_t stream);
cudaError_t rt_gemm_skinny_bf16(const void* X, long ldx, const void* W, const void* Wu, long ldw, float* ws,
                                void* out, long ldo, int M, int N, int K, int* status, cudaStream_t stream);
cudaError_t rt_gemm_swiglu_bf16(const void* A, long lda, const void* Bg, const void* Bu, long ldb, void* C, long ldc,
                                int M, int N, int K, int choice, int* status, cudaStream_t stream);

// Teacher-block kernels (bf16 activations, fp32 parameters).
cudaError_t rt_rmsnorm_1p(const void* x, const void* h, const float* w, void* sum_out, void* out, long rows, int C,
                          float eps, cudaStream_t stream);
cudaError_t rt_conv1d_silu(const void* x, long xs, const void* state, const float* weight, void* y, void* new_state,
                           int B, int T, int C, int K, cudaStream_t stream);
cudaError_t rt_gated_rmsnorm(const void* x, const void* z, const float* w, void* out, long rows, int D, int heads,
                             long zs, float eps, cudaStream_t stream);
cudaError_t rt_norm_rope(const void* src, long src_stride, long head_stride, const float* w, const float* inv_freq,
                         void* dst, int B, int T, int heads, long dst_batch_stride, int pos0, int D, int rot, float eps,
                         cudaStream_t stream);
cudaError_t rt_embed_rows(const long* ids, const void* table, long vocab, void* out, int width, long rows,
                          cudaStream_t stream);
cudaError_t rt_copy_rows(const void* src, long src_stride, void* dst, int B, int T, long dst_batch_stride, int width,
                         cudaStream_t stream);
long rt_gdn_workspace_floats(int B, int T, int Hk, int Hv, int D, long row_stride);
long rt_gdn_serial_workspace_floats(int B, int T, int Hk, int D);
cudaError_t rt_gdn_forward_serial(const void* qkv, long row_stride, const void* a, const void* b, long ab_stride,
                                  const float* A_log, const float* dt_bias, float* state, void* out, float* work,
                                  int B, int T, int Hk, int Hv, int D, cudaStream_t stream);
cudaError_t rt_gdn_forward(const void* qkv, long row_stride, const void* a, const void* b, long ab_stride,
                           const float* A_log, const float* dt_bias, float* state, void* out, float* work, int B,
                           int T, int Hk, int Hv, int D, cudaStream_t stream);

// TimeMix student stages and the flat optimizer (student_ops.cu).
cudaError_t rt_tm_mix(const void* x, const void* shift, const float* coef, void* out, int B, int T, int C,
                      cudaStream_t s);
long rt_tm_mix_bwd_scratch(int B, int T, int C);
cudaError_t rt_tm_mix_bwd(const void* x, const void* shift, const void* dmix, float* dcoef, int B, int T, int C,
                          float* scratch, cudaStream_t s);
cudaError_t rt_tm_pre_wkv(const void* k, const void* lw, const void* la, const float* w0, const float* a0,
                          const float* k_k, const float* k_a, void* w_in, void* k_in, void* a_in, void* b_in,
                          long rows, int H, int N, cudaStream_t s);
cudaError_t rt_tm_post_wkv(const void* y, const void* r, const void* kp, const void* v, const void* g,
                           const float* ln_w, const float* ln_b, const float* r_k, void* out, float* stats, long rows,
                           int H, int N, cudaStream_t s);
cudaError_t rt_tm_post_wkv_bwd(const void* dout, const void* y, const void* r, const void* kp, const void* v,
                               const void* g, const float* ln_w, const float* ln_b, const float* r_k,
                               const float* stats, void* dy, void* dg, float* dr, float* dk, float* dv, float* dln_w,
                               float* dln_b, float* dr_k, long rows, int H, int N, cudaStream_t s);
cudaError_t rt_tm_pre_wkv_bwd(const float* g_r, const float* g_w, const float* g_kp, const float* g_v,
                              const float* g_a, const float* g_b, const float* b_r, const float* b_kp,
                              const float* b_v, const void* k, const void* la, const float* w0, const float* a0,
                              const float* k_k, const float* k_a, void* dr, void* dk, void* dv, void* dlw, void* dla,
                              float* dw0, float* da0, float* dk_k, float* dk_a, long rows, int H, int N,
                              cudaStream_t s);
cudaError_t rt_act(void* x, long n, int mode, cudaStream_t s);
cudaError_t rt_act_bwd(const void* h, void* dh, long n, int mode, cudaStream_t s);
cudaError_t rt_nmse_loss(const void* pred, const void* target, float* stats, void* dpred, long rows, int C, float eps,
                         cudaStream_t s);
int rt_flat_adamw_scratch();
cudaError_t rt_flat_adamw(float* p, float* g, float* m, float* v, void* shadow, long n, long decay_numel,
                          float* stats, float* scratch, float* report, float lr, float beta1, float beta2,
                          float eps, float weight_decay, float clip, int step, cudaStream_t s);
cudaError_t rt_zero_f32(float* p, long n, cudaStream_t s);
cudaError_t rt_copy_bytes(void* dst, const void* src, long nbytes, cudaStream_t s);
cudaError_t rt_to_bf16(const float* src, void* dst, long n, cudaStream_t s);

// Flash attention forward (head_dim 256, GQA, causal with cache offset, fused sigmoid gate).
cudaError_t rt_flash_attention_fwd(const void* q, const void* keys, const void* values, const void* gate,
                                   long gate_row, long gate_head, void* out, int B, int T, int Hq, int Hkv, int offset,
                                   int cap, int* status, cudaStream_t stream);

// ---- peer-memory gradient exchange (csrc/parallel/peer_exchange.cu)
int rt_exchange_signal_words();
cudaError_t rt_exchange_update(float* const* grads, float* const* params, void* const* shadows, unsigned* const* sigs,
                               int rank, int world, long n, float* m, float* v, float* stats, float* report, float lr,
                               float beta1, float beta2, float eps, float weight_decay, float clip, int step,
                               long decay_numel, unsigned epoch, double limit_s, int blocks, int mode,
                               cudaStream_t s);
void rt_exchange_shard(long n, int rank, int world, long* out4);
cudaError_t rt_ipc_export(const void* ptr, void* handle64, long* offset);
cudaError_t rt_ipc_open(const void* handle64, void** base);
cudaError_t rt_ipc_close(void* base);

#ifdef __cplusplus
}
#endif

