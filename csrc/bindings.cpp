// PyTorch bindings of the sm_100a kernels. Kernels live in .cu files behind
// plain C entry points (pointers + sizes + stream); this file does the shape,
// dtype and device checks, allocates outputs, and launches on the current
// stream of the tensors' device.
#include <torch/extension.h>

#include <map>
#include <string>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <vector>

#include "api.h"

namespace {

void check_cuda(cudaError_t err, const char* what) {
  TORCH_CHECK(err == cudaSuccess, what, " failed: ", cudaGetErrorString(err));
}

int dtype_code(const at::Tensor& t) {
  if (t.scalar_type() == at::kBFloat16) return 1;
  TORCH_CHECK(t.scalar_type() == at::kFloat, "expected bf16 or fp32 tensor");
  return 0;
}

cudaStream_t stream_of(const at::Tensor& t) { return at::cuda::getCurrentCUDAStream(t.device().index()); }

void check_wkv(const at::Tensor& r, const std::vector<at::Tensor>& xs) {
  TORCH_CHECK(r.is_cuda() && r.is_contiguous() && r.dim() == 4, "expected contiguous CUDA [B,T,H,N]");
  TORCH_CHECK(r.size(1) > 0 && r.size(3) >= 2 && r.size(3) <= 128, "invalid T or head size (2..128)");
  dtype_code(r);
  for (auto& x : xs)
    TORCH_CHECK(x.device() == r.device() && x.sizes() == r.sizes() && x.scalar_type() == r.scalar_type() &&
                    x.is_contiguous(),
                "WKV7 input mismatch");
}

// The tcgen05 path (chunks of 64 steps) serves bf16 inputs with head size 64 and at least 128 steps; shorter
// calls, fp32 inputs and other head sizes run the chunk-16 CUDA-core kernels.
bool g_wkv7_tc_enabled = true;
bool wkv7_use_tc(const at::Tensor& r) {
  return g_wkv7_tc_enabled && r.scalar_type() == at::kBFloat16 && r.size(3) == 64 && r.size(1) >= 128;
}

// Returns (y, end, checkpoints, records). `checkpoints` [B, H, chunks + 1, N, N] holds the chunk-start states
// and the final state; `records` is the tcgen05 path's per-chunk record (G, H0, Q, Y0, T; the backward reads
// it) and is empty on the CUDA-core path.
std::vector<at::Tensor> wkv7_forward(at::Tensor r, at::Tensor w, at::Tensor k, at::Tensor v, at::Tensor a,
                                     at::Tensor b, at::Tensor s0, bool save_checkpoints) {
  check_wkv(r, {w, k, v, a, b});
  c10::cuda::CUDAGuard guard(r.device());
  const int B = r.size(0), T = r.size(1), H = r.size(2), N = r.size(3);
  TORCH_CHECK(s0.device() == r.device() && s0.scalar_type() == at::kFloat && s0.is_contiguous() &&
                  s0.sizes() == at::IntArrayRef({B, H, N, N}),
              "s0 must be contiguous CUDA fp32 [B,H,N,N]");
  auto y = at::empty_like(r);
  auto end = at::empty_like(s0);
  auto none = at::empty({0}, s0.options());
  if (wkv7_use_tc(r)) {
    const int chunks = (T + rt_wkv7_tc_chunk_len() - 1) / rt_wkv7_tc_chunk_len();
    auto ckpt = at::empty({B, H, chunks + 1, N, N}, s0.options());
    auto rec = at::empty({rt_wkv7_tc_workspace_floats(B, T, H)}, s0.options());
    check_cuda(rt_wkv7_tc_forward(B, T, H, r.data_ptr(), w.data_ptr(), k.data_ptr(), v.data_ptr(), a.data_ptr(),
                                  b.data_ptr(), s0.data_ptr<float>(), y.data_ptr(), end.data_ptr<float>(),
                                  ckpt.data_ptr<float>(), rec.data_ptr<float>(), stream_of(r)),
               "wkv7_forward (tcgen05)");
    if (!save_checkpoints) return {y, end, none, none};
    return {y, end, ckpt, rec};
  }
  const int chunks = (T + rt_wkv7_chunk_len() - 1) / rt_wkv7_chunk_len();
  auto ckpt = save_checkpoints ? at::empty({B, H, chunks + 1, N, N}, s0.options()) : none;
  const long scan_ws = T > 4 ? rt_wkv7_scan_workspace_floats(B, T, H, N) : 0;
  if (scan_ws > 0) {  // head sizes 32/64/128: parallel per-chunk pass + light serial scan
    auto work = at::empty({scan_ws}, s0.options());
    check_cuda(rt_wkv7_scan_forward(dtype_code(r), B, T, H, N, r.data_ptr(), w.data_ptr(), k.data_ptr(),
                                    v.data_ptr(), a.data_ptr(), b.data_ptr(), s0.data_ptr<float>(), y.data_ptr(),
                                    end.data_ptr<float>(), save_checkpoints ? ckpt.data_ptr<float>() : nullptr,
                                    work.data_ptr<float>(), stream_of(r)),
               "wkv7_forward (scan)");
    return {y, end, ckpt, none};
  }
  check_cuda(rt_wkv7_forward(dtype_code(r), B, T, H, N, r.data_ptr(), w.data_ptr(), k.data_ptr(), v.data_ptr(),
                             a.data_ptr(), b.data_ptr(), s0.data_ptr<float>(), y.data_ptr(), end.data_ptr<float>(),
                             save_checkpoints ? ckpt.data_ptr<float>() : nullptr, stream_of(r)),
             "wkv7_forward");
  return {y, end, ckpt, none};
}

std::vector<at::Tensor> wkv7_backward(at::Tensor r, at::Tensor w, at::Tensor k, at::Tensor v, at::Tensor a,
                                      at::Tensor b, at::Tensor ckpt, at::Tensor rec, at::Tensor dy, at::Tensor dend) {
  check_wkv(r, {w, k, v, a, b, dy});
  c10::cuda::CUDAGuard guard(r.device());
  const int B = r.size(0), T = r.size(1), H = r.size(2), N = r.size(3);
  const bool tc = rec.numel() > 0;
  TORCH_CHECK(!tc || (r.scalar_type() == at::kBFloat16 && N == 64),
              "tcgen05 WKV7 records given for a call the tcgen05 path does not serve");
  const int len = tc ? rt_wkv7_tc_chunk_len() : rt_wkv7_chunk_len();
  const int chunks = (T + len - 1) / len;
  TORCH_CHECK(ckpt.device() == r.device() && ckpt.scalar_type() == at::kFloat && ckpt.is_contiguous() &&
                  ckpt.sizes() == at::IntArrayRef({B, H, chunks + 1, N, N}),
              "invalid chunk checkpoints");
  // An undefined dend stands for a zero end-state gradient (the kernels then read none).
  TORCH_CHECK(!dend.defined() || (dend.device() == r.device() && dend.scalar_type() == at::kFloat &&
                                  dend.is_contiguous() && dend.sizes() == at::IntArrayRef({B, H, N, N})),
              "invalid dend");
  const float* dend_ptr = dend.defined() ? dend.data_ptr<float>() : nullptr;
  auto opts = r.options().dtype(at::kFloat);
  std::vector<at::Tensor> g;
  for (int i = 0; i < 6; ++i) g.push_back(at::empty(r.sizes(), opts));
  g.push_back(at::empty({B, H, N, N}, opts));
  if (tc) {
    TORCH_CHECK(rec.device() == r.device() && rec.scalar_type() == at::kFloat && rec.is_contiguous() &&
                    rec.numel() == rt_wkv7_tc_workspace_floats(B, T, H),
                "invalid tcgen05 WKV7 records");
    auto work = at::empty({rt_wkv7_tc_backward_workspace_floats(B, T, H)}, opts);
    check_cuda(rt_wkv7_tc_backward(B, T, H, r.data_ptr(), w.data_ptr(), k.data_ptr(), v.data_ptr(), a.data_ptr(),
                                   b.data_ptr(), ckpt.data_ptr<float>(), rec.data_ptr<float>(), dy.data_ptr(),
                                   dend_ptr, g[0].data_ptr<float>(), g[1].data_ptr<float>(),
                                   g[2].data_ptr<float>(), g[3].data_ptr<float>(), g[4].data_ptr<float>(),
                                   g[5].data_ptr<float>(), g[6].data_ptr<float>(), work.data_ptr<float>(),
                                   stream_of(r)),
               "wkv7_backward (tcgen05)");
    return g;
  }
  auto work = at::empty({rt_wkv7_backward_workspace_floats(B, T, H, N)}, opts);
  check_cuda(rt_wkv7_backward(dtype_code(r), B, T, H, N, r.data_ptr(), w.data_ptr(), k.data_ptr(), v.data_ptr(),
                              a.data_ptr(), b.data_ptr(), ckpt.data_ptr<float>(), dy.data_ptr(),
                              dend_ptr, g[0].data_ptr<float>(), g[1].data_ptr<float>(),
                              g[2].data_ptr<float>(), g[3].data_ptr<float>(), g[4].data_ptr<float>(),
                              g[5].data_ptr<float>(), g[6].data_ptr<float>(), work.data_ptr<float>(), stream_of(r)),
             "wkv7_backward");
  return g;
}

// Operand view for the GEMM: a 2-D bf16 tensor with unit inner stride. Returns (ptr, ld).
struct Operand {
  const void* ptr;
  long ld;
};

Operand operand(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.scalar_type() == at::kBFloat16, name, " must be a 2-D CUDA bf16 tensor");
  TORCH_CHECK(t.stride(1) == 1 && t.stride(0) >= t.size(1) && t.stride(0) % 8 == 0, name,
              " needs unit inner stride and a row stride that is a multiple of 8");
  return {t.data_ptr(), (long)t.stride(0)};
}

at::Tensor status_tensor(const at::Tensor& like) {
  return at::zeros({1}, like.options().dtype(at::kInt));
}

// out = a_op(A) . b_op(B)^T where a_op is identity ([M,K]) or transpose ([K,M] stored), same for B.
// epi 0: returns new bf16 [M,N]; epi 1: new fp32; epi 2: accumulates alpha * result into `out` (fp32).
at::Tensor gemm(at::Tensor A, bool a_t, at::Tensor B, bool b_t, int64_t epi, double alpha, c10::optional<at::Tensor> out,
                int64_t tile) {
  c10::cuda::CUDAGuard guard(A.device());
  auto a = operand(A, "A");
  auto b = operand(B, "B");
  const long M = a_t ? A.size(1) : A.size(0), K = a_t ? A.size(0) : A.size(1);
  const long N = b_t ? B.size(1) : B.size(0), KB = b_t ? B.size(0) : B.size(1);
  TORCH_CHECK(K == KB, "GEMM inner dimensions differ: ", K, " vs ", KB);
  if (epi == 0 && M <= 32 && !a_t && !b_t && !out.has_value() && tile == 0) {  // decode-sized: split-K weight streaming
    auto C = at::empty({M, N}, A.options().dtype(at::kBFloat16));
    auto ws = at::empty({M, N}, A.options().dtype(at::kFloat));
    check_cuda(rt_gemm_skinny_bf16(a.ptr, a.ld, b.ptr, nullptr, b.ld, ws.data_ptr<float>(), C.data_ptr(), N, M, N,
                                   K, nullptr, stream_of(A)),
               "gemm (skinny)");
    return C;
  }
  at::Tensor C;
  if (epi == 2) {
    TORCH_CHECK(out.has_value(), "accumulate epilogue needs `out`");
    C = *out;
    TORCH_CHECK(C.scalar_type() == at::kFloat && C.is_contiguous() && C.size(0) == M && C.size(1) == N,
                "accumulator must be contiguous fp32 [M, N]");
  } else if (out.has_value()) {
    C = *out;
    TORCH_CHECK(C.is_contiguous() && C.size(0) == M && C.size(1) == N &&
                    C.scalar_type() == (epi == 0 ? at::kBFloat16 : at::kFloat),
                "invalid output tensor");
  } else {
    C = at::empty({M, N}, A.options().dtype(epi == 0 ? at::kBFloat16 : at::kFloat));
  }
  if (tile) {
    check_cuda(rt_gemm_bf16_tile(a.ptr, a.ld, a_t, b.ptr, b.ld, b_t, C.data_ptr(), C.stride(0), M, N, K, (int)epi,
                                 (float)alpha, (int)tile, nullptr, stream_of(A)),
               "gemm (fixed tile)");
    return C;
  }
  check_cuda(rt_gemm_bf16(a.ptr, a.ld, a_t, b.ptr, b.ld, b_t, C.data_ptr(), C.stride(0), M, N, K, (int)epi,
                          (float)alpha, nullptr, stream_of(A)),
             "gemm");
  return C;
}

// outs[g] = a_op(A[g]) . b_op(B[g])^T for up to 3 problems of one shape, layout and epilogue, in one launch (see
// `gemm`). `outs` empty: new outputs (epi 0 bf16, epi 1 fp32); epi 2 accumulates into the given fp32 `outs`.
std::vector<at::Tensor> gemm_group(std::vector<at::Tensor> As, bool a_t, std::vector<at::Tensor> Bs, bool b_t,
                                   int64_t epi, double alpha, std::vector<at::Tensor> outs, int64_t tile) {
  const size_t G = As.size();
  TORCH_CHECK(G >= 1 && G <= 3 && Bs.size() == G && (outs.empty() || outs.size() == G),
              "gemm_group: 1 to 3 problems, one B (and out) per A");
  c10::cuda::CUDAGuard guard(As[0].device());
  const void* ap[3];
  const void* bp[3];
  void* cp[3];
  const Operand a0 = operand(As[0], "A"), b0 = operand(Bs[0], "B");
  const long M = a_t ? As[0].size(1) : As[0].size(0), K = a_t ? As[0].size(0) : As[0].size(1);
  const long N = b_t ? Bs[0].size(1) : Bs[0].size(0), KB = b_t ? Bs[0].size(0) : Bs[0].size(1);
  TORCH_CHECK(K == KB, "GEMM inner dimensions differ: ", K, " vs ", KB);
  TORCH_CHECK(epi != 2 || !outs.empty(), "accumulate epilogue needs `outs`");
  const auto ctype = epi == 0 ? at::kBFloat16 : at::kFloat;
  for (size_t g = 0; g < G; ++g) {
    const Operand a = operand(As[g], "A"), b = operand(Bs[g], "B");
    TORCH_CHECK(As[g].sizes() == As[0].sizes() && Bs[g].sizes() == Bs[0].sizes() && a.ld == a0.ld && b.ld == b0.ld,
                "gemm_group: every problem needs the same shapes and strides");
    if (outs.size() < G) outs.push_back(at::empty({M, N}, As[0].options().dtype(ctype)));
    const at::Tensor& C = outs[g];
    TORCH_CHECK(C.is_cuda() && C.scalar_type() == ctype && C.dim() == 2 && C.size(0) == M && C.size(1) == N &&
                    C.stride(1) == 1 && C.stride(0) == outs[0].stride(0),
                "gemm_group: outputs must be [M, N] with unit inner stride and one row stride, ",
                epi == 0 ? "bf16" : "fp32");
    ap[g] = a.ptr;
    bp[g] = b.ptr;
    cp[g] = C.data_ptr();
  }
  check_cuda(rt_gemm_bf16_group((int)G, ap, a0.ld, a_t, bp, b0.ld, b_t, cp, outs[0].stride(0), M, N, K, (int)epi,
                                (float)alpha, tile ? (int)tile : -1, nullptr, stream_of(As[0])),
             "gemm_group");
  return outs;
}

at::Tensor gemm_swiglu(at::Tensor A, at::Tensor Bg, at::Tensor Bu, int64_t tile) {
  c10::cuda::CUDAGuard guard(A.device());
  auto a = operand(A, "A");
  auto g = operand(Bg, "Bg");
  auto u = operand(Bu, "Bu");
  TORCH_CHECK(g.ld == u.ld && Bg.sizes() == Bu.sizes(), "gate and up weights must share shape and stride");
  const long M = A.size(0), K = A.size(1), N = Bg.size(0);
  TORCH_CHECK(Bg.size(1) == K, "SwiGLU inner dimension mismatch");
  auto C = at::empty({M, N}, A.options());
  if (M <= 32) {  // decode-sized: split-K weight streaming of both operands, fused silu * up
    auto ws = at::empty({2 * M, N}, A.options().dtype(at::kFloat));
    check_cuda(rt_gemm_skinny_bf16(a.ptr, a.ld, g.ptr, u.ptr, g.ld, ws.data_ptr<float>(), C.data_ptr(), N, M, N, K,
                                   nullptr, stream_of(A)),
               "gemm_swiglu (skinny)");
    return C;
  }
  check_cuda(rt_gemm_swiglu_bf16(a.ptr, a.ld, g.ptr, u.ptr, g.ld, C.data_ptr(), N, M, N, K, tile ? (int)tile : -1,
                                 nullptr, stream_of(A)),
             "gemm_swiglu");
  return C;
}

void check_bf16(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), name,
              " must be a contiguous CUDA bf16 tensor");
}

at::Tensor f32(const at::Tensor& w) { return w.to(at::kFloat).contiguous(); }

at::Tensor rmsnorm_1p(at::Tensor x, at::Tensor w, double eps) {
  check_bf16(x, "x");
  c10::cuda::CUDAGuard guard(x.device());
  const long C = x.size(-1), rows = x.numel() / C;
  auto wf = f32(w);
  auto out = at::empty_like(x);
  check_cuda(rt_rmsnorm_1p(x.data_ptr(), nullptr, wf.data_ptr<float>(), nullptr, out.data_ptr(), rows, C, eps,
                           stream_of(x)),
             "rmsnorm_1p");
  return out;
}

std::vector<at::Tensor> add_rmsnorm_1p(at::Tensor x, at::Tensor h, at::Tensor w, double eps) {
  check_bf16(x, "x");
  check_bf16(h, "h");
  TORCH_CHECK(x.sizes() == h.sizes(), "residual shapes differ");
  c10::cuda::CUDAGuard guard(x.device());
  const long C = x.size(-1), rows = x.numel() / C;
  auto wf = f32(w);
  auto sum = at::empty_like(x), out = at::empty_like(x);
  check_cuda(rt_rmsnorm_1p(x.data_ptr(), h.data_ptr(), wf.data_ptr<float>(), sum.data_ptr(), out.data_ptr(), rows, C,
                           eps, stream_of(x)),
             "add_rmsnorm_1p");
  return {sum, out};
}

// x: [B, T, C] bf16 with unit channel stride and any token stride (a column slice of a wider projection output).
std::vector<at::Tensor> conv1d_silu(at::Tensor x, at::Tensor state, at::Tensor weight) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 3 && x.stride(2) == 1,
              "x must be [B, T, C] bf16 rows (unit channel stride)");
  const long xs = x.size(1) > 1 ? x.stride(1) : x.stride(0);  // token row stride (a size-1 dim has any stride)
  TORCH_CHECK(x.size(0) == 1 || x.stride(0) == x.size(1) * xs, "x rows must be evenly spaced over batch and time");
  check_bf16(state, "state");
  c10::cuda::CUDAGuard guard(x.device());
  const int B = x.size(0), T = x.size(1), C = x.size(2), K = weight.size(-1);
  TORCH_CHECK(state.size(0) == B && state.size(1) == K - 1 && state.size(2) == C, "conv state must be [B, K-1, C]");
  auto wf = f32(weight.reshape({C, K}));
  auto y = at::empty({B, T, C}, x.options()), ns = at::empty_like(state);
  check_cuda(rt_conv1d_silu(x.data_ptr(), xs, state.data_ptr(), wf.data_ptr<float>(), y.data_ptr(),
                            ns.data_ptr(), B, T, C, K, stream_of(x)),
             "conv1d_silu");
  return {y, ns};
}

// x: contiguous [..., D] rows; z: the same rows as [tokens, heads * D] with unit inner stride and any token stride.
at::Tensor gated_rmsnorm(at::Tensor x, at::Tensor z, at::Tensor w, double eps) {
  check_bf16(x, "x");
  c10::cuda::CUDAGuard guard(x.device());
  const long D = w.numel(), rows = x.numel() / D;
  TORCH_CHECK(z.is_cuda() && z.scalar_type() == at::kBFloat16 && z.stride(-1) == 1, "z must be bf16 rows");
  const at::Tensor z2 = z.dim() == 2 ? z : z.contiguous().view({-1, z.size(-1)});
  TORCH_CHECK(z2.size(1) % D == 0 && z2.size(0) * (z2.size(1) / D) == rows, "z rows do not match x");
  const int heads = z2.size(1) / D;
  auto wf = f32(w);
  auto out = at::empty_like(x);
  check_cuda(rt_gated_rmsnorm(x.data_ptr(), z2.data_ptr(), wf.data_ptr<float>(), out.data_ptr(), rows, D, heads,
                              z2.stride(0), eps, stream_of(x)),
             "gated_rmsnorm");
  return out;
}

// src: [B*T, row] bf16 rows whose head h starts at h * (row_stride / heads); writes RMSNorm(1+w) + RoPE
// (angle position rope_pos0 + t) into dst[b, dst_pos0 + t, head, :] of dst [B, cap, heads, D].
void norm_rope_(at::Tensor src, int64_t heads, at::Tensor w, at::Tensor inv_freq, at::Tensor dst, int64_t rope_pos0,
                int64_t dst_pos0, int64_t rot, double eps) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.dim() == 2 && src.stride(-1) == 1,
              "src must be 2-D bf16 rows");
  check_bf16(dst, "dst");
  TORCH_CHECK(dst.dim() == 4 && dst.size(2) == heads, "dst must be [B, cap, heads, D]");
  c10::cuda::CUDAGuard guard(src.device());
  const int B = dst.size(0), D = dst.size(3);
  const int T = src.size(0) / B;
  TORCH_CHECK(dst_pos0 + T <= dst.size(1), "cache too small");
  auto wf = f32(w), fq = f32(inv_freq);
  TORCH_CHECK(src.size(1) % heads == 0, "src width must be heads x head stride");
  check_cuda(rt_norm_rope(src.data_ptr(), src.stride(0), src.size(1) / heads, wf.data_ptr<float>(), fq.data_ptr<float>(),
                          dst.data_ptr<at::BFloat16>() + dst_pos0 * heads * D, B, T, heads, dst.stride(0),
                          (int)rope_pos0, D, rot, eps, stream_of(src)),
             "norm_rope");
}

// ids [..] int64 -> [.., width] bf16 rows of `table` [vocab, width] (bf16, contiguous).
at::Tensor embed_rows(at::Tensor ids, at::Tensor table) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kLong && table.is_cuda() &&
                  table.scalar_type() == at::kBFloat16 && table.is_contiguous() && table.dim() == 2,
              "embed_rows needs int64 ids and a contiguous bf16 [vocab, width] table on the GPU");
  c10::cuda::CUDAGuard guard(ids.device());
  auto flat = ids.contiguous();
  auto sizes = ids.sizes().vec();
  sizes.push_back(table.size(1));
  auto out = at::empty(sizes, table.options());
  check_cuda(rt_embed_rows(reinterpret_cast<const long*>(flat.data_ptr<int64_t>()), table.data_ptr(),
                           table.size(0), out.data_ptr(), (int)table.size(1), flat.numel(), stream_of(table)),
             "embed_rows");
  return out;
}

void copy_rows_(at::Tensor src, at::Tensor dst, int64_t pos0) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.dim() == 2 && src.stride(-1) == 1,
              "src must be 2-D bf16 rows");
  check_bf16(dst, "dst");
  c10::cuda::CUDAGuard guard(src.device());
  const int B = dst.size(0);
  const int width = dst.size(2) * dst.size(3);
  const int T = src.size(0) / B;
  TORCH_CHECK(pos0 + T <= dst.size(1) && src.size(1) >= width, "cache too small or rows too narrow");
  const long src_stride = src.stride(0);
  check_cuda(rt_copy_rows(src.data_ptr(), src_stride, dst.data_ptr<at::BFloat16>() + pos0 * width, B, T, dst.stride(0),
                          width, stream_of(src)),
             "copy_rows");
}

// GDN forward on the conv output `qkv` [B, T, 2*Hk*D + Hv*D]; a, b: [B, T, Hv]; state [B, Hv, D, D] fp32
// (updated in place). Returns o [B, T, Hv, D] bf16.
at::Tensor gdn_forward(at::Tensor qkv, at::Tensor a, at::Tensor b, at::Tensor A_log, at::Tensor dt_bias,
                       at::Tensor state, int64_t Hk, int64_t Hv, int64_t D) {
  check_bf16(qkv, "qkv");
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == at::kBFloat16 && a.stride(-1) == 1, "a must be bf16");
  TORCH_CHECK(b.is_cuda() && b.scalar_type() == at::kBFloat16 && b.stride(-1) == 1 && a.stride(-2) == b.stride(-2),
              "b must be bf16 with the stride of a");
  TORCH_CHECK(state.is_cuda() && state.scalar_type() == at::kFloat && state.is_contiguous(), "state must be fp32");
  c10::cuda::CUDAGuard guard(qkv.device());
  const int B = qkv.size(0), T = qkv.size(1);
  TORCH_CHECK(qkv.size(2) == 2 * Hk * D + Hv * D, "qkv width mismatch");
  auto work = at::empty({rt_gdn_workspace_floats(B, T, Hk, Hv, D, qkv.size(2))}, state.options());
  auto out = at::empty({B, T, Hv, D}, qkv.options());
  auto al = f32(A_log), dt = f32(dt_bias);
  check_cuda(rt_gdn_forward(qkv.data_ptr(), qkv.size(2), a.data_ptr(), b.data_ptr(), a.stride(-2), al.data_ptr<float>(),
                            dt.data_ptr<float>(), state.data_ptr<float>(), out.data_ptr(), work.data_ptr<float>(), B, T,
                            Hk, Hv, D, stream_of(qkv)),
             "gdn_forward");
  return out;
}

// ------------------------------------------------------------------ TimeMix student stages
// Raw-pointer bindings: the Python layer (models/student_fused.py) owns shapes and buffers.
#define PTR(t) ((t).data_ptr())
#define FPTR(t) ((t).data_ptr<float>())
void need(bool ok, const char* msg) { TORCH_CHECK(ok, msg); }

void tm_mix(at::Tensor x, at::Tensor shift, at::Tensor coef, at::Tensor out) {
  need(x.is_contiguous() && shift.is_contiguous() && out.is_contiguous() && coef.is_contiguous(), "tm_mix layout");
  c10::cuda::CUDAGuard guard(x.device());
  check_cuda(rt_tm_mix(PTR(x), PTR(shift), FPTR(coef), PTR(out), x.size(0), x.size(1), x.size(2), stream_of(x)),
             "tm_mix");
}
void tm_mix_bwd(at::Tensor x, at::Tensor shift, at::Tensor dmix, at::Tensor dcoef) {
  c10::cuda::CUDAGuard guard(x.device());
  const long n = rt_tm_mix_bwd_scratch(x.size(0), x.size(1), x.size(2));
  auto scratch = n > 0 ? at::empty({n}, x.options().dtype(at::kFloat)) : at::Tensor();
  check_cuda(rt_tm_mix_bwd(PTR(x), PTR(shift), PTR(dmix), FPTR(dcoef), x.size(0), x.size(1), x.size(2),
                           n > 0 ? scratch.data_ptr<float>() : nullptr, stream_of(x)),
             "tm_mix_bwd");
}
void tm_pre_wkv(at::Tensor k, at::Tensor lw, at::Tensor la, at::Tensor w0, at::Tensor a0, at::Tensor k_k,
                at::Tensor k_a, at::Tensor w_in, at::Tensor k_in, at::Tensor a_in, at::Tensor b_in, int64_t H,
                int64_t N) {
  c10::cuda::CUDAGuard guard(k.device());
  check_cuda(rt_tm_pre_wkv(PTR(k), PTR(lw), PTR(la), FPTR(w0), FPTR(a0), FPTR(k_k), FPTR(k_a), PTR(w_in), PTR(k_in),
                           PTR(a_in), PTR(b_in), k.numel() / (H * N), H, N, stream_of(k)),
             "tm_pre_wkv");
}
void tm_post_wkv(at::Tensor y, at::Tensor r, at::Tensor kp, at::Tensor v, at::Tensor g, at::Tensor ln_w,
                 at::Tensor ln_b, at::Tensor r_k, at::Tensor out, at::Tensor stats, int64_t H, int64_t N) {
  c10::cuda::CUDAGuard guard(y.device());
  check_cuda(rt_tm_post_wkv(PTR(y), PTR(r), PTR(kp), PTR(v), PTR(g), FPTR(ln_w), FPTR(ln_b), FPTR(r_k), PTR(out),
                            FPTR(stats), y.numel() / (H * N), H, N, stream_of(y)),
             "tm_post_wkv");
}
void tm_post_wkv_bwd(at::Tensor dout, at::Tensor y, at::Tensor r, at::Tensor kp, at::Tensor v, at::Tensor g,
                     at::Tensor ln_w, at::Tensor ln_b, at::Tensor r_k, at::Tensor stats, at::Tensor dy, at::Tensor dg,
                     at::Tensor dr, at::Tensor dk, at::Tensor dv, at::Tensor dln_w, at::Tensor dln_b,
                     at::Tensor dr_k, int64_t H, int64_t N) {
  c10::cuda::CUDAGuard guard(y.device());
  check_cuda(rt_tm_post_wkv_bwd(PTR(dout), PTR(y), PTR(r), PTR(kp), PTR(v), PTR(g), FPTR(ln_w), FPTR(ln_b), FPTR(r_k),
                                FPTR(stats), PTR(dy), PTR(dg), FPTR(dr), FPTR(dk), FPTR(dv), FPTR(dln_w), FPTR(dln_b),
                                FPTR(dr_k), y.numel() / (H * N), H, N, stream_of(y)),
             "tm_post_wkv_bwd");
}
void tm_pre_wkv_bwd(std::vector<at::Tensor> gw, std::vector<at::Tensor> bonus, at::Tensor k, at::Tensor la,
                    at::Tensor w0, at::Tensor a0, at::Tensor k_k, at::Tensor k_a, std::vector<at::Tensor> outs,
                    std::vector<at::Tensor> pgrads, int64_t H, int64_t N) {
  need(gw.size() == 6 && bonus.size() == 3 && outs.size() == 5 && pgrads.size() == 4, "tm_pre_wkv_bwd arity");
  c10::cuda::CUDAGuard guard(k.device());
  check_cuda(rt_tm_pre_wkv_bwd(FPTR(gw[0]), FPTR(gw[1]), FPTR(gw[2]), FPTR(gw[3]), FPTR(gw[4]), FPTR(gw[5]),
                               FPTR(bonus[0]), FPTR(bonus[1]), FPTR(bonus[2]), PTR(k), PTR(la), FPTR(w0), FPTR(a0),
                               FPTR(k_k), FPTR(k_a), PTR(outs[0]), PTR(outs[1]), PTR(outs[2]), PTR(outs[3]),
                               PTR(outs[4]), FPTR(pgrads[0]), FPTR(pgrads[1]), FPTR(pgrads[2]), FPTR(pgrads[3]),
                               k.numel() / (H * N), H, N, stream_of(k)),
             "tm_pre_wkv_bwd");
}
void act_(at::Tensor x, int64_t mode) {
  c10::cuda::CUDAGuard guard(x.device());
  check_cuda(rt_act(PTR(x), x.numel(), mode, stream_of(x)), "act");
}
void act_bwd_(at::Tensor h, at::Tensor dh, int64_t mode) {
  c10::cuda::CUDAGuard guard(h.device());
  check_cuda(rt_act_bwd(PTR(h), PTR(dh), h.numel(), mode, stream_of(h)), "act_bwd");
}
// Per-row KL(softmax(teacher) || softmax(student)) of two [rows, V] logit matrices (bf16 or fp32, unit inner stride).
at::Tensor kl_rows(at::Tensor student, at::Tensor teacher) {
  c10::cuda::CUDAGuard guard(student.device());
  TORCH_CHECK(student.is_cuda() && teacher.is_cuda() && student.dim() == 2 && student.sizes() == teacher.sizes() &&
                  student.scalar_type() == teacher.scalar_type() && student.stride(1) == 1 && teacher.stride(1) == 1,
              "kl_rows: two CUDA [rows, V] logit matrices of one dtype with unit inner stride");
  TORCH_CHECK(student.scalar_type() == at::kBFloat16 || student.scalar_type() == at::kFloat, "kl_rows: bf16 or fp32");
  const long rows = student.size(0), V = student.size(1);
  auto out = at::empty({rows}, student.options().dtype(at::kFloat));
  const int segments = rt_kl_segments(rows, V);
  auto work = at::empty({std::max(1L, rt_kl_workspace_floats(rows, segments))}, out.options());
  check_cuda(rt_kl_rows(student.scalar_type() == at::kBFloat16 ? 1 : 0, student.data_ptr(), teacher.data_ptr(), rows, V,
                        student.stride(0), teacher.stride(0), segments, work.data_ptr<float>(), out.data_ptr<float>(),
                        stream_of(student)),
             "kl_rows");
  return out;
}

// Student output projection fused with the distillation loss: returns dpred [M, N] bf16; stats += [sum nmse,
// sum cos, rows] (x [M, K] bf16, w [N, K] bf16, target [M, N] bf16; p = x w^T is never stored).
at::Tensor gemm_nmse(at::Tensor x, at::Tensor w, at::Tensor target, at::Tensor stats, double eps) {
  c10::cuda::CUDAGuard guard(x.device());
  auto a = operand(x, "x");
  auto b = operand(w, "w");
  check_bf16(target, "target");
  const long M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && target.numel() == M * N, "gemm_nmse: shape mismatch");
  TORCH_CHECK(stats.is_cuda() && stats.scalar_type() == at::kFloat && stats.numel() >= 3 && stats.is_contiguous(),
              "stats must be fp32 [3]");
  auto dpred = at::empty({M, N}, x.options().dtype(at::kBFloat16));
  auto rowsum = at::empty({M, 4}, x.options().dtype(at::kFloat));
  auto s = stream_of(x);
  check_cuda(rt_loss_rows_prep(target.data_ptr(), rowsum.data_ptr<float>(), M, N, s), "loss_rows_prep");
  check_cuda(rt_gemm_nmse_bf16(a.ptr, a.ld, b.ptr, b.ld, dpred.data_ptr(), N, target.data_ptr(),
                               rowsum.data_ptr<float>(), M, N, K, (float)eps, nullptr, s),
             "gemm_nmse");
  check_cuda(rt_loss_rows_finish(rowsum.data_ptr<float>(), stats.data_ptr<float>(), M, N, (float)eps, s),
             "loss_rows_finish");
  return dpred;
}

void nmse_loss(at::Tensor pred, at::Tensor target, at::Tensor stats, c10::optional<at::Tensor> dpred, double eps) {
  need(pred.is_contiguous() && target.is_contiguous() && pred.sizes() == target.sizes(), "loss operands");
  c10::cuda::CUDAGuard guard(pred.device());
  const long C = pred.size(-1);
  check_cuda(rt_nmse_loss(PTR(pred), PTR(target), FPTR(stats), dpred ? PTR(*dpred) : nullptr, pred.numel() / C, C,
                          eps, stream_of(pred)),
             "nmse_loss");
}
void flat_adamw(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> shadow,
                int64_t decay_numel, at::Tensor stats, at::Tensor norm2, at::Tensor report, double lr, double beta1,
                double beta2, double eps, double wd, double clip, int64_t step) {
  need(p.numel() == g.numel() && p.numel() == m.numel() && p.numel() == v.numel(), "flat buffer sizes");
  need(norm2.scalar_type() == at::kFloat && norm2.numel() >= rt_flat_adamw_scratch(),
       "flat_adamw scratch needs flat_adamw_scratch() fp32 words");
  c10::cuda::CUDAGuard guard(p.device());
  check_cuda(rt_flat_adamw(FPTR(p), FPTR(g), FPTR(m), FPTR(v), shadow ? PTR(*shadow) : nullptr, p.numel(), decay_numel,
                           FPTR(stats), FPTR(norm2), FPTR(report), lr, beta1, beta2, eps, wd, clip, step,
                           stream_of(p)),
             "flat_adamw");
}
void to_bf16_(at::Tensor src, at::Tensor dst) {
  need(src.numel() == dst.numel(), "to_bf16 sizes");
  c10::cuda::CUDAGuard guard(src.device());
  check_cuda(rt_to_bf16(FPTR(src), PTR(dst), src.numel(), stream_of(src)), "to_bf16");
}

// ---- peer-memory gradient exchange. Pointer lists hold one device address per rank (int64), peers' addresses
// already mapped into this process by ipc_open.
void exchange_update(std::vector<int64_t> grads, std::vector<int64_t> params, std::vector<int64_t> shadows,
                     std::vector<int64_t> sigs, int64_t rank, int64_t world, int64_t n, at::Tensor m, at::Tensor v,
                     at::Tensor stats, at::Tensor report, double lr, double beta1, double beta2, double eps, double wd,
                     double clip, int64_t step, int64_t decay_numel, int64_t epoch, double limit_s, int64_t blocks,
                     int64_t mode) {
  need((int64_t)grads.size() == world && (int64_t)params.size() == world && (int64_t)shadows.size() == world &&
           (int64_t)sigs.size() == world, "one pointer per rank");
  need(m.numel() == n && v.numel() == n && m.is_cuda() && m.scalar_type() == at::kFloat, "moment buffers");
  std::vector<float*> g(world), p(world);
  std::vector<void*> sh(world);
  std::vector<unsigned*> sg(world);
  for (int q = 0; q < world; ++q) {
    g[q] = reinterpret_cast<float*>(grads[q]);
    p[q] = reinterpret_cast<float*>(params[q]);
    sh[q] = reinterpret_cast<void*>(shadows[q]);
    sg[q] = reinterpret_cast<unsigned*>(sigs[q]);
  }
  c10::cuda::CUDAGuard guard(m.device());
  check_cuda(rt_exchange_update(g.data(), p.data(), sh.data(), sg.data(), (int)rank, (int)world, n, FPTR(m), FPTR(v),
                                FPTR(stats), FPTR(report), lr, beta1, beta2, eps, wd, clip, (int)step, decay_numel,
                                (unsigned)epoch, limit_s, (int)blocks, (int)mode, stream_of(m)),
             "exchange_update");
}
py::tuple ipc_export(at::Tensor t) {
  need(t.is_cuda(), "ipc_export needs a CUDA tensor");
  c10::cuda::CUDAGuard guard(t.device());
  char handle[64];
  long offset = 0;
  check_cuda(rt_ipc_export(t.data_ptr(), handle, &offset), "ipc_export");
  return py::make_tuple(py::bytes(handle, 64), (int64_t)offset);
}
int64_t ipc_open(py::bytes handle, int64_t device) {
  std::string h = handle;
  need(h.size() == 64, "IPC handle size");
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* base = nullptr;
  check_cuda(rt_ipc_open(h.data(), &base), "ipc_open");
  return reinterpret_cast<int64_t>(base);
}
void ipc_close(int64_t base, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  check_cuda(rt_ipc_close(reinterpret_cast<void*>(base)), "ipc_close");
}
std::vector<int64_t> exchange_shard(int64_t n, int64_t rank, int64_t world) {
  long out[4];
  rt_exchange_shard(n, (int)rank, (int)world, out);
  return {out[0], out[1], out[2], out[3]};
}

// q [B,T,Hq,256]; keys/values [B,cap,Hkv,256]; gate rows: qg [B*T, Hq*512] with the gate in the second half of
// every head's 512 values. Returns [B,T,Hq,256] bf16.
at::Tensor flash_attention(at::Tensor q, at::Tensor keys, at::Tensor values, at::Tensor qg, int64_t offset) {
  check_bf16(q, "q");
  check_bf16(keys, "keys");
  check_bf16(values, "values");
  TORCH_CHECK(q.dim() == 4 && q.size(3) == 256 && keys.dim() == 4 && keys.size(3) == 256 && keys.sizes() == values.sizes(),
              "flash_attention expects head_dim 256");
  TORCH_CHECK(qg.is_cuda() && qg.scalar_type() == at::kBFloat16 && qg.stride(-1) == 1, "gate must be bf16 rows");
  c10::cuda::CUDAGuard guard(q.device());
  const int B = q.size(0), T = q.size(1), Hq = q.size(2), Hkv = keys.size(2), cap = keys.size(1);
  TORCH_CHECK(qg.dim() == 2 && qg.size(0) == (long)B * T && qg.size(1) >= (long)Hq * 512,
              "gate rows must be [B*T, >= Hq*512] (per head [q | gate])");
  auto out = at::empty_like(q);
  check_cuda(rt_flash_attention_fwd(q.data_ptr(), keys.data_ptr(), values.data_ptr(),
                                    static_cast<const at::BFloat16*>(qg.data_ptr()) + 256, (long)qg.stride(0), 512,
                                    out.data_ptr(), B, T, Hq, Hkv, (int)offset, cap, nullptr, stream_of(q)),
             "flash_attention");
  return out;
}

// Native executor of one fused TimeMix student micro-step (reference theseus/timemix.py:66-89 forward, with the
// hand-written backward): mix, the r/k/v and LoRA GEMMs, pre-WKV, WKV7, post-WKV, the output GEMM with the loss in
// its epilogue, and the backward of all of it, issued from C++ on the current stream (about 40 launches; the Python
// sequence of the same calls cost milliseconds of host time per micro-step). Weights are bf16 views, the small
// parameter vectors fp32 views, gradients views into the flat fp32 gradient buffer; all of them stay valid for the
// life of the student (the flat buffers are never reallocated).
class StudentStep {
 public:
  StudentStep(std::map<std::string, at::Tensor> w, std::map<std::string, at::Tensor> p,
              std::map<std::string, at::Tensor> g, c10::optional<at::Tensor> grad_tail, int64_t H, int64_t N)
      : W_(std::move(w)), P_(std::move(p)), G_(std::move(g)), tail_(grad_tail), H_(H), N_(N) {
    for (const char* n : {"receptance", "key", "value", "output", "w1", "w2", "a1", "a2", "g1", "g2"})
      need(W_.count(n) && W_.at(n).scalar_type() == at::kBFloat16, "StudentStep: missing bf16 weight");
    for (const char* n : {"coef", "w0", "a0", "k_k", "k_a", "r_k", "ln_w", "ln_b"})
      need(P_.count(n) && P_.at(n).scalar_type() == at::kFloat && P_.at(n).is_contiguous(),
           "StudentStep: missing fp32 parameter vector");
  }

  // Inference forward: (prediction [B, T, C] bf16, new shift [B, C], end state [B, H, N, N]).
  std::vector<at::Tensor> forward(at::Tensor x, c10::optional<at::Tensor> shift, c10::optional<at::Tensor> wkv0) {
    c10::cuda::CUDAGuard guard(x.device());
    Saved s = run_forward(x, shift, wkv0, false);
    auto pred = mm(s.yg, W_.at("output"), false);
    return {pred.view(x.sizes()), last_token(s.x), s.end};
  }

  // Training micro-step: stats (fp32 [3]) += [sum nmse, sum cos, tokens]; gradients stored (first) or accumulated
  // into the flat buffer. Returns (new shift, end state).
  std::vector<at::Tensor> forward_backward(at::Tensor x, at::Tensor target, c10::optional<at::Tensor> shift,
                                           c10::optional<at::Tensor> wkv0, double eps, bool first, at::Tensor stats) {
    need(!G_.empty(), "StudentStep: built without gradient buffers");
    c10::cuda::CUDAGuard guard(x.device());
    const int64_t B = x.size(0), T = x.size(1), C = x.size(2), M = B * T, H = H_, N = N_;
    if (first && tail_.has_value() && tail_->numel() > 0)
      check_cuda(rt_zero_f32(tail_->data_ptr<float>(), tail_->numel(), stream_of(x)), "zero gradient tail");
    Saved s = run_forward(x, shift, wkv0, true);
    auto dpred = gemm_nmse(s.yg, W_.at("output"), target.reshape({M, C}).to(at::kBFloat16).contiguous(), stats, eps);
    // output projection
    auto dyg = mm(dpred, W_.at("output"), true);
    grad(dpred, true, s.yg, true, "output", first);
    // post-WKV backward
    auto dy = at::empty_like(dpred), dg = at::empty_like(dpred);
    auto f32 = dpred.options().dtype(at::kFloat);
    std::vector<at::Tensor> bonus = {at::empty({M, C}, f32), at::empty({M, C}, f32), at::empty({M, C}, f32)};
    tm_post_wkv_bwd(dyg, s.y, s.r, s.k_in, s.v, s.g, P_.at("ln_w"), P_.at("ln_b"), P_.at("r_k"), s.gn, dy, dg,
                    bonus[0], bonus[1], bonus[2], G_.at("ln_w"), G_.at("ln_b"), G_.at("r_k"), H, N);
    const std::vector<int64_t> shape = {B, T, H, N};
    auto gw = wkv7_backward(s.r.view(shape), s.w_in.view(shape), s.k_in.view(shape), s.v.view(shape),
                            s.a_in.view(shape), s.b_in.view(shape), s.ckpt, s.rec, dy.view(shape), at::Tensor());
    std::vector<at::Tensor> d5;
    for (int i = 0; i < 5; ++i) d5.push_back(at::empty_like(dpred));  // dr, dk, dv, dlw, dla
    tm_pre_wkv_bwd({gw[0], gw[1], gw[2], gw[3], gw[4], gw[5]}, bonus, s.k, s.la, P_.at("w0"), P_.at("a0"),
                   P_.at("k_k"), P_.at("k_a"), d5, {G_.at("w0"), G_.at("a0"), G_.at("k_k"), G_.at("k_a")}, H, N);
    gw.clear();
    bonus.clear();
    auto dmix = at::empty_like(s.mix);
    auto xm = [&](int i) { return s.mix.select(0, i); };  // xr, xw, xk, xv, xa, xg
    // r, k, v projections: input gradients as one grouped launch, weight gradients as another
    if (grouped()) {
      const std::vector<at::Tensor> drkv = {d5[0], d5[1], d5[2]};
      gemm_group(drkv, false, {W_.at("receptance"), W_.at("key"), W_.at("value")}, true, 0, 1.0,
                 {dmix.select(0, 0), dmix.select(0, 2), dmix.select(0, 3)}, 0);
      gemm_group(drkv, true, {xm(0), xm(2), xm(3)}, true, first ? 1 : 2, 1.0,
                 {G_.at("receptance"), G_.at("key"), G_.at("value")}, 0);
    } else {
      const std::pair<int, const char*> proj[3] = {{0, "receptance"}, {2, "key"}, {3, "value"}};
      for (int i = 0; i < 3; ++i) {
        gemm(d5[i], false, W_.at(proj[i].second), true, 0, 1.0, dmix.select(0, proj[i].first), 0);
        grad(d5[i], true, xm(proj[i].first), true, proj[i].second, first);
      }
    }
    // decay LoRA: lw = tanh(xw w1) w2
    acc(s.hw, d5[3], "w2");
    auto dhw = mm(d5[3], W_.at("w2"), false);
    act_bwd_(s.hw, dhw, 0);
    acc(xm(1), dhw, "w1");
    gemm(dhw, false, W_.at("w1"), false, 0, 1.0, dmix.select(0, 1), 0);
    // in-context-rate LoRA: la = (xa a1) a2
    acc(s.ha, d5[4], "a2");
    auto dha = mm(d5[4], W_.at("a2"), false);
    acc(xm(4), dha, "a1");
    gemm(dha, false, W_.at("a1"), false, 0, 1.0, dmix.select(0, 4), 0);
    // gate LoRA: g = sigmoid(xg g1) g2
    acc(s.hg, dg, "g2");
    auto dhg = mm(dg, W_.at("g2"), false);
    act_bwd_(s.hg, dhg, 1);
    acc(xm(5), dhg, "g1");
    gemm(dhg, false, W_.at("g1"), false, 0, 1.0, dmix.select(0, 5), 0);
    tm_mix_bwd(s.x, s.shift, dmix, G_.at("coef"));
    return {last_token(s.x), s.end};
  }

 private:
  struct Saved {
    at::Tensor x, shift, mix, r, k, v, hw, ha, hg, lw, la, g, w_in, k_in, a_in, b_in, y, ckpt, rec, yg, gn, end;
  };

  // x[:, T - 1] as a new [B, C] tensor (the next chunk's token-shift state), copied by this package's kernel.
  static at::Tensor last_token(const at::Tensor& x) {
    const int64_t B = x.size(0), T = x.size(1), C = x.size(2);
    auto out = at::empty({B, C}, x.options());
    const long row = C * (long)x.element_size();
    for (int64_t b = 0; b < B; ++b)
      check_cuda(rt_copy_bytes(static_cast<uint8_t*>(out.data_ptr()) + b * row,
                               static_cast<const uint8_t*>(x.data_ptr()) + (b * T + T - 1) * row, row, stream_of(x)),
                 "last token");
    return out;
  }

  // The r/k/v projections as grouped launches (THESEUS_GROUPED_GEMM=0: three launches each, for comparison).
  static bool grouped() {
    static const bool on = [] {
      const char* e = getenv("THESEUS_GROUPED_GEMM");
      return !(e && e[0] == '0');
    }();
    return on;
  }

  static at::Tensor mm(const at::Tensor& a, const at::Tensor& b, bool b_t) {
    return gemm(a, false, b, b_t, 0, 1.0, c10::nullopt, 0);
  }
  // Gradient of a big matrix: stored on the first micro-step of an update, accumulated after.
  void grad(const at::Tensor& a, bool a_t, const at::Tensor& b, bool b_t, const char* name, bool first) {
    gemm(a, a_t, b, b_t, first ? 1 : 2, 1.0, G_.at(name), 0);
  }
  // LoRA gradient: always accumulated (the tail of the flat buffer was cleared on the first micro-step).
  void acc(const at::Tensor& a, const at::Tensor& b, const char* name) {
    gemm(a, true, b, true, 2, 1.0, G_.at(name), 0);
  }

  Saved run_forward(at::Tensor x_in, c10::optional<at::Tensor> shift, c10::optional<at::Tensor> wkv0, bool keep) {
    Saved s;
    const int64_t B = x_in.size(0), T = x_in.size(1), C = x_in.size(2), M = B * T, H = H_, N = N_;
    s.x = x_in.to(at::kBFloat16).contiguous();
    auto zeros = [&](std::vector<int64_t> shape, at::ScalarType type) {  // cleared by this package's kernel
      auto t = at::empty(shape, s.x.options().dtype(type));
      check_cuda(rt_zero_f32(static_cast<float*>(t.data_ptr()), t.numel() * (long)t.element_size() / 4,
                             stream_of(t)),
                 "zero state");
      return t;
    };
    s.shift = shift.has_value() ? shift->to(at::kBFloat16).contiguous() : zeros({B, C}, at::kBFloat16);
    auto state = wkv0.has_value() ? wkv0->to(at::kFloat).contiguous() : zeros({B, H, N, N}, at::kFloat);
    s.mix = at::empty({6, M, C}, s.x.options());
    tm_mix(s.x, s.shift, P_.at("coef"), s.mix);
    auto xm = [&](int i) { return s.mix.select(0, i); };
    if (M > 32 && grouped()) {  // r, k, v as one grouped launch (three 5120-wide GEMMs alone leave most of a wave idle)
      auto rkv = gemm_group({xm(0), xm(2), xm(3)}, false, {W_.at("receptance"), W_.at("key"), W_.at("value")},
                            false, 0, 1.0, {}, 0);
      s.r = rkv[0];
      s.k = rkv[1];
      s.v = rkv[2];
    } else {  // decode-sized: split-K weight streaming per projection
      s.r = mm(xm(0), W_.at("receptance"), false);
      s.k = mm(xm(2), W_.at("key"), false);
      s.v = mm(xm(3), W_.at("value"), false);
    }
    s.hw = mm(xm(1), W_.at("w1"), true);
    act_(s.hw, 0);
    s.lw = mm(s.hw, W_.at("w2"), true);
    s.ha = mm(xm(4), W_.at("a1"), true);
    s.la = mm(s.ha, W_.at("a2"), true);
    s.hg = mm(xm(5), W_.at("g1"), true);
    act_(s.hg, 1);
    s.g = mm(s.hg, W_.at("g2"), true);
    s.w_in = at::empty_like(s.r);
    s.k_in = at::empty_like(s.r);
    s.a_in = at::empty_like(s.r);
    s.b_in = at::empty_like(s.r);
    tm_pre_wkv(s.k, s.lw, s.la, P_.at("w0"), P_.at("a0"), P_.at("k_k"), P_.at("k_a"), s.w_in, s.k_in, s.a_in, s.b_in,
               H, N);
    const std::vector<int64_t> shape = {B, T, H, N};
    auto out = wkv7_forward(s.r.view(shape), s.w_in.view(shape), s.k_in.view(shape), s.v.view(shape),
                            s.a_in.view(shape), s.b_in.view(shape), state, keep);
    s.y = out[0];
    s.end = out[1];
    s.ckpt = out[2];
    s.rec = out[3];
    s.yg = at::empty_like(s.r);
    s.gn = at::empty({M * H * 3}, s.x.options().dtype(at::kFloat));
    tm_post_wkv(s.y, s.r, s.k_in, s.v, s.g, P_.at("ln_w"), P_.at("ln_b"), P_.at("r_k"), s.yg, s.gn, H, N);
    return s;
  }

  std::map<std::string, at::Tensor> W_, P_, G_;
  c10::optional<at::Tensor> tail_;
  int64_t H_, N_;
};

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of rwkv_theseus_b200";
  m.def("wkv7_forward", &wkv7_forward, "chunked WKV7 forward (y, end state, chunk checkpoints, tcgen05 records)");
  m.def("wkv7_backward", &wkv7_backward, "chunked WKV7 backward (dr, dw, dk, dv, da, db, ds0)");
  m.def("gemm", &gemm, "tcgen05 GEMM: a_op(A) . b_op(B)^T with bf16/fp32/accumulate epilogue",
        py::arg("A"), py::arg("a_t"), py::arg("B"), py::arg("b_t"), py::arg("epi") = 0, py::arg("alpha") = 1.0,
        py::arg("out") = py::none(), py::arg("tile") = 0);
  m.def("gemm_group", &gemm_group, "up to 3 tcgen05 GEMMs of one shape in one launch (shared stream-K schedule)",
        py::arg("A"), py::arg("a_t"), py::arg("B"), py::arg("b_t"), py::arg("epi") = 0, py::arg("alpha") = 1.0,
        py::arg("outs") = std::vector<at::Tensor>(), py::arg("tile") = 0);
  m.def("gemm_set_lane", [](int64_t lane) { check_cuda(rt_gemm_set_lane((int)lane), "gemm_set_lane"); },
        "issue lane (0 or 1) of this thread's next GEMMs: each lane has its own stream-K workspace");
  m.def("gemm_set_concurrent", [](bool on) { rt_gemm_set_concurrent(on ? 1 : 0); },
        "GEMMs of both lanes may overlap: parallel split-K tile choices run as stream-K");
  m.def("gemm_fault", []() { return rt_gemm_fault(); },
        "1 if a GEMM gave up a bounded wait since the last call (then cleared); synchronizes the device");
  m.def("kl_rows", &kl_rows, "per-row KL(teacher || student) over the vocabulary in one pass", py::arg("student"),
        py::arg("teacher"));
  m.def("gemm_nmse", &gemm_nmse, "output GEMM with the NMSE/cosine loss in the epilogue: returns d loss / d p",
        py::arg("x"), py::arg("w"), py::arg("target"), py::arg("stats"), py::arg("eps"));
  m.def("gemm_swiglu", &gemm_swiglu, "silu(A . Bg^T) * (A . Bu^T) in one tcgen05 GEMM", py::arg("A"), py::arg("Bg"),
        py::arg("Bu"), py::arg("tile") = 0);
  m.def("rmsnorm_1p", &rmsnorm_1p);
  m.def("add_rmsnorm_1p", &add_rmsnorm_1p);
  m.def("conv1d_silu", &conv1d_silu);
  m.def("gated_rmsnorm", &gated_rmsnorm);
  m.def("norm_rope_", &norm_rope_);
  m.def("copy_rows_", &copy_rows_);
  m.def("embed_rows", &embed_rows, "embedding lookup (int64 ids, bf16 table) by this package's kernel");
  m.def("gdn_forward", &gdn_forward);
  m.def("tm_mix", &tm_mix);
  m.def("tm_mix_bwd", &tm_mix_bwd);
  m.def("tm_pre_wkv", &tm_pre_wkv);
  m.def("tm_post_wkv", &tm_post_wkv);
  m.def("tm_post_wkv_bwd", &tm_post_wkv_bwd);
  m.def("tm_pre_wkv_bwd", &tm_pre_wkv_bwd);
  m.def("act_", &act_);
  m.def("act_bwd_", &act_bwd_);
  m.def("nmse_loss", &nmse_loss, py::arg("pred"), py::arg("target"), py::arg("stats"), py::arg("dpred"),
        py::arg("eps"));
  m.def("flat_adamw", &flat_adamw, "norm (fixed-order sum), clip, AdamW, bf16 refresh, report; clears stats");
  m.def("flat_adamw_scratch", []() { return rt_flat_adamw_scratch(); });
  m.def("zero_", [](at::Tensor t) {
        const long bytes = t.numel() * (long)t.element_size();
        TORCH_CHECK(t.is_cuda() && t.is_contiguous() && bytes % 4 == 0, "zero_ needs a contiguous CUDA tensor of 4k bytes");
        c10::cuda::CUDAGuard guard(t.device());
        check_cuda(rt_zero_f32(static_cast<float*>(t.data_ptr()), bytes / 4, stream_of(t)), "zero");
      }, "t = 0 with this package's kernel");
  m.def("copy_", [](at::Tensor dst, at::Tensor src) {
        TORCH_CHECK(dst.is_cuda() && src.is_cuda() && dst.is_contiguous() && src.is_contiguous() &&
                        dst.scalar_type() == src.scalar_type() && dst.numel() == src.numel(),
                    "copy_ needs contiguous CUDA tensors of one dtype and size");
        c10::cuda::CUDAGuard guard(dst.device());
        check_cuda(rt_copy_bytes(dst.data_ptr(), src.data_ptr(), dst.numel() * (long)dst.element_size(),
                                 stream_of(dst)),
                   "copy");
      }, "dst = src with this package's kernel");
  m.def("to_bf16_", &to_bf16_);
  m.def("flash_attention", &flash_attention);
  m.def("exchange_update", &exchange_update, "peer-memory reduce-scatter + clip + AdamW + all-gather of one layer");
  m.def("exchange_shard", &exchange_shard);
  m.def("exchange_signal_words", []() { return rt_exchange_signal_words(); });
  m.def("ipc_export", &ipc_export);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("wkv7_chunk_len", []() { return rt_wkv7_chunk_len(); });
  m.def("wkv7_tc_fault", []() { return rt_wkv7_tc_fault() | (rt_wkv7_tc_bwd_fault() << 12); },
        "1 if a tcgen05 WKV7 kernel gave up a bounded wait since the last call (synchronizes)");
  m.def("fault_words_async", [](at::Tensor out) {
        TORCH_CHECK(out.scalar_type() == at::kInt && out.numel() >= 3 && out.is_contiguous(),
                    "fault_words_async needs a contiguous int32 tensor of 3 words");
        cudaStream_t s = at::cuda::getCurrentCUDAStream();
        int* p = out.data_ptr<int>();
        check_cuda(rt_gemm_fault_async(p, s), "gemm fault word");
        check_cuda(rt_wkv7_tc_fault_async(p + 1, s), "wkv7 forward fault word");
        check_cuda(rt_wkv7_tc_bwd_fault_async(p + 2, s), "wkv7 backward fault word");
      },
      "enqueue on the current stream: copy the GEMM / WKV7 fault words into `out` (pinned) and clear them");
  py::class_<StudentStep>(m, "StudentStep")
      .def(py::init<std::map<std::string, at::Tensor>, std::map<std::string, at::Tensor>,
                    std::map<std::string, at::Tensor>, c10::optional<at::Tensor>, int64_t, int64_t>(),
           py::arg("weights"), py::arg("params"), py::arg("grads"), py::arg("grad_tail"), py::arg("H"), py::arg("N"))
      .def("forward", &StudentStep::forward, py::arg("x"), py::arg("shift"), py::arg("wkv0"))
      .def("forward_backward", &StudentStep::forward_backward, py::arg("x"), py::arg("target"), py::arg("shift"),
           py::arg("wkv0"), py::arg("eps"), py::arg("first"), py::arg("stats"));
  m.def("wkv7_tc_enable", [](bool on) { g_wkv7_tc_enabled = on; },
        "route bf16 head-64 calls of >= 128 steps to the tcgen05 kernels (default) or to the chunk-16 kernels");
}
