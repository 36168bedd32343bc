// PyTorch bindings of the sm_100a kernels. Kernels live in .cu files behind
// plain C entry points (pointers + sizes + stream); this file does the shape,
// dtype and device checks, allocates outputs, and launches on the current
// stream of the tensors' device.
#include <torch/extension.h>
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

std::vector<at::Tensor> wkv7_forward(at::Tensor r, at::Tensor w, at::Tensor k, at::Tensor v, at::Tensor a,
                                     at::Tensor b, at::Tensor s0, bool save_checkpoints) {
  check_wkv(r, {w, k, v, a, b});
  c10::cuda::CUDAGuard guard(r.device());
  const int B = r.size(0), T = r.size(1), H = r.size(2), N = r.size(3);
  TORCH_CHECK(s0.device() == r.device() && s0.scalar_type() == at::kFloat && s0.is_contiguous() &&
                  s0.sizes() == at::IntArrayRef({B, H, N, N}),
              "s0 must be contiguous CUDA fp32 [B,H,N,N]");
  const int chunks = (T + rt_wkv7_chunk_len() - 1) / rt_wkv7_chunk_len();
  auto y = at::empty_like(r);
  auto end = at::empty_like(s0);
  auto ckpt = save_checkpoints ? at::empty({B, H, chunks + 1, N, N}, s0.options()) : at::empty({0}, s0.options());
  check_cuda(rt_wkv7_forward(dtype_code(r), B, T, H, N, r.data_ptr(), w.data_ptr(), k.data_ptr(), v.data_ptr(),
                             a.data_ptr(), b.data_ptr(), s0.data_ptr<float>(), y.data_ptr(), end.data_ptr<float>(),
                             save_checkpoints ? ckpt.data_ptr<float>() : nullptr, stream_of(r)),
             "wkv7_forward");
  return {y, end, ckpt};
}

std::vector<at::Tensor> wkv7_backward(at::Tensor r, at::Tensor w, at::Tensor k, at::Tensor v, at::Tensor a,
                                      at::Tensor b, at::Tensor ckpt, at::Tensor dy, at::Tensor dend) {
  check_wkv(r, {w, k, v, a, b, dy});
  c10::cuda::CUDAGuard guard(r.device());
  const int B = r.size(0), T = r.size(1), H = r.size(2), N = r.size(3);
  const int chunks = (T + rt_wkv7_chunk_len() - 1) / rt_wkv7_chunk_len();
  TORCH_CHECK(ckpt.device() == r.device() && ckpt.scalar_type() == at::kFloat && ckpt.is_contiguous() &&
                  ckpt.sizes() == at::IntArrayRef({B, H, chunks + 1, N, N}),
              "invalid chunk checkpoints");
  TORCH_CHECK(dend.device() == r.device() && dend.scalar_type() == at::kFloat && dend.is_contiguous() &&
                  dend.sizes() == at::IntArrayRef({B, H, N, N}),
              "invalid dend");
  auto opts = r.options().dtype(at::kFloat);
  std::vector<at::Tensor> g;
  for (int i = 0; i < 6; ++i) g.push_back(at::empty(r.sizes(), opts));
  g.push_back(at::empty({B, H, N, N}, opts));
  check_cuda(rt_wkv7_backward(dtype_code(r), B, T, H, N, r.data_ptr(), w.data_ptr(), k.data_ptr(), v.data_ptr(),
                              a.data_ptr(), b.data_ptr(), ckpt.data_ptr<float>(), dy.data_ptr(),
                              dend.data_ptr<float>(), g[0].data_ptr<float>(), g[1].data_ptr<float>(),
                              g[2].data_ptr<float>(), g[3].data_ptr<float>(), g[4].data_ptr<float>(),
                              g[5].data_ptr<float>(), g[6].data_ptr<float>(), stream_of(r)),
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
at::Tensor gemm(at::Tensor A, bool a_t, at::Tensor B, bool b_t, int64_t epi, double alpha, c10::optional<at::Tensor> out) {
  c10::cuda::CUDAGuard guard(A.device());
  auto a = operand(A, "A");
  auto b = operand(B, "B");
  const long M = a_t ? A.size(1) : A.size(0), K = a_t ? A.size(0) : A.size(1);
  const long N = b_t ? B.size(1) : B.size(0), KB = b_t ? B.size(0) : B.size(1);
  TORCH_CHECK(K == KB, "GEMM inner dimensions differ: ", K, " vs ", KB);
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
  check_cuda(rt_gemm_bf16(a.ptr, a.ld, a_t, b.ptr, b.ld, b_t, C.data_ptr(), C.stride(0), M, N, K, (int)epi,
                          (float)alpha, nullptr, stream_of(A)),
             "gemm");
  return C;
}

at::Tensor gemm_swiglu(at::Tensor A, at::Tensor Bg, at::Tensor Bu) {
  c10::cuda::CUDAGuard guard(A.device());
  auto a = operand(A, "A");
  auto g = operand(Bg, "Bg");
  auto u = operand(Bu, "Bu");
  TORCH_CHECK(g.ld == u.ld && Bg.sizes() == Bu.sizes(), "gate and up weights must share shape and stride");
  const long M = A.size(0), K = A.size(1), N = Bg.size(0);
  TORCH_CHECK(Bg.size(1) == K, "SwiGLU inner dimension mismatch");
  auto C = at::empty({M, N}, A.options());
  check_cuda(rt_gemm_swiglu_bf16(a.ptr, a.ld, g.ptr, u.ptr, g.ld, C.data_ptr(), N, M, N, K, nullptr, stream_of(A)),
             "gemm_swiglu");
  return C;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of rwkv_theseus_b200";
  m.def("wkv7_forward", &wkv7_forward, "chunked WKV7 forward (y, end state, chunk checkpoints)");
  m.def("wkv7_backward", &wkv7_backward, "chunked WKV7 backward (dr, dw, dk, dv, da, db, ds0)");
  m.def("gemm", &gemm, "tcgen05 GEMM: a_op(A) . b_op(B)^T with bf16/fp32/accumulate epilogue",
        py::arg("A"), py::arg("a_t"), py::arg("B"), py::arg("b_t"), py::arg("epi") = 0, py::arg("alpha") = 1.0,
        py::arg("out") = py::none());
  m.def("gemm_swiglu", &gemm_swiglu, "silu(A . Bg^T) * (A . Bu^T) in one tcgen05 GEMM");
  m.def("wkv7_chunk_len", []() { return rt_wkv7_chunk_len(); });
}
