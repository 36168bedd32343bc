"""TimeMix student on CUDA: fused kernels with a hand-written backward.

Same math as ``models.timemix.TimeMix.forward`` under bf16 autocast (the
reference path, ``theseus/timemix.py:66-89``) but scheduled as:

forward
    mix (token shift, 6 lerps)                       1 kernel
    r, k, v projections; LoRA down/up for w, a, g    9 tcgen05 GEMMs (+ tanh / sigmoid)
    pre-WKV (decay, ICL rate, kk, k', a/b inputs)   1 kernel
    chunked WKV7 (chunk checkpoints kept)            1 kernel
    post-WKV (GroupNorm, bonus, output gate)         1 kernel
    output projection + NMSE/cosine row sums and     1 GEMM (loss in the epilogue; the prediction
      d loss / d prediction                            is never stored) + row prep / finish
backward
    output projection dX / dW                        2 GEMMs (dW accumulates into the fp32 flat buffer)
    post-WKV backward (+ ln_x, r_k partial sums)     1 kernel
    WKV7 backward (no history, no atomics)           1 kernel
    pre-WKV backward (+ w0, a0, k_k, k_a)            1 kernel
    projection and LoRA dX / dW                      15 GEMMs (+ 2 activation backwards)
    mix backward (x_* partial sums)                  1 kernel

Weight operands come from a bf16 copy of the flat fp32 parameters that the
optimizer kernel refreshes after every update (the value autocast would use);
transposed operands are read MN-major by the GEMM, never materialised.

Issue: the whole micro-step (and the inference forward) is one call into the
native executor ``StudentStep`` (``csrc/bindings.cpp``), which launches the
kernels above from C++; Python only passes the chunk, target and state.

CUDA graphs: a micro-step is ~40 launches whose host-side issue can still exceed
their device time on short chunks, so (config ``student_graphs``, default on) the second
micro-step of a given shape is captured once as a CUDA graph and every later one
is a replay (full ``chunk_tokens`` chunks only; the shorter last chunk of a
document runs eagerly): the chunk's input and target are copied into static buffers, the
carried state lives in static buffers (zeroed at a document boundary), and the
loss sums accumulate straight into the student's statistics tensor. The first micro-step of a shape runs
eagerly, so the GEMM tile choices are measured before any capture. All students'
graphs share one memory pool: their intermediates die inside the replay, and
replays are serialised on the training stream.
"""
import torch

from ..ops import native

_MIX = ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g")
_POOLS = {}  # device index -> memory pool shared by the micro-step graphs


class _StepGraph:
    """One captured micro-step of fixed input shape and ``first`` flag."""

    def __init__(self, fused, shape, target_dtype, first, eps, stats):
        B, T, C = shape
        dev = fused.device
        self.x = torch.zeros(B, T, C, device=dev, dtype=torch.bfloat16)
        self.y = torch.zeros(B, T, C, device=dev, dtype=target_dtype)
        self.shift = torch.zeros(B, C, device=dev, dtype=torch.bfloat16)
        self.wkv = torch.zeros(B, fused.H, fused.N, fused.N, device=dev, dtype=torch.float32)
        self.state = {"shift": self.shift, "wkv": self.wkv}
        pool = _POOLS.setdefault(dev.index, torch.cuda.graph_pool_handle())
        self.graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize(dev)
        ext = native()
        with torch.cuda.graph(self.graph, pool=pool, capture_error_mode="thread_local"):  # records, runs nothing
            new_state = fused._forward_backward(self.x, self.y, self.state, eps, stats, first)
            ext.copy_(self.shift, new_state["shift"])
            ext.copy_(self.wkv, new_state["wkv"])

    def run(self, x, target, state):
        ext = native()  # copies and clears by this package's kernels
        ext.copy_(self.x, x.contiguous())
        ext.copy_(self.y, target.contiguous())
        if state is None:
            ext.zero_(self.shift)
            ext.zero_(self.wkv)
        elif state is not self.state:
            ext.copy_(self.shift, state["shift"].to(torch.bfloat16).contiguous())
            ext.copy_(self.wkv, state["wkv"].float().contiguous())
        self.graph.replay()
        return self.state


class FusedStudent:
    def __init__(self, student):
        self.student = student
        core, flat = student.core, student.flat
        self.C, self.H, self.N = core.width, core.heads, core.head_size
        self.device = flat.param.device
        self.shadow = torch.empty(flat.numel, device=self.device, dtype=torch.bfloat16)
        self.scratch = torch.zeros(native().flat_adamw_scratch(), device=self.device)  # optimizer partial norms
        start = flat.offsets[flat.names.index("x_r")]
        if [flat.names[flat.names.index("x_r") + i] for i in range(6)] != list(_MIX):
            raise RuntimeError("unexpected flat parameter order")
        self.coef = flat.param[start:start + 6 * self.C]
        self.dcoef = flat.grad[start:start + 6 * self.C]
        self.use_graphs = bool(student.cfg.get("student_graphs", True))
        self.graphs = {}  # (shape, target dtype, first, eps) -> _StepGraph, or None after one eager run
        self.refresh_weights()
        # Native executor of the micro-step: views of the bf16 shadow weights, the fp32 vectors and the gradients.
        mats = {"receptance": "receptance.weight", "key": "key.weight", "value": "value.weight",
                "output": "output.weight", "w1": "w1", "w2": "w2", "a1": "a1", "a2": "a2", "g1": "g1", "g2": "g2"}
        vecs = {"w0": "w0", "a0": "a0", "k_k": "k_k", "k_a": "k_a", "r_k": "r_k", "ln_w": "ln_x.weight",
                "ln_b": "ln_x.bias"}
        weights = {key: self.w(name) for key, name in mats.items()}
        params = {key: self.p(name) for key, name in vecs.items()} | {"coef": self.coef}
        grads = {key: self.g(name) for key, name in mats.items()}
        grads |= {key: self.g(name).reshape(-1) for key, name in vecs.items()} | {"coef": self.dcoef}
        tail = flat.grad[student.decay_numel:]
        self.native = native().StudentStep(weights, params, grads, tail, self.H, self.N)

    # ------------------------------------------------------------------ helpers
    def refresh_weights(self):
        native().to_bf16_(self.student.flat.param, self.shadow)

    def w(self, name):
        """bf16 copy of a weight matrix."""
        return self.student.flat.view(self.shadow, name)

    def p(self, name):
        return self.student.flat.view(self.student.flat.param, name).reshape(-1)

    def g(self, name):
        return self.student.flat.view(self.student.flat.grad, name)

    @staticmethod
    def mm(a, a_t, b, b_t):
        return native().gemm(a, a_t, b, b_t, 0, 1.0, None)

    @staticmethod
    def mm_acc(grad, a, a_t, b, b_t):
        native().gemm(a, a_t, b, b_t, 2, 1.0, grad)

    def mm_grad(self, name, first, a, a_t, b, b_t):
        """Weight gradient of a big matrix: stored on the first micro-step of an update, accumulated after."""
        native().gemm(a, a_t, b, b_t, 1 if first else 2, 1.0, self.g(name))

    # ------------------------------------------------------------------ forward
    @torch.no_grad()
    def forward(self, x, state):
        """Inference forward (validation): (prediction, new state)."""
        shift, wkv0 = (None, None) if state is None else (state["shift"], state["wkv"])
        pred, new_shift, end = self.native.forward(x, shift, wkv0)
        return pred, {"shift": new_shift, "wkv": end}

    # ------------------------------------------------------------------ training micro-step
    @torch.no_grad()
    def forward_backward(self, x, target, state, eps, stats, first=False):
        """One micro-step; ``stats`` (fp32 [3], a persistent tensor) += [sum nmse, sum cos, tokens]. ``first``: the
        gradient buffer holds a finished update's values; the four big matrices' gradients are then stored (not
        accumulated) and the rest of the buffer is cleared. Returns the new state; with graphs, its tensors are
        static buffers of the step's graph that the next replay of the same shape overwrites."""
        if not self.use_graphs or x.shape[1] != self.student.cfg["chunk_tokens"]:
            # graphs only for full chunks: the shorter last chunk of a document varies in length
            return self._forward_backward(x, target, state, eps, stats, first)
        key = (tuple(x.shape), target.dtype, bool(first), float(eps), stats.data_ptr())
        step = self.graphs.get(key)
        if step is None:
            if key not in self.graphs:  # first use of this shape: eager (measures GEMM tiles), capture next time
                self.graphs[key] = None
                return self._forward_backward(x, target, state, eps, stats, first)
            step = self.graphs[key] = _StepGraph(self, tuple(x.shape), target.dtype, bool(first), float(eps), stats)
        return step.run(x, target, state)

    def _forward_backward(self, x, target, state, eps, stats, first):
        shift, wkv0 = (None, None) if state is None else (state["shift"], state["wkv"])
        new_shift, end = self.native.forward_backward(x, target, shift, wkv0, float(eps), bool(first), stats)
        return {"shift": new_shift, "wkv": end}

    # ------------------------------------------------------------------ update
    @torch.no_grad()
    def update(self, lr, step):
        st = self.student
        cfg, flat = st.cfg, st.flat
        beta1, beta2 = cfg["betas"]
        native().flat_adamw(flat.param, flat.grad, flat.exp_avg, flat.exp_avg_sq, self.shadow, st.decay_numel,
                            st.stats, self.scratch, st.report, float(lr), float(beta1), float(beta2),
                            float(cfg["adam_eps"]), float(cfg["weight_decay"]), float(cfg["clip_norm"]), int(step))


class FusedTimeMixInference:
    """Inference forward of an installed (frozen, bf16) TimeMix with the fused kernels of ``FusedStudent``.

    Same math as ``TimeMix.forward`` (reference ``theseus/timemix.py:66-89``): 1 mix kernel, the r/k/v and
    LoRA GEMMs, pre-WKV, WKV7 (token-by-token kernel for decode-sized calls), post-WKV and the output
    GEMM. The small fp32 vectors are copied once at construction; the module's weights must not change
    afterwards (installed students are frozen).
    """

    def __init__(self, core):
        self.core = core
        self.C, self.H, self.N = core.width, core.heads, core.head_size
        f32 = lambda t: t.detach().float().reshape(-1).contiguous()  # noqa: E731
        bf = lambda t: t.detach().to(torch.bfloat16).contiguous()  # noqa: E731
        params = {"coef": torch.cat([f32(getattr(core, "x_" + n)) for n in "rwkvag"])}
        params |= {n: f32(getattr(core, n)) for n in ("w0", "a0", "k_k", "k_a", "r_k")}
        params |= {"ln_w": f32(core.ln_x.weight), "ln_b": f32(core.ln_x.bias)}
        weights = {n: bf(getattr(core, n).weight) for n in ("receptance", "key", "value", "output")}
        weights |= {n: bf(getattr(core, n)) for n in ("w1", "w2", "a1", "a2", "g1", "g2")}
        self.native = native().StudentStep(weights, params, {}, None, self.H, self.N)

    @torch.no_grad()
    def __call__(self, x, state):
        shift, wkv0 = (None, None) if state is None else (state["shift"], state["wkv"])
        pred, new_shift, end = self.native.forward(x, shift, wkv0)
        return pred, {"shift": new_shift, "wkv": end}
