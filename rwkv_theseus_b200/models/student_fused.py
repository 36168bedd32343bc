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

CUDA graphs: a micro-step is ~100 launches whose host-side issue costs more than
their device time, so (config ``student_graphs``, default on) the second
micro-step of a given shape is captured once as a CUDA graph and every later one
is a replay (full ``chunk_tokens`` chunks only; the shorter last chunk of a
document runs eagerly): the chunk's input and target are copied into static buffers, the
carried state lives in static buffers (zeroed at a document boundary), and the
statistics come back through a static buffer. The first micro-step of a shape runs
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

    def __init__(self, fused, shape, target_dtype, first, eps):
        B, T, C = shape
        dev = fused.device
        self.x = torch.zeros(B, T, C, device=dev, dtype=torch.bfloat16)
        self.y = torch.zeros(B, T, C, device=dev, dtype=target_dtype)
        self.shift = torch.zeros(B, C, device=dev, dtype=torch.bfloat16)
        self.wkv = torch.zeros(B, fused.H, fused.N, fused.N, device=dev, dtype=torch.float32)
        self.stats = torch.zeros(3, device=dev)
        self.state = {"shift": self.shift, "wkv": self.wkv}
        pool = _POOLS.setdefault(dev.index, torch.cuda.graph_pool_handle())
        self.graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(self.graph, pool=pool, capture_error_mode="thread_local"):
            stats, new_state = fused._forward_backward(self.x, self.y, self.state, eps, first)
            self.stats.copy_(stats)
            self.shift.copy_(new_state["shift"])
            self.wkv.copy_(new_state["wkv"])

    def run(self, x, target, state):
        self.x.copy_(x)
        self.y.copy_(target)
        if state is None:
            self.shift.zero_()
            self.wkv.zero_()
        elif state is not self.state:
            self.shift.copy_(state["shift"])
            self.wkv.copy_(state["wkv"])
        self.graph.replay()
        return self.stats, self.state


class FusedStudent:
    def __init__(self, student):
        self.student = student
        core, flat = student.core, student.flat
        self.C, self.H, self.N = core.width, core.heads, core.head_size
        self.device = flat.param.device
        self.shadow = torch.empty(flat.numel, device=self.device, dtype=torch.bfloat16)
        self.norm2 = torch.zeros(1, device=self.device)
        start = flat.offsets[flat.names.index("x_r")]
        if [flat.names[flat.names.index("x_r") + i] for i in range(6)] != list(_MIX):
            raise RuntimeError("unexpected flat parameter order")
        self.coef = flat.param[start:start + 6 * self.C]
        self.dcoef = flat.grad[start:start + 6 * self.C]
        self.use_graphs = bool(student.cfg.get("student_graphs", True))
        self.graphs = {}  # (shape, target dtype, first, eps) -> _StepGraph, or None after one eager run
        self.refresh_weights()

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

    def _state(self, x, state):
        B = x.shape[0]
        if state is None:
            return (torch.zeros(B, self.C, device=x.device, dtype=torch.bfloat16),
                    torch.zeros(B, self.H, self.N, self.N, device=x.device, dtype=torch.float32))
        return state["shift"].to(torch.bfloat16).contiguous(), state["wkv"].float().contiguous()

    # ------------------------------------------------------------------ forward
    def _forward(self, x, state, keep, project=True):
        B, T, C = x.shape
        M, H, N = B * T, self.H, self.N
        x = x.to(torch.bfloat16).contiguous()
        shift, wkv0 = self._state(x, state)
        ext = native()
        mix = torch.empty(6, M, C, device=x.device, dtype=torch.bfloat16)
        ext.tm_mix(x, shift, self.coef, mix)
        xr, xw, xk, xv, xa, xg = mix.unbind(0)
        r = self.mm(xr, False, self.w("receptance.weight"), False)
        k = self.mm(xk, False, self.w("key.weight"), False)
        v = self.mm(xv, False, self.w("value.weight"), False)
        hw = self.mm(xw, False, self.w("w1"), True)
        ext.act_(hw, 0)
        lw = self.mm(hw, False, self.w("w2"), True)
        ha = self.mm(xa, False, self.w("a1"), True)
        la = self.mm(ha, False, self.w("a2"), True)
        hg = self.mm(xg, False, self.w("g1"), True)
        ext.act_(hg, 1)
        g = self.mm(hg, False, self.w("g2"), True)
        w_in, k_in, a_in, b_in = (torch.empty_like(r) for _ in range(4))
        ext.tm_pre_wkv(k, lw, la, self.p("w0"), self.p("a0"), self.p("k_k"), self.p("k_a"),
                       w_in, k_in, a_in, b_in, H, N)
        shape = (B, T, H, N)
        wkv_in = [t.view(shape) for t in (r, w_in, k_in, v, a_in, b_in)]
        y, end, ckpt, rec = ext.wkv7_forward(*wkv_in, wkv0, keep)
        yg = torch.empty_like(r)
        gn = torch.empty(M * H * 3, device=x.device)
        ext.tm_post_wkv(y, r, k_in, v, g, self.p("ln_x.weight"), self.p("ln_x.bias"), self.p("r_k"), yg, gn, H, N)
        pred = self.mm(yg, False, self.w("output.weight"), False) if project else None
        new_state = {"shift": x[:, -1].clone(), "wkv": end}
        saved = None
        if keep:
            saved = dict(x=x, shift=shift, mix=mix, r=r, k=k, v=v, hw=hw, ha=ha, hg=hg, lw=lw, la=la, g=g,
                         w_in=w_in, k_in=k_in, a_in=a_in, b_in=b_in, y=y, ckpt=ckpt, rec=rec, yg=yg, gn=gn)
        return pred, new_state, saved

    @torch.no_grad()
    def forward(self, x, state):
        pred, new_state, _ = self._forward(x, state, False)
        return pred.view(x.shape), new_state

    # ------------------------------------------------------------------ training micro-step
    @torch.no_grad()
    def forward_backward(self, x, target, state, eps, first=False):
        """One micro-step. ``first``: the gradient buffer holds a finished update's values; the four big
        matrices' gradients are then stored (not accumulated) and the rest of the buffer is cleared.
        Returns (statistics [3], new state); with graphs, both are static buffers of the step's graph that
        the next replay of the same shape overwrites."""
        if not self.use_graphs or x.shape[1] != self.student.cfg["chunk_tokens"]:
            # graphs only for full chunks: the shorter last chunk of a document varies in length
            return self._forward_backward(x, target, state, eps, first)
        key = (tuple(x.shape), target.dtype, bool(first), float(eps))
        step = self.graphs.get(key)
        if step is None:
            if key not in self.graphs:  # first use of this shape: eager (measures GEMM tiles), capture next time
                self.graphs[key] = None
                return self._forward_backward(x, target, state, eps, first)
            step = self.graphs[key] = _StepGraph(self, tuple(x.shape), target.dtype, bool(first), float(eps))
        return step.run(x, target, state)

    def _forward_backward(self, x, target, state, eps, first):
        B, T, C = x.shape
        M, H, N = B * T, self.H, self.N
        ext = native()
        if first:
            self.student.flat.grad[self.student.decay_numel:].zero_()
        _, new_state, s = self._forward(x, state, True, project=False)
        stats = torch.zeros(3, device=x.device)
        # output projection with the loss in its epilogue: d loss / d prediction directly (no prediction tensor)
        dpred = ext.gemm_nmse(s["yg"], self.w("output.weight"), target.reshape(M, C).to(torch.bfloat16).contiguous(),
                              stats, float(eps))
        pred = dpred  # shape/dtype template for the gradient buffers below
        # output projection
        dyg = self.mm(dpred, False, self.w("output.weight"), True)
        self.mm_grad("output.weight", first, dpred, True, s["yg"], True)
        # post-WKV backward
        dy = torch.empty_like(pred)
        dg = torch.empty_like(pred)
        bonus = [torch.empty(M, C, device=x.device) for _ in range(3)]
        ext.tm_post_wkv_bwd(dyg, s["y"], s["r"], s["k_in"], s["v"], s["g"], self.p("ln_x.weight"),
                            self.p("ln_x.bias"), self.p("r_k"), s["gn"], dy, dg, bonus[0], bonus[1], bonus[2],
                            self.g("ln_x.weight"), self.g("ln_x.bias"), self.g("r_k"), H, N)
        shape = (B, T, H, N)
        wkv_in = [s[n].view(shape) for n in ("r", "w_in", "k_in", "v", "a_in", "b_in")]
        dend = torch.zeros(B, H, N, N, device=x.device)
        gw = ext.wkv7_backward(*wkv_in, s["ckpt"], s["rec"], dy.view(shape), dend)
        dr, dk, dv, dlw, dla = (torch.empty_like(pred) for _ in range(5))
        ext.tm_pre_wkv_bwd(list(gw[:6]), bonus, s["k"], s["la"], self.p("w0"), self.p("a0"), self.p("k_k"),
                           self.p("k_a"), [dr, dk, dv, dlw, dla],
                           [self.g("w0").reshape(-1), self.g("a0").reshape(-1), self.g("k_k").reshape(-1),
                            self.g("k_a").reshape(-1)], H, N)
        del gw, bonus
        mix = s["mix"]
        dmix = torch.empty_like(mix)
        xr, xw, xk, xv, xa, xg = mix.unbind(0)
        # r, k, v projections
        for grad_out, inp, name, slot in ((dr, xr, "receptance.weight", 0), (dk, xk, "key.weight", 2),
                                          (dv, xv, "value.weight", 3)):
            ext.gemm(grad_out, False, self.w(name), True, 0, 1.0, dmix[slot])
            self.mm_grad(name, first, grad_out, True, inp, True)
        # decay LoRA: lw = tanh(xw w1) w2
        self.mm_acc(self.g("w2"), s["hw"], True, dlw, True)
        dhw = self.mm(dlw, False, self.w("w2"), False)
        ext.act_bwd_(s["hw"], dhw, 0)
        self.mm_acc(self.g("w1"), xw, True, dhw, True)
        ext.gemm(dhw, False, self.w("w1"), False, 0, 1.0, dmix[1])
        # ICL-rate LoRA: la = (xa a1) a2
        self.mm_acc(self.g("a2"), s["ha"], True, dla, True)
        dha = self.mm(dla, False, self.w("a2"), False)
        self.mm_acc(self.g("a1"), xa, True, dha, True)
        ext.gemm(dha, False, self.w("a1"), False, 0, 1.0, dmix[4])
        # gate LoRA: g = sigmoid(xg g1) g2
        self.mm_acc(self.g("g2"), s["hg"], True, dg, True)
        dhg = self.mm(dg, False, self.w("g2"), False)
        ext.act_bwd_(s["hg"], dhg, 1)
        self.mm_acc(self.g("g1"), xg, True, dhg, True)
        ext.gemm(dhg, False, self.w("g1"), False, 0, 1.0, dmix[5])
        ext.tm_mix_bwd(s["x"], s["shift"], dmix, self.dcoef)
        return stats, new_state

    # ------------------------------------------------------------------ update
    @torch.no_grad()
    def update(self, lr, step):
        st = self.student
        cfg, flat = st.cfg, st.flat
        beta1, beta2 = cfg["betas"]
        native().flat_adamw(flat.param, flat.grad, flat.exp_avg, flat.exp_avg_sq, self.shadow, st.decay_numel,
                            st.stats, self.norm2, st.report, float(lr), float(beta1), float(beta2),
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
        self.coef = torch.cat([f32(getattr(core, "x_" + n)) for n in "rwkvag"])
        self.vec = {n: f32(getattr(core, n)) for n in ("w0", "a0", "k_k", "k_a", "r_k")}
        self.ln_w, self.ln_b = f32(core.ln_x.weight), f32(core.ln_x.bias)
        bf = lambda t: t.detach().to(torch.bfloat16).contiguous()  # noqa: E731
        self.mat = {n: bf(getattr(core, n).weight) for n in ("receptance", "key", "value", "output")}
        self.mat.update({n: bf(getattr(core, n)) for n in ("w1", "w2", "a1", "a2", "g1", "g2")})

    @torch.no_grad()
    def __call__(self, x, state):
        B, T, C = x.shape
        M, H, N = B * T, self.H, self.N
        ext = native()
        mm = lambda a, b, b_t: ext.gemm(a, False, b, b_t, 0, 1.0, None)  # noqa: E731
        x = x.to(torch.bfloat16).contiguous()
        if state is None:
            shift = torch.zeros(B, C, device=x.device, dtype=torch.bfloat16)
            wkv0 = torch.zeros(B, H, N, N, device=x.device, dtype=torch.float32)
        else:
            shift, wkv0 = state["shift"].to(torch.bfloat16).contiguous(), state["wkv"].float().contiguous()
        mix = torch.empty(6, M, C, device=x.device, dtype=torch.bfloat16)
        ext.tm_mix(x, shift, self.coef, mix)
        xr, xw, xk, xv, xa, xg = mix.unbind(0)
        W = self.mat
        r, k, v = mm(xr, W["receptance"], False), mm(xk, W["key"], False), mm(xv, W["value"], False)
        hw = mm(xw, W["w1"], True)
        ext.act_(hw, 0)
        lw = mm(hw, W["w2"], True)
        la = mm(mm(xa, W["a1"], True), W["a2"], True)
        hg = mm(xg, W["g1"], True)
        ext.act_(hg, 1)
        g = mm(hg, W["g2"], True)
        w_in, k_in, a_in, b_in = (torch.empty_like(r) for _ in range(4))
        V = self.vec
        ext.tm_pre_wkv(k, lw, la, V["w0"], V["a0"], V["k_k"], V["k_a"], w_in, k_in, a_in, b_in, H, N)
        shape = (B, T, H, N)
        y, end, _, _ = ext.wkv7_forward(*[t.view(shape) for t in (r, w_in, k_in, v, a_in, b_in)], wkv0, False)
        yg = torch.empty_like(r)
        gn = torch.empty(M * H * 3, device=x.device)
        ext.tm_post_wkv(y, r, k_in, v, g, self.ln_w, self.ln_b, V["r_k"], yg, gn, H, N)
        out = mm(yg, W["output"], False)
        return out.view(B, T, C), {"shift": x[:, -1].clone(), "wkv": end}
