"""WKV7 forward in chunked WY form, in plain PyTorch: the algebra a tensor-core chunk kernel implements.

The per-token recurrence (``ops.wkv7.reference``; reference ``theseus/wkv7.py:16-28``) is, per head with
state S[i][j] (value i, key j),

    S_t = S_{t-1} diag(d_t) + (S_{t-1} a_t) b_t^T + v_t k_t^T,   y_t = S_t r_t,   d_t = exp(-e^{-1/2} sigmoid(w_t)).

Inside a chunk of L steps let Lambda_t = sum_{tau <= t} log d_tau (per key, Lambda_{-1} = 0) and

    a~_t = e^{Lambda_{t-1}} a_t,  r~_t = e^{Lambda_t} r_t,  b~_s = e^{-Lambda_s} b_s,  k~_s = e^{-Lambda_s} k_s,
    M_ab[t][s] = a~_t . b~_s (s < t),  M_ak = a~ . k~ (s < t),  M_rb = r~ . b~ (s <= t),  M_rk = r~ . k~ (s <= t).

With u_t = S_{t-1} a_t (rows of U) and S0 the chunk-start state:

    U = (I - M_ab)^{-1} (A~ S0^T + M_ak V)          (unit lower-triangular solve)
    Y = R~ S0^T + M_rb U + M_rk V
    S_L = S0 diag(e^{Lambda_{L-1}}) + U^T B^ + V^T K^,   B^ = e^{Lambda_{L-1}} b~,  K^ = e^{Lambda_{L-1}} k~.

Every exponent that reaches a product is a difference Lambda_t - Lambda_s <= 0 or Lambda_{L-1} - Lambda_s <= 0
once the factors are paired, and e^{-Lambda_s} stays below e^{0.61 L} (about 7e16 for L = 64), inside fp32 range.
All chunk terms except the three S0 products are state-free, so they can be formed for every chunk in parallel;
the serial pass per chunk is U, Y and the state update.
"""
import torch

from .wkv7 import LOG_DECAY_SCALE


def wkv7_chunked(r, w, k, v, a, b, state, chunk=64, dtype=torch.float64):
    """Chunked WY evaluation of the WKV7 forward; inputs [B, T, H, N], state [B, H, N, N]. Returns (y, final
    state) in `dtype` (float64 by default: this is an oracle for the chunk algebra, not a fast path)."""
    B, T, H, N = r.shape
    r, w, k, v, a, b = [x.to(dtype) for x in (r, w, k, v, a, b)]
    logd = -LOG_DECAY_SCALE * torch.sigmoid(w)                       # log d_t, [B, T, H, N]
    S = state.to(dtype).clone()                                      # [B, H, N(i), N(j)]
    ys = []
    for t0 in range(0, T, chunk):
        t1 = min(T, t0 + chunk)
        L = t1 - t0
        sl = lambda x: x[:, t0:t1].transpose(1, 2)                   # noqa: E731  [B, H, L, N]
        rc, kc, vc, ac, bc, ld = map(sl, (r, k, v, a, b, logd))
        lam = torch.cumsum(ld, 2)                                    # Lambda_t
        lam_prev = torch.cat([torch.zeros_like(lam[:, :, :1]), lam[:, :, :-1]], 2)
        at, rt = ac * torch.exp(lam_prev), rc * torch.exp(lam)
        bt, kt = bc * torch.exp(-lam), kc * torch.exp(-lam)
        strict = torch.tril(torch.ones(L, L, dtype=torch.bool, device=r.device), -1)
        incl = torch.tril(torch.ones(L, L, dtype=torch.bool, device=r.device))
        m_ab = (at @ bt.transpose(-1, -2)) * strict
        m_ak = (at @ kt.transpose(-1, -2)) * strict
        m_rb = (rt @ bt.transpose(-1, -2)) * incl
        m_rk = (rt @ kt.transpose(-1, -2)) * incl
        eye = torch.eye(L, dtype=dtype, device=r.device)
        rhs = at @ S.transpose(-1, -2) + m_ak @ vc                   # [B, H, L, N(i)]
        U = torch.linalg.solve_triangular(eye - m_ab, rhs, upper=False, unitriangular=True)
        Y = rt @ S.transpose(-1, -2) + m_rb @ U + m_rk @ vc
        lam_last = lam[:, :, -1:]                                    # Lambda_{L-1}
        bh, kh = bt * torch.exp(lam_last), kt * torch.exp(lam_last)
        S = S * torch.exp(lam_last) + U.transpose(-1, -2) @ bh + vc.transpose(-1, -2) @ kh
        ys.append(Y.transpose(1, 2))                                 # [B, L, H, N]
    return torch.cat(ys, 1), S


def wkv7_chunked_backward(r, w, k, v, a, b, state, dy, dstate_end, chunk=64, dtype=torch.float64):
    """Explicit chunked backward of wkv7_chunked (no autograd): gradients (dr, dw, dk, dv, da, db, dstate0) for
    output gradients dy [B, T, H, N] and a final-state gradient [B, H, N, N]. Per chunk, from its chunk-start
    state S0 (recomputed by a forward pass) and the chunk-end state gradient dS:

        dU = M_rb^T dY + B^ dS^T,   dZ = W^T dU,   dV = M_rk^T dY + M_ak^T dZ + K^ dS^T,
        dS0 = dS D_L + dY^T R~ + dZ^T A~,
        dM_rb = (dY U^T) incl,  dM_rk = (dY V^T) incl,  dM_ab = (dZ U^T) strict,  dM_ak = (dZ V^T) strict,
        dA~ = dZ S0 + dM_ab B~ + dM_ak K~,   dR~ = dY S0 + dM_rb B~ + dM_rk K~,
        dB~ = dM_ab^T A~ + dM_rb^T R~ + (U dS) D_L,   dK~ = dM_ak^T A~ + dM_rk^T R~ + (V dS) D_L,

    then the decayed vectors map back to the raw inputs and to d Lambda, which a reverse cumulative sum turns into
    d log d_t and the sigmoid's derivative into dw."""
    B, T, H, N = r.shape
    r, w, k, v, a, b = [x.to(dtype) for x in (r, w, k, v, a, b)]
    dy, dS = dy.to(dtype), dstate_end.to(dtype).clone()
    sg = torch.sigmoid(w)
    logd = -LOG_DECAY_SCALE * sg
    starts, S = [], state.to(dtype).clone()  # chunk-start states, forward
    bounds = [(t0, min(T, t0 + chunk)) for t0 in range(0, T, chunk)]
    for t0, t1 in bounds:
        starts.append(S)
        _, S = wkv7_chunked(r[:, t0:t1], w[:, t0:t1], k[:, t0:t1], v[:, t0:t1], a[:, t0:t1], b[:, t0:t1], S,
                            chunk=t1 - t0, dtype=dtype)
    grads = {n: torch.zeros_like(r) for n in ("r", "w", "k", "v", "a", "b")}
    for (t0, t1), S0 in reversed(list(zip(bounds, starts))):
        L = t1 - t0
        sl = lambda x: x[:, t0:t1].transpose(1, 2)                   # noqa: E731  [B, H, L, N]
        rc, kc, vc, ac, bc, ld, dY = map(sl, (r, k, v, a, b, logd, dy))
        lam = torch.cumsum(ld, 2)
        lam_prev = torch.cat([torch.zeros_like(lam[:, :, :1]), lam[:, :, :-1]], 2)
        At, Rt = ac * torch.exp(lam_prev), rc * torch.exp(lam)
        Bt, Kt = bc * torch.exp(-lam), kc * torch.exp(-lam)
        DL = torch.exp(lam[:, :, -1:])                               # [B, H, 1, N]
        Bh, Kh = Bt * DL, Kt * DL
        strict = torch.tril(torch.ones(L, L, dtype=torch.bool, device=r.device), -1).to(dtype)
        incl = torch.tril(torch.ones(L, L, dtype=torch.bool, device=r.device)).to(dtype)
        Mab, Mak = (At @ Bt.transpose(-1, -2)) * strict, (At @ Kt.transpose(-1, -2)) * strict
        Mrb, Mrk = (Rt @ Bt.transpose(-1, -2)) * incl, (Rt @ Kt.transpose(-1, -2)) * incl
        eye = torch.eye(L, dtype=dtype, device=r.device)
        Z = At @ S0.transpose(-1, -2) + Mak @ vc
        U = torch.linalg.solve_triangular(eye - Mab, Z, upper=False, unitriangular=True)
        # state-side gradients
        dU = Mrb.transpose(-1, -2) @ dY + Bh @ dS.transpose(-1, -2)
        dZ = torch.linalg.solve_triangular((eye - Mab).transpose(-1, -2), dU, upper=True, unitriangular=True)
        dV = Mrk.transpose(-1, -2) @ dY + Mak.transpose(-1, -2) @ dZ + Kh @ dS.transpose(-1, -2)
        dS_prev = dS * DL + dY.transpose(-1, -2) @ Rt + dZ.transpose(-1, -2) @ At
        # chunk-matrix gradients
        dMrb, dMrk = (dY @ U.transpose(-1, -2)) * incl, (dY @ vc.transpose(-1, -2)) * incl
        dMab, dMak = (dZ @ U.transpose(-1, -2)) * strict, (dZ @ vc.transpose(-1, -2)) * strict
        dBh, dKh = U @ dS, vc @ dS                                   # through S_L = S0 D + U^T B^ + V^T K^
        dAt = dZ @ S0 + dMab @ Bt + dMak @ Kt
        dRt = dY @ S0 + dMrb @ Bt + dMrk @ Kt
        dBt = dMab.transpose(-1, -2) @ At + dMrb.transpose(-1, -2) @ Rt + dBh * DL
        dKt = dMak.transpose(-1, -2) @ At + dMrk.transpose(-1, -2) @ Rt + dKh * DL
        # raw inputs and d Lambda
        dlam = dRt * Rt - dBt * Bt - dKt * Kt                        # at step t
        dlam_prev = dAt * At                                         # belongs to step t-1
        dlam = dlam + torch.cat([dlam_prev[:, :, 1:], torch.zeros_like(dlam_prev[:, :, :1])], 2)
        dDL = (dS * S0).sum(-2, keepdim=True) * DL + (dBh * Bh).sum(-2, keepdim=True) + (dKh * Kh).sum(-2, keepdim=True)
        dlam[:, :, -1:] += dDL
        dlogd = torch.flip(torch.cumsum(torch.flip(dlam, [2]), 2), [2])  # d log d_tau = sum_{t >= tau} dLambda_t
        put = lambda name, x: grads[name][:, t0:t1].copy_(x.transpose(1, 2))  # noqa: E731
        put("r", dRt * torch.exp(lam))
        put("a", dAt * torch.exp(lam_prev))
        put("b", dBt * torch.exp(-lam))
        put("k", dKt * torch.exp(-lam))
        put("v", dV)
        sgc = sl(sg)
        put("w", dlogd * (-LOG_DECAY_SCALE) * sgc * (1 - sgc))
        dS = dS_prev
    return grads["r"], grads["w"], grads["k"], grads["v"], grads["a"], grads["b"], dS
