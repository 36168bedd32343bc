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
