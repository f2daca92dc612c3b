"""float64 numpy restatements of the reference's recurrent loops (oracle).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Each function follows the reference loop step for step, vectorised over the
independent axes (batch, channels, heads) exactly as the reference vectorises
them with torch, and additionally returns the final recurrent state that the
reference keeps local.  All arithmetic is float64 so the oracle's own rounding
is far below every tolerance used against it.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "softplus",
    "silu",
    "sigmoid",
    "logsigmoid",
    "selective_scan",
    "tfla_recurrent",
    "ssd_scan",
    "slstm_recurrent",
    "rmsnorm",
    "causal_conv1d",
]


def softplus(x):
    """torch.nn.functional.softplus (beta=1, threshold=20), in float64."""
    x = np.asarray(x, dtype=np.float64)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def sigmoid(x):
    x = np.asarray(x, dtype=np.float64)
    return 0.5 * (1.0 + np.tanh(0.5 * x))


def logsigmoid(x):
    x = np.asarray(x, dtype=np.float64)
    return -softplus(-x)


def silu(x):
    x = np.asarray(x, dtype=np.float64)
    return x * sigmoid(x)


def rmsnorm(x, weight, eps=1e-6):
    """RMSNorm.forward (hybrid_xmamba/layers/normalization.py:32-34)."""
    x = np.asarray(x, dtype=np.float64)
    rms = np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return np.asarray(weight, np.float64) * (x / rms)


def causal_conv1d(x, weight, bias=None, *, activation=None, init_state=None):
    """The Mamba pre-scan convolution (hybrid_xmamba/layers/mamba_block.py:101-104):
    nn.Conv1d(D, D, K, groups=D, padding=K-1) over (B, D, L), trimmed to the
    first L outputs, optionally followed by SiLU; here on x (B, L, D):
        out[b, t, c] = bias[c] + sum_k weight[c, k] * x[b, t - (K-1) + k, c]
    with x before t = 0 from init_state (B, D, K-1) or zero.
    Returns (out, final_state) — final_state[b, c, j] = x[b, L-(K-1)+j, c]."""
    x = np.asarray(x, np.float64)
    w = np.asarray(weight, np.float64).reshape(np.shape(weight)[0], -1)
    bsz, L, d = x.shape
    K = w.shape[1]
    pre = np.zeros((bsz, K - 1, d)) if init_state is None else np.swapaxes(np.asarray(init_state, np.float64), 1, 2)
    xp = np.concatenate([pre, x], axis=1)                      # (B, K-1+L, D)
    out = np.zeros((bsz, L, d)) + (0.0 if bias is None else np.asarray(bias, np.float64))
    for k in range(K):
        out += w[:, k] * xp[:, k:k + L, :]
    if activation == "silu":
        out = silu(out)
    fin = np.swapaxes(xp[:, xp.shape[1] - (K - 1):, :], 1, 2) if K > 1 else np.zeros((bsz, d, 0))
    return out, fin


def selective_scan(x, dt, A, B, C, D=None, z=None, *, z_mode="mul",
                   delta_bias=None, delta_softplus=False,
                   discretization="euler", h0=None):
    """Selective scan in the reference (batch, seqlen, dim) layout.

    Follows ``selective_scan_pytorch`` (hybrid_xmamba/kernels/selective_scan/
    scan_interface.py:103-152) for ``discretization="euler"``:
        A_discrete = exp(A * dt_t)                               (:140)
        h = A_discrete * h + (dt_t * x_t) * B_t                  (:143-144)
        y_t = sum(h * C_t, -1) + D * x_t                          (:147-148)
    and the Triton kernel's ZOH/Taylor rule (scan_triton.py:135-160) for
    ``discretization="zoh"``:  Bbar = (exp(dA)-1)/A * B, or dt*B if |dA|<0.01.
    ``z`` gating: ``z_mode="mul"`` is ``y * z`` (scan_interface.py:57-58);
    ``"silu"`` is ``y * silu(z)`` (mamba_block.py:130).
    ``delta_bias``/``delta_softplus`` apply softplus(dt + bias) first
    (mamba_block.py:115-116 with dt_proj's bias folded in).

    Shapes: x, dt, z (Bt, L, Dm); A (Dm, N); B, C (Bt, L, N); D (Dm,);
    h0 (Bt, Dm, N).  Returns (y (Bt, L, Dm), h_final (Bt, Dm, N)).
    """
    x = np.asarray(x, np.float64)
    dt = np.asarray(dt, np.float64)
    A = np.asarray(A, np.float64)
    B = np.asarray(B, np.float64)
    C = np.asarray(C, np.float64)
    bt, L, dm = x.shape
    n = A.shape[1]
    if delta_bias is not None:
        dt = dt + np.asarray(delta_bias, np.float64)[None, None, :]
    if delta_softplus:
        dt = softplus(dt)
    h = np.zeros((bt, dm, n)) if h0 is None else np.array(h0, np.float64, copy=True)
    Dv = None if D is None else np.asarray(D, np.float64)
    y = np.empty((bt, L, dm))
    for t in range(L):
        x_t = x[:, t, :]
        dt_t = dt[:, t, :]
        dA = A[None, :, :] * dt_t[:, :, None]
        A_bar = np.exp(dA)
        if discretization == "euler":
            Bbar = dt_t[:, :, None] * B[:, t, None, :]
        elif discretization == "zoh":
            taylor = dt_t[:, :, None] * B[:, t, None, :]
            with np.errstate(divide="ignore", invalid="ignore"):
                exact = (A_bar - 1.0) / A[None, :, :] * B[:, t, None, :]
            Bbar = np.where(np.abs(dA) < 0.01, taylor, exact)
        else:
            raise ValueError(discretization)
        h = A_bar * h + Bbar * x_t[:, :, None]
        y_t = np.sum(h * C[:, t, None, :], axis=-1)
        if Dv is not None:
            y_t = y_t + Dv[None, :] * x_t
        y[:, t, :] = y_t
    if z is not None:
        z = np.asarray(z, np.float64)
        if z_mode == "mul":
            y = y * z
        elif z_mode == "silu":
            y = y * silu(z)
        else:
            raise ValueError(z_mode)
    return y, h


def tfla_recurrent(q, k, v, i_gate, f_gate, C0=None, n0=None):
    """mLSTM recurrence of ``tfla_forward_pytorch``
    (hybrid_xmamba/kernels/tfla/tfla_interface.py:84-139), float64.

    q, k, v, i_gate, f_gate: (B, H, L, D) with i_gate = exp(preact) and
    f_gate in (0, 1) already applied (the reference takes activated gates).
        C = f_t[..., None] * C + i_t[..., None] * (k_t v_t^T)     (:122-128)
        n = f_t * n + i_t * k_t                                     (:123,129)
        h_t = (q_t C) / clamp(q_t . n, min=1)                       (:132-136)
    Gates broadcast from (B, H, L) to (B, H, L, D) when given per head.
    Returns (h (B,H,L,Dv), C (B,H,Dk,Dv), n (B,H,Dk)).
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    bsz, nh, L, dk = q.shape
    dv = v.shape[-1]
    ig = np.asarray(i_gate, np.float64)
    fg = np.asarray(f_gate, np.float64)
    if ig.ndim == 3:
        ig = np.broadcast_to(ig[..., None], (bsz, nh, L, dk))
    if fg.ndim == 3:
        fg = np.broadcast_to(fg[..., None], (bsz, nh, L, dk))
    C = np.zeros((bsz, nh, dk, dv)) if C0 is None else np.array(C0, np.float64, copy=True)
    n = np.zeros((bsz, nh, dk)) if n0 is None else np.array(n0, np.float64, copy=True)
    out = np.empty((bsz, nh, L, dv))
    for t in range(L):
        q_t, k_t, v_t = q[:, :, t], k[:, :, t], v[:, :, t]
        i_t, f_t = ig[:, :, t], fg[:, :, t]
        C = f_t[..., None] * C + i_t[..., None] * (k_t[..., :, None] * v_t[..., None, :])
        n = f_t * n + i_t * k_t
        num = np.einsum("bhd,bhde->bhe", q_t, C)
        den = np.maximum(np.einsum("bhd,bhd->bh", q_t, n), 1.0)[..., None]
        out[:, :, t] = num / den
    return out, C, n


def ssd_scan(x, dt, A, B, C, D=None, *, dt_bias=None, dt_softplus=False, h0=None):
    """Mamba-2 SSD (ngroups=1) as the reference's Euler selective scan.

    The reference has no SSD kernel; with channel d = (head, p) the SSD
    recurrence is exactly ``selective_scan_pytorch`` (scan_interface.py:
    103-152) with A[d, :] = A[head], delta[b, t, d] = dt[b, t, head] and the
    shared B, C.  x (Bt, L, H, P); dt (Bt, L, H); A, D, dt_bias (H,);
    B, C (Bt, L, N); h0 (Bt, H, P, N).  Returns (y (Bt,L,H,P), h (Bt,H,P,N)).
    """
    x = np.asarray(x, np.float64)
    bt, L, nh, p = x.shape
    n = np.asarray(B).shape[-1]
    dt = np.asarray(dt, np.float64)
    if dt_bias is not None:
        dt = dt + np.asarray(dt_bias, np.float64)[None, None, :]
    if dt_softplus:
        dt = softplus(dt)
    A = np.asarray(A, np.float64)
    A_full = np.repeat(A[:, None], p, axis=0)[:, None].repeat(n, axis=1).reshape(nh * p, n)
    dt_full = np.repeat(dt, p, axis=2)  # (bt, L, H*P) with head-major channels
    D_full = None if D is None else np.repeat(np.asarray(D, np.float64), p)
    h0_full = None if h0 is None else np.asarray(h0, np.float64).reshape(bt, nh * p, n)
    y, h = selective_scan(x.reshape(bt, L, nh * p), dt_full, A_full, B, C, D_full, h0=h0_full)
    return y.reshape(bt, L, nh, p), h.reshape(bt, nh, p, n)


def slstm_recurrent(gates_pre, norm_weight, *, R=None, eps=1e-6,
                    exponential_gate=True, h0=None, c0=None):
    """sLSTM recurrence of ``sLSTMBlock.forward``
    (hybrid_xmamba/layers/slstm_block.py:91-127), float64.

    gates_pre: (B, L, H, 4, hd) = gate_proj output viewed per head, with the
    4 gate blocks in the order gates.chunk(4, -1) yields them: i, f, o, c~
    (slstm_block.py:87-91).  Per step:
        i = exp(g_i) (or sigmoid), f = sigmoid(g_f), o = sigmoid(g_o),
        c~ = tanh(g_c)                                        (:94-102)
        c = f * c + i * c~                                     (:119)
        h = o * tanh(RMSNorm_hd(c))                            (:122-125)
    ``R`` (H, hd, 4*hd) adds the block-diagonal recurrent term h_{t-1} @ R[h]
    to the pre-activations; the reference has no R (R=None reproduces it).
    h0, c0: (B, H, hd).  Returns (h_seq (B, L, H, hd), h (B,H,hd), c (B,H,hd)).
    """
    g = np.asarray(gates_pre, np.float64)
    bsz, L, nh, four, hd = g.shape
    assert four == 4
    h = np.zeros((bsz, nh, hd)) if h0 is None else np.array(h0, np.float64, copy=True)
    c = np.zeros((bsz, nh, hd)) if c0 is None else np.array(c0, np.float64, copy=True)
    Rm = None if R is None else np.asarray(R, np.float64)
    w = np.asarray(norm_weight, np.float64)
    out = np.empty((bsz, L, nh, hd))
    for t in range(L):
        gt = g[:, t]  # (B, H, 4, hd)
        if Rm is not None:
            gt = gt + np.einsum("bhd,hde->bhe", h, Rm).reshape(bsz, nh, 4, hd)
        gi, gf, go, gc = gt[:, :, 0], gt[:, :, 1], gt[:, :, 2], gt[:, :, 3]
        ig = np.exp(gi) if exponential_gate else sigmoid(gi)
        fg = sigmoid(gf)
        og = sigmoid(go)
        ct = np.tanh(gc)
        c = fg * c + ig * ct
        h = og * np.tanh(rmsnorm(c, w, eps))
        out[:, t] = h
    return out, h, c
