"""Chunkwise mLSTM backward: replaces TFLAFunction.backward's re-run of the step
loop under autograd (hybrid_xmamba/kernels/tfla/tfla_interface.py:52-81).

Per (b, h) and chunk of ``chunk`` steps (key channel j, b_t the in-chunk sum
of log f up to t, g its chunk total, rho = g / 2):

    Qs = q e^(b - rho),  Ks = k e^(log_i + rho - b)         (hxm_mlstm_bwd_prepare)
    state entering chunk k:  X_k  (dqk x (dv + 1), the normalizer n as the
    column of ones appended to v), X_{k+1} = e^g X_k + e^rho Ks^T [v | 1]
                                                             (hxm_chunk_state_scan)
    S = causal(Qs Ks^T),  [num | den] = (e^rho Qs) X_k + S [v | 1]
    dnum = dh / max(den, 1),  dden = -[den >= 1] (dh . h) / max(den, 1)
    adjoint leaving chunk k:  Y_k = e^g Y_{k+1} + (e^rho Qs)^T [dnum | dden]
                                                             (hxm_chunk_state_scan, reverse)
    dS = causal([dnum | dden] [v | 1]^T)
    dL/dQs = dS Ks + e^rho ([dnum | dden] X_k^T)
    dL/dKs = dS^T Qs + e^rho ([v | 1] Y_k^T)
    dv = S^T dnum + (e^rho Ks) Y_k[:, :dv]
    dq, dk, dlog_i, dlog_f, di                               (hxm_mlstm_bwd_finalize)

The chunk GEMMs are batched fp32 cuBLAS calls (torch.matmul); the gate
scaling, the two chunk-level recurrences and the gate gradients (a suffix sum
over the whole sequence) are this library's kernels.  Memory: two fp32 state
arrays of (B, H, L / chunk, dqk, dv + 1).  Exponents are bounded by half of a
chunk's total log forget gate, which must stay above about -170 per channel
for 64-step chunks.
"""
from __future__ import annotations

import torch

from ... import _lib
from .._common import dtype_code, ptr, require_cuda, stream_of

__all__ = ["mlstm_chunkwise_bwd"]


def _scan(x, decay, reverse, stream):
    a = _lib.ChunkScanArgs()
    a.groups, a.nchunks, a.rows, a.cols = x.shape[0] * x.shape[1], x.shape[2], x.shape[3], x.shape[4]
    a.x, a.decay, a.reverse = ptr(x), ptr(decay), int(reverse)
    _lib.call("hxm_chunk_state_scan", a, stream)


def mlstm_chunkwise_bwd(q, k, v, log_i, log_f, dh, *, chunk: int = 64, gate_grads: str = "auto"):
    """Gradients of h = mLSTM(q, k, v, log_i, log_f) from a zero state.

    q, k (B, H, L, Dqk), v (B, H, L, Dv) bf16 or fp32; log_i, log_f fp32 per
    head (B, H, L) or per channel (B, H, L, Dqk); dh (B, H, L, Dv).  Returns
    fp32 (dq, dk, dv, dlog_i, dlog_f, di): di is the gradient for the gate
    value i = exp(log_i), formed without dividing by i.  Gate gradients are
    per head for per-head gates unless gate_grads="channel" (the per-channel
    values, e.g. for gates given as expanded (B, H, L, Dqk) views).
    """
    who = "mlstm_chunkwise_bwd"
    dev = require_cuda(q, k, v, log_i, log_f, dh, who=who)
    bsz, nh, L, dqk = q.shape
    dv = v.shape[-1]
    if k.shape != q.shape or v.shape[:3] != q.shape[:3] or dh.shape != v.shape:
        raise ValueError(f"{who}: q, k (B,H,L,Dqk), v and dh (B,H,L,Dv) expected")
    if log_i.shape == (bsz, nh, L) and log_f.shape == (bsz, nh, L):
        gate_mode = 0
    elif log_i.shape == (bsz, nh, L, dqk) and log_f.shape == (bsz, nh, L, dqk):
        gate_mode = 1
    else:
        raise ValueError(f"{who}: gates must be (B,H,L) or (B,H,L,Dqk); got {tuple(log_i.shape)} {tuple(log_f.shape)}")
    f32 = dict(device=dev, dtype=torch.float32)
    per_channel_out = gate_mode == 1 or gate_grads == "channel"
    if L == 0:
        z = lambda *s: torch.zeros(*s, **f32)
        gs = (bsz, nh, L, dqk) if per_channel_out else (bsz, nh, L)
        return z(bsz, nh, L, dqk), z(bsz, nh, L, dqk), z(bsz, nh, L, dv), z(*gs), z(*gs), z(*gs)
    io = q.dtype if q.dtype in (torch.float32, torch.bfloat16) else torch.float32
    unit = lambda t: t if t.stride(-1) == 1 else t.contiguous()
    q, k = (unit(t if t.dtype == io else t.to(io)) for t in (q, k))
    gi, gf = log_i.float(), log_f.float()
    if gate_mode == 1:
        gi, gf = unit(gi), unit(gf)
    c = int(chunk)
    nch = (L + c - 1) // c
    Lp = nch * c
    st = stream_of(dev)

    qs = torch.empty(bsz, nh, Lp, dqk, **f32)
    ks = torch.empty_like(qs)
    rho, erho, eg = (torch.empty(bsz, nh, nch, dqk, **f32) for _ in range(3))
    a = _lib.MlstmBwdArgs()
    a.batch, a.heads, a.seqlen, a.dqk, a.chunk, a.gate_mode = bsz, nh, L, dqk, c, gate_mode
    a.io_dtype = dtype_code(q)
    a.q, a.q_stride = ptr(q), q.stride()[:3]
    a.k, a.k_stride = ptr(k), k.stride()[:3]
    a.log_i, a.i_stride = ptr(gi), gi.stride()[:3]
    a.log_f, a.f_stride = ptr(gf), gf.stride()[:3]
    a.q_scaled, a.k_scaled, a.rho, a.e_rho, a.e_g = ptr(qs), ptr(ks), ptr(rho), ptr(erho), ptr(eg)
    _lib.call("hxm_mlstm_bwd_prepare", a, st)

    Qc = qs.view(bsz, nh, nch, c, dqk)
    Kc = ks.view(bsz, nh, nch, c, dqk)
    er = erho.unsqueeze(-2)  # (B, H, nch, 1, Dqk)
    va = torch.zeros(bsz, nh, Lp, dv + 1, **f32)
    va[:, :, :L, :dv] = v
    va[..., dv] = 1.0
    Vc = va.view(bsz, nh, nch, c, dv + 1)
    dhp = torch.zeros(bsz, nh, Lp, dv, **f32)
    dhp[:, :, :L] = dh
    dHc = dhp.view(bsz, nh, nch, c, dv)

    Kr = Kc * er
    X = torch.matmul(Kr.transpose(-1, -2), Vc)  # increments -> states entering each chunk
    _scan(X, eg, False, st)
    causal = torch.ones(c, c, device=dev, dtype=torch.bool).tril_()
    S = torch.matmul(Qc, Kc.transpose(-1, -2)).masked_fill_(~causal, 0.0)
    Qr = Qc * er
    numa = torch.matmul(Qr, X).add_(torch.matmul(S, Vc))
    num, den = numa[..., :dv], numa[..., dv]
    Dm = den.clamp(min=1.0)
    dnum = dHc / Dm.unsqueeze(-1)
    dden = -(den >= 1.0).float() * (dnum * num).sum(-1) / Dm
    dNa = torch.cat([dnum, dden.unsqueeze(-1)], -1)
    Y = torch.matmul(Qr.transpose(-1, -2), dNa)  # increments -> adjoints leaving each chunk
    _scan(Y, eg, True, st)
    dS = torch.matmul(dNa, Vc.transpose(-1, -2)).masked_fill_(~causal, 0.0)
    dQs = torch.matmul(dS, Kc).add_(er * torch.matmul(dNa, X.transpose(-1, -2)))
    dKs = torch.matmul(dS.transpose(-1, -2), Qc).add_(er * torch.matmul(Vc, Y.transpose(-1, -2)))
    dVa = torch.matmul(S.transpose(-1, -2), dNa).add_(torch.matmul(Kr, Y))
    dv_out = dVa.view(bsz, nh, Lp, dv + 1)[:, :, :L, :dv]

    dq, dk, dli, dlf, di = (torch.empty(bsz, nh, L, dqk, **f32) for _ in range(5))
    csum = torch.empty(bsz, nh, nch, dqk, **f32)
    a.dq_scaled, a.dk_scaled, a.chunk_sum = ptr(dQs), ptr(dKs), ptr(csum)
    a.dq, a.dk, a.dlog_i, a.dlog_f, a.d_i = ptr(dq), ptr(dk), ptr(dli), ptr(dlf), ptr(di)
    _lib.call("hxm_mlstm_bwd_finalize", a, st)
    if not per_channel_out:
        dli, dlf, di = dli.sum(-1), dlf.sum(-1), di.sum(-1)
    return dq, dk, dv_out, dli, dlf, di
