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
    dq, dk, dlog_i, di                                       (hxm_mlstm_bwd_finalize)
    dlog_f_t = dg_k + sum_{s >= t in chunk k} (q . dq - (i k) . d(i k))_s,
    dg_k = <Y_k, X_{k+1}> per key row (the chunk's total log forget gate
    decays the state it passes on)                           (hxm_mlstm_bwd_finalize)

That separable form serves per-channel gates.  Per-head gates take the exact
decay-matrix form (``_bwd_heads``): S = causal(Q (i k)^T) * e^(b_t - b_s) with
inter-chunk factors e^b and e^(g - b), all at most 1, so no decay overflows;
their in-chunk gate term is rowsum(W) - colsum(W) + the two inter-chunk
terms, W = dL/dS * S, with W's diagonal (the largest entries under strong
decay, present in both sums) left out exactly instead of cancelled in
rounding.

For bf16 inputs the chunk GEMMs are this library's tcgen05 kernel
(hxm_chunk_gemm, tfla_bwd_tc.py); otherwise (fp32 inputs, and per-channel
gates too strong for 128-step chunks) they are batched cuBLAS calls
(torch.matmul; fp32, or TF32 when asked for); the gate
scaling, the two chunk-level recurrences and the gate gradients (a suffix sum
over the whole sequence) are this library's kernels.  Memory: two fp32 state
arrays of (B, H, L / chunk, dqk, w), w = dv + 1 rounded up to 8.

Range (per-channel gates): the factors above are e^x with |x| at most
|g| / 2 + max |log i| over the chunk.  ``_channel_chunk`` picks the longest
chunk (the requested one, then halves down to 8 steps) for which every chunk
of the input keeps x <= MAX_EXP, so strong forget gates (e.g. logsigmoid of
N(-4, 1) pre-activations, about -520 per 128 steps) shorten the chunk instead
of overflowing; gates out of reach even at 8 steps (or not finite, f = 0)
raise.  Per-head gates need no such choice (their form has no growing factor).
"""
from __future__ import annotations

import contextlib

import torch

from ... import _lib
from .._common import dtype_code, ptr, require_cuda, stream_of

__all__ = ["mlstm_chunkwise_bwd"]

MAX_EXP = 60.0  # largest exponent of a chunk factor (fp32 holds e^88; margin for the GEMM sums)
MIN_CHUNK = 8


@contextlib.contextmanager
def _gemm_precision(tf32: bool):
    """fp32 chunk GEMMs on the TF32 tensor-core path (10-bit operands, fp32
    accumulation) while the block runs; restores the caller's setting."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = bool(tf32)
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _scan(x, decay, reverse, stream, scale=None, scaled=None):
    a = _lib.ChunkScanArgs()
    a.groups, a.nchunks, a.rows, a.cols = x.shape[0] * x.shape[1], x.shape[2], x.shape[3], x.shape[4]
    a.x, a.decay, a.reverse = ptr(x), ptr(decay), int(reverse)
    a.scale, a.scaled = ptr(scale), ptr(scaled)
    _lib.call("hxm_chunk_state_scan", a, stream)


def _out_grads(numa, dh, lp, w, normalize, st):
    """[dnum | dden | 0 ...] per chunk row (hxm_mlstm_bwd_normalizer): dh over
    max(den, 1) and the clamp branch's dden, or dh alone without the
    normalizer; zero rows past the sequence."""
    bsz, nh, L, dv = dh.shape
    if dh.dtype not in (torch.float32, torch.bfloat16):
        dh = dh.float()
    if dh.stride(-1) != 1:
        dh = dh.contiguous()
    out = torch.empty(bsz, nh, lp, w, device=dh.device, dtype=torch.float32)
    a = _lib.MlstmBwdNormArgs()
    a.batch, a.heads, a.seqlen, a.padded_len, a.dv, a.width = bsz, nh, L, lp, dv, w
    a.normalize, a.io_dtype = int(bool(normalize)), dtype_code(dh)
    a.outputs, a.out = ptr(numa), ptr(out)
    a.dh, a.dh_stride = ptr(dh), dh.stride()[:3]
    _lib.call("hxm_mlstm_bwd_normalizer", a, st)
    return out


def _chunk_dg(Y, X, dims):
    """<adjoint leaving chunk k, state leaving chunk k> = <Y_k, X_{k+1}> per
    key row (hxm_chunk_state_dot; 0 for the last chunk, whose adjoint is zero),
    summed over the rows too when dims covers them."""
    out = torch.empty(Y.shape[:4], device=Y.device, dtype=torch.float32)
    a = _lib.ChunkDotArgs()
    a.groups, a.nchunks, a.rows, a.cols = Y.shape[0] * Y.shape[1], Y.shape[2], Y.shape[3], Y.shape[4]
    a.adj, a.state, a.out = ptr(Y), ptr(X), ptr(out)
    _lib.call("hxm_chunk_state_dot", a, stream_of(Y.device))
    return out.sum(-1) if -2 in dims else out


def _bwd_heads(q, k, v, li, lf, dout, c, normalize, per_channel_out, st):
    """Per-head gates li, lf (B, H, L): the exact decay-matrix chunkwise form.
    normalize=False drops the normalizer (h = q C, the SSD recurrence)."""
    bsz, nh, L, dqk = q.shape
    dv = v.shape[-1]
    dev = q.device
    f32 = dict(device=dev, dtype=torch.float32)
    nch = (L + c - 1) // c
    Lp = nch * c
    Q = torch.zeros(bsz, nh, Lp, dqk, **f32)
    Q[:, :, :L] = q
    K = torch.zeros(bsz, nh, Lp, dqk, **f32)
    K[:, :, :L] = k
    Q, K = Q.view(bsz, nh, nch, c, dqk), K.view(bsz, nh, nch, c, dqk)
    w = (dv + int(normalize) + 7) // 8 * 8
    va = torch.zeros(bsz, nh, Lp, w, **f32)
    va[:, :, :L, :dv] = v
    if normalize:
        va[..., dv] = 1.0
    Vc = va.view(bsz, nh, nch, c, w)
    lip = torch.full((bsz, nh, Lp), float("-inf"), **f32)
    lip[:, :, :L] = li
    lfp = torch.zeros(bsz, nh, Lp, **f32)
    lfp[:, :, :L] = lf
    b = lfp.view(bsz, nh, nch, c).cumsum(-1)
    g = b[..., -1:]
    ig = torch.exp(lip).view(bsz, nh, nch, c)
    Kp = K * ig.unsqueeze(-1)
    causal = torch.ones(c, c, device=dev, dtype=torch.bool).tril_()
    Lm = torch.exp((b.unsqueeze(-1) - b.unsqueeze(-2)).masked_fill_(~causal, float("-inf")))
    eb = torch.exp(b).unsqueeze(-1)
    egb = torch.exp(g - b).unsqueeze(-1)
    eg = torch.exp(g[..., 0]).unsqueeze(-1).expand(bsz, nh, nch, dqk).contiguous()
    Kd = Kp * egb
    X = torch.matmul(Kd.transpose(-1, -2), Vc)  # increments -> states entering each chunk
    _scan(X, eg, False, st)
    S = torch.matmul(Q, Kp.transpose(-1, -2)).mul_(Lm)
    Qe = Q * eb
    QX = torch.matmul(Qe, X)
    numa = QX + torch.matmul(S, Vc) if normalize else None
    dNa = _out_grads(numa, dout, Lp, w, normalize, st).view(bsz, nh, nch, c, w)
    del numa
    Y = torch.matmul(Qe.transpose(-1, -2), dNa)  # increments -> adjoints leaving each chunk
    _scan(Y, eg, True, st)
    dSf = torch.matmul(dNa, Vc.transpose(-1, -2))  # dL/dS
    dS = dSf * Lm                                     # dL/d(Q (i k)^T)
    VY = torch.matmul(Vc, Y.transpose(-1, -2))
    dQ = torch.matmul(dS, Kp).add_(eb * torch.matmul(dNa, X.transpose(-1, -2)))
    dKp = torch.matmul(dS.transpose(-1, -2), Q).add_(egb * VY)
    dVa = torch.matmul(S.transpose(-1, -2), dNa).add_(torch.matmul(Kd, Y))
    un = lambda t: t.reshape(bsz, nh, Lp, *t.shape[4:])[:, :, :L]
    dk = ig.unsqueeze(-1) * dKp
    di_c = K * dKp                                   # per channel: k . d(i k)
    if per_channel_out:  # the gate identity per channel, in-chunk part
        db = Q * dQ - Kp * dKp
        dg = _chunk_dg(Y, X, (-1,))
    else:
        di_c = di_c.sum(-1)
        W = dSf.mul_(S)
        W.diagonal(dim1=-2, dim2=-1).zero_()  # in both sums: its net term is exactly zero
        db = W.sum(-1) - W.sum(-2) + (dNa * QX).sum(-1) - (Kd * VY).sum(-1)
        dg = _chunk_dg(Y, X, (-1, -2))
    dlf = db.flip(3).cumsum(3).flip(3).add_(dg.unsqueeze(3))
    dlf = dlf.reshape(bsz, nh, Lp, *dlf.shape[4:])[:, :, :L]
    dlf[:, :, 0] = 0.0  # f at the first step multiplies the zero state
    di = di_c.reshape(bsz, nh, Lp, *di_c.shape[4:])[:, :, :L]
    igL = torch.exp(li.float())
    dli = di * (igL.unsqueeze(-1) if per_channel_out else igL)
    return un(dQ), un(dk), un(dVa)[..., :dv], dli, dlf, di


def mlstm_chunkwise_bwd(q, k, v, log_i, log_f, dh, *, chunk: int = 64, gate_grads: str = "auto", tf32=None,
                        tensor_cores=None, precise: bool = True):
    """Gradients of h = mLSTM(q, k, v, log_i, log_f) from a zero state.

    q, k (B, H, L, Dqk), v (B, H, L, Dv) bf16 or fp32; log_i, log_f fp32 per
    head (B, H, L) or per channel (B, H, L, Dqk); dh (B, H, L, Dv).  Returns
    fp32 (dq, dk, dv, dlog_i, dlog_f, di): di is the gradient for the gate
    value i = exp(log_i), formed without dividing by i.  Gate gradients are
    per head for per-head gates unless gate_grads="channel" (the per-channel
    values, e.g. for gates given as expanded (B, H, L, Dqk) views).  tf32:
    chunk GEMMs on TF32 tensor cores (default: when q is bf16, whose own
    rounding is coarser; relative gradient error ~1e-3 — except per-channel
    gates strong enough to shorten the chunk, which run fp32) or in full fp32.
    tensor_cores: run the chunk GEMMs as hxm_chunk_gemm (tcgen05, bf16 high /
    low split operands, 128-step chunks, 64 for per-channel gates whose
    128-step factors leave e^+-MAX_EXP; the default for bf16 inputs) instead of
    the library GEMMs above (tf32 then does not apply); gates too strong for
    64-step chunk factors take the library path with a shorter chunk.
    precise (default): every fp32 operand is split (gradient error ~3e-5
    against float64); precise=False splits only the gate-scaled q, k (~1e-3,
    as TF32 GEMMs, up to ~3e-2 for per-channel gates with long memory, where
    the normalizer's dq = (C dh - n (dh . h)) / den cancels) in up to 0.7x
    the time.
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
    st = stream_of(dev)
    use_tc = (io == torch.bfloat16) if tensor_cores is None else bool(tensor_cores)
    if use_tc and io != torch.bfloat16:
        raise ValueError(f"{who}: tensor_cores needs bf16 q, k (got {io})")
    if use_tc:
        v = unit(v if v.dtype == io else v.to(io))
        from . import tfla_bwd_tc as tc
        if gate_mode == 0:
            return tc.bwd_heads_tc(q, k, v, gi, gf, dh, per_channel_out, st, split_states=precise)
        cc = _channel_chunk(gi, gf, tc.TC_CHUNKS[0])
        if cc in tc.TC_CHUNKS:
            return tc.bwd_channels_tc(q, k, v, gi, gf, dh, cc, st, split_states=precise)
        # gates too strong for 64-step chunk factors: the library path below, whose shorter
        # chunk runs fp32 GEMMs
    if gate_mode == 0:
        with _gemm_precision(io == torch.bfloat16 if tf32 is None else tf32):
            return _bwd_heads(q, k, v, gi, gf, dh, c, True, per_channel_out, st)
    cc = _channel_chunk(gi, gf, c)
    # Gates strong enough to shorten the chunk make the forget-gate gradient a difference of
    # large in-chunk sums: TF32 operands (10-bit mantissa) lose it, so those run in fp32.
    with _gemm_precision((io == torch.bfloat16 and cc == c) if tf32 is None else tf32):
        return _bwd_channels(q, k, v, gi, gf, dh, cc, st)


def _channel_chunk(gi, gf, chunk):
    """The longest chunk length <= chunk (halving, at least MIN_CHUNK) whose
    separable factors stay within e^+-MAX_EXP for these per-channel gates
    (B, H, L, Dqk): max over chunks and channels of |g| / 2 + max |log i|,
    g the chunk's total log forget gate.  Lengths are tried longest first, one
    pass over the gates and one host synchronization each (usually just one)."""
    bsz, nh, L, dqk = gf.shape
    c = int(chunk)
    if c < MIN_CHUNK:
        raise ValueError(f"mlstm_chunkwise_bwd: chunk {chunk} < {MIN_CHUNK}")
    worst = float("inf")
    while c >= MIN_CHUNK:
        nch, pad = (L + c - 1) // c, (-L) % c
        lf = gf if not pad else torch.nn.functional.pad(gf, (0, 0, 0, pad))
        li = gi if not pad else torch.nn.functional.pad(gi, (0, 0, 0, pad))
        x = lf.reshape(bsz, nh, nch, c, dqk).sum(3).mul_(-0.5).add_(li.reshape(bsz, nh, nch, c, dqk).abs().amax(3))
        worst = float(torch.nan_to_num(x.amax(), nan=float("inf")))
        if worst <= MAX_EXP:
            return c
        c //= 2
    raise RuntimeError(
        f"mlstm_chunkwise_bwd: per-channel gates out of range for the chunkwise backward (a {c * 2}-step "
        f"chunk needs e^{worst:.1f} > e^{MAX_EXP:.0f}: forget gates near 0 or not finite)")


def _bwd_channels(q, k, v, gi, gf, dh, c, st):
    """Per-channel gates: the separable chunk scaling of hxm_mlstm_bwd_prepare."""
    bsz, nh, L, dqk = q.shape
    dv = v.shape[-1]
    dev = q.device
    f32 = dict(device=dev, dtype=torch.float32)
    nch = (L + c - 1) // c
    Lp = nch * c

    qs, ks, qd, kd = (torch.empty(bsz, nh, Lp, dqk, **f32) for _ in range(4))
    rho, erho, eg = (torch.empty(bsz, nh, nch, dqk, **f32) for _ in range(3))
    a = _lib.MlstmBwdArgs()
    a.batch, a.heads, a.seqlen, a.dqk, a.chunk, a.gate_mode = bsz, nh, L, dqk, c, 1
    a.io_dtype = dtype_code(q)
    a.q, a.q_stride = ptr(q), q.stride()[:3]
    a.k, a.k_stride = ptr(k), k.stride()[:3]
    a.log_i, a.i_stride = ptr(gi), gi.stride()[:3]
    a.log_f, a.f_stride = ptr(gf), gf.stride()[:3]
    a.q_scaled, a.k_scaled, a.rho, a.e_rho, a.e_g = ptr(qs), ptr(ks), ptr(rho), ptr(erho), ptr(eg)
    a.q_decayed, a.k_decayed = ptr(qd), ptr(kd)
    _lib.call("hxm_mlstm_bwd_prepare", a, st)

    Qc = qs.view(bsz, nh, nch, c, dqk)
    Kc = ks.view(bsz, nh, nch, c, dqk)
    Qr = qd.view(bsz, nh, nch, c, dqk)  # e^rho Qs = q e^b
    Kr = kd.view(bsz, nh, nch, c, dqk)  # e^rho Ks = i k e^(g - b)
    w = (dv + 1 + 7) // 8 * 8  # [v | 1 | 0 ...]: rows of 32-byte multiples for the GEMMs
    va = torch.zeros(bsz, nh, Lp, w, **f32)
    va[:, :, :L, :dv] = v
    va[..., dv] = 1.0
    Vc = va.view(bsz, nh, nch, c, w)

    # states entering each chunk X (for dg) and their e^rho row-scaled copy Xs (for the GEMMs)
    X = torch.matmul(Kr.transpose(-1, -2), Vc)
    Xs = torch.empty_like(X)
    _scan(X, eg, False, st, erho, Xs)
    causal = torch.ones(c, c, device=dev, dtype=torch.bool).tril_()
    S = torch.matmul(Qc, Kc.transpose(-1, -2)).masked_fill_(~causal, 0.0)
    numa = torch.matmul(Qc, Xs).add_(torch.matmul(S, Vc))
    dNa = _out_grads(numa, dh, Lp, w, True, st).view(bsz, nh, nch, c, w)
    del numa
    # adjoints leaving each chunk Y and their e^rho row-scaled copy Ys
    Y = torch.matmul(Qr.transpose(-1, -2), dNa)
    Ys = torch.empty_like(Y)
    _scan(Y, eg, True, st, erho, Ys)
    dS = torch.matmul(dNa, Vc.transpose(-1, -2)).masked_fill_(~causal, 0.0)
    dQs = torch.matmul(dS, Kc).add_(torch.matmul(dNa, Xs.transpose(-1, -2)))
    del Xs
    dKs = torch.matmul(dS.transpose(-1, -2), Qc).add_(torch.matmul(Vc, Ys.transpose(-1, -2)))
    dVa = torch.matmul(S.transpose(-1, -2), dNa).add_(torch.matmul(Kc, Ys))
    del Ys
    dv_out = dVa.view(bsz, nh, Lp, w)[:, :, :L, :dv]

    dg = _chunk_dg(Y, X, (-1,))
    dq, dk, dli, dlf, di = (torch.empty(bsz, nh, L, dqk, **f32) for _ in range(5))
    a.dq_scaled, a.dk_scaled, a.chunk_dg = ptr(dQs), ptr(dKs), ptr(dg)
    a.dq, a.dk, a.dlog_i, a.dlog_f, a.d_i = ptr(dq), ptr(dk), ptr(dli), ptr(dlf), ptr(di)
    _lib.call("hxm_mlstm_bwd_finalize", a, st)
    return dq, dk, dv_out, dli, dlf, di
