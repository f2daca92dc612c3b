"""Chunkwise mLSTM backward with the chunk contractions on the tensor cores.

The algebra is that of ``tfla_bwd`` (the chunkwise restatement of the
reference's recompute-under-autograd backward,
hybrid_xmamba/kernels/tfla/tfla_interface.py:52-81); this path runs every
chunk GEMM as hxm_chunk_gemm (tcgen05, bf16 operands, fp32 accumulation in
TMEM), fusing:
  * the causal mask and, for per-head gates, the decay exp(b_t - b_s) of the
    step matrices S = Q K^T and dS = dN V^T into the GEMM epilogue;
  * the sums of products (dQ = dS K + dN X^T, dK = dS^T Q + V Y^T,
    dV = S^T dN + K Y, num = Q X + S V) into one accumulator;
  * the transposed operands (K^T, Q^T, S^T, dS^T, X^T, Y^T), read MN-major by
    the MMA instead of transposed copies.

Precision: the backward is a difference of large terms (the normalizer's
dq = (C dh - n (dh . h)) / den, the gate identity q . dq - k . dk), so
operand rounding is amplified: plain bf16 operands (unit roundoff 2^-8) give
gradient errors of 1-7 % where the fp32 path gives 1e-6 and TF32 (2^-11)
1e-3.  Measured on B200, the error comes first from the gate-scaled q and k
(q e^(b - rho), i k e^(...)): rounding them alone gives 1-2 %.  So those are
split into a bf16 high part and the bf16 rounding of the remainder
(x = hi + lo to about 2^-16), and a product with a split operand is formed as
hi*hi + hi*lo + lo*hi (lo*lo is below the fp32 accumulation error): gradient
error ~1e-3 against float64, as with TF32 GEMMs.  With split_states (the
callers' precise=True) the states, adjoints and normalizer gradients are split
too: ~3e-5.  The producing kernels (hxm_mlstm_bwd_prepare, the chunk-state
scan, the normalizer, the GEMM epilogue) write the split operands directly.
bf16 inputs q, k, v are exact and never split.

Chunk length: 128 steps (one 128-row MMA tile per chunk); per-channel gates
whose 128-step chunk factors would leave e^+-MAX_EXP use 64 steps (rows 64..127
of each tile are zero-filled by TMA), and gates too strong for 64 take the
fp32 library path with a shorter chunk.
"""
from __future__ import annotations

from typing import NamedTuple

import torch

from ... import _lib
from .._common import dtype_code, ptr
from ..chunk_gemm import chunk_gemm

MAX_GROUPS = 1 << 24  # groups per hxm_chunk_gemm launch
MAX_PROD = 4        # products per launch
# Split the states, adjoints and normalizer gradients too (not only the gate-scaled q, k):
# gradient error ~3e-5 instead of ~1e-3 against float64 (TF32 GEMMs: ~1e-3), at up to 1.4x
# the time.  The callers' precise=False leaves them as bf16 high parts.
SPLIT_STATES = False

__all__ = ["bwd_channels_tc", "bwd_heads_tc", "TC_CHUNKS"]
TC_CHUNKS = (128, 64)


class Split(NamedTuple):
    """An fp32 operand as bf16 high and low parts (x ~ hi + lo to ~2^-16)."""
    hi: torch.Tensor
    lo: torch.Tensor

    def __getitem__(self, idx):  # slicing applies to both parts (tuple indexing stays positional)
        if isinstance(idx, int):
            return tuple.__getitem__(self, idx)
        return Split(self.hi[idx], self.lo[idx])


def split(x: torch.Tensor) -> Split:
    hi = x.to(torch.bfloat16)
    return Split(hi, (x - hi.float()).to(torch.bfloat16))


def scale_split(x, scale, padded_len, group, keep_lo=True):
    """hxm_scale_split: x (batch, steps, cols) (unit column stride) times scale
    (batch, padded_len, cols / group) fp32 (or None), zero past the steps, as a
    bf16 split operand (batch, padded_len, cols) (the high part alone without
    keep_lo) in one pass."""
    if x.stride(-1) != 1 or x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float().contiguous()
    bsz, L, cols = x.shape
    hi, lo = _bf16_pair((bsz, padded_len, cols), x.device, keep_lo)
    a = _lib.ScaleSplitArgs()
    a.batch, a.seqlen, a.padded_len, a.cols, a.group = bsz, L, padded_len, cols, group
    a.io_dtype = dtype_code(x)
    a.x, a.x_stride = ptr(x), x.stride()[:2]
    if scale is not None:
        scale = scale.float().contiguous()
        assert scale.numel() == bsz * padded_len * (cols // group)
    a.scale, a.hi, a.lo = ptr(scale), ptr(hi), ptr(lo)
    _lib.call("hxm_scale_split", a, torch.cuda.current_stream(x.device).cuda_stream)
    return _as_operand(hi, lo)


def _terms(A, ta, B, tb):
    """The bf16 products of op(A) op(B), A / B a bf16 tensor (exact) or a Split."""
    a_s, b_s = isinstance(A, Split), isinstance(B, Split)
    if a_s and b_s:
        return [(A.hi, ta, B.hi, tb), (A.hi, ta, B.lo, tb), (A.lo, ta, B.hi, tb)]
    if a_s:
        return [(A.hi, ta, B, tb), (A.lo, ta, B, tb)]
    if b_s:
        return [(A, ta, B.hi, tb), (A, ta, B.lo, tb)]
    return [(A, ta, B, tb)]


def _launch(products, *, out=None, out_bf16=None, out_bf16_lo=None, decay=None, **kw):
    """One hxm_chunk_gemm call over (G, rows, cols) operands, in slices of at most
    MAX_GROUPS groups."""
    G = products[0][0].shape[0]
    if G <= MAX_GROUPS:
        return chunk_gemm(products, out=out, out_bf16=out_bf16, out_bf16_lo=out_bf16_lo, decay=decay, **kw)
    for g0 in range(0, G, MAX_GROUPS):
        sl = slice(g0, min(G, g0 + MAX_GROUPS))
        cut = lambda t: None if t is None else t[sl]  # noqa: E731
        chunk_gemm([(A[sl], ta, B[sl], tb) for A, ta, B, tb in products], out=cut(out), out_bf16=cut(out_bf16),
                   out_bf16_lo=cut(out_bf16_lo), decay=cut(decay), **kw)


def mm(pairs, m, n, *, out=None, want_split=False, mask=False, decay=None, accumulate=False):
    """sum over pairs (A, trans_a, B, trans_b) of op(A) op(B), per group, with
    the split operands expanded into bf16 products; at most MAX_PROD products
    per launch, later launches accumulating.  Returns the fp32 result (out, or
    a new (G, m, n) tensor when needed) and, with want_split, its Split."""
    prods = [t for p in pairs for t in _terms(*p)]
    G = prods[0][0].shape[0]
    dev = prods[0][0].device
    # launches group products of equal K when that takes no more launches (each extra launch
    # re-reads and re-writes the fp32 output): the kernel then alternates their K slices, so
    # the operand two terms of a split product share is read from L2 the second time
    by_k = {}
    for pr in prods:
        by_k.setdefault(pr[0].shape[1] if pr[1] else pr[0].shape[2], []).append(pr)
    calls = [g[i:i + MAX_PROD] for g in by_k.values() for i in range(0, len(g), MAX_PROD)]
    if len(calls) > -(-len(prods) // MAX_PROD):
        calls = [prods[i:i + MAX_PROD] for i in range(0, len(prods), MAX_PROD)]
    if out is None and (not want_split or len(calls) > 1):
        out = torch.empty(G, m, n, device=dev, dtype=torch.float32)
    sp = None
    if want_split:
        sp = Split(torch.empty(G, m, n, device=dev, dtype=torch.bfloat16),
                   torch.empty(G, m, n, device=dev, dtype=torch.bfloat16))
    for i, call in enumerate(calls):
        last = i == len(calls) - 1
        _launch(call, out=out, out_bf16=sp.hi if (sp and last) else None, out_bf16_lo=sp.lo if (sp and last) else None,
                mask=mask, decay=decay, accumulate=accumulate or i > 0)
    return out, sp


def _values(v, L, Lp, w, G, c):
    """[v | 1 | 0 ...] per chunk row, bf16 (G, c, w): the normalizer n rides along
    as the column of ones (exact in bf16 for bf16 v)."""
    bsz, nh = v.shape[:2]
    dv = v.shape[-1]
    va = torch.zeros(bsz, nh, Lp, w, device=v.device, dtype=torch.bfloat16)
    va[:, :, :L, :dv] = v
    va[..., dv] = 1.0
    return va.view(G, c, w)


def _bf16_pair(shape, dev, lo=True):
    hi = torch.empty(*shape, device=dev, dtype=torch.bfloat16)
    return hi, (torch.empty_like(hi) if lo else None)


def _as_operand(hi, lo):
    """A Split, or the high part alone when the low part was not kept."""
    return Split(hi, lo) if lo is not None else hi


def _view(op, *shape):
    """The operand (Split or bf16 tensor) viewed as shape."""
    return Split(op.hi.view(*shape), op.lo.view(*shape)) if isinstance(op, Split) else op.view(*shape)


def _scan_split(x, decay, reverse, st, scale=None, split_lo=True, dot=None):
    """Row mode of hxm_chunk_state_scan over the increments x (groups, nch, rows,
    cols) fp32, read only: the exclusive (scaled) states as a bf16 split operand
    (the low part only when split_lo).  dot = (the state scan's Split, its scale or
    None): also the chunk gradients <x_out[k], state[k + 1]> (groups, nch, rows).
    Returns (operand, dg or None)."""
    hi, lo = _bf16_pair(x.shape, x.device, split_lo)
    a = _lib.ChunkScanArgs()
    a.groups, a.nchunks, a.rows, a.cols = x.shape[0] * x.shape[1], x.shape[2], x.shape[3], x.shape[4]
    a.x, a.decay, a.reverse = ptr(x), ptr(decay), int(reverse)
    a.scale, a.scaled_hi, a.scaled_lo, a.skip_state = ptr(scale), ptr(hi), ptr(lo), 1
    dg = None
    if dot is not None:
        dg = torch.empty(x.shape[:4], device=x.device, dtype=torch.float32)
        a.dot_hi, a.dot_lo, a.dot_scale, a.dot_out = ptr(dot[0].hi), ptr(dot[0].lo), ptr(dot[1]), ptr(dg)
    _lib.call("hxm_chunk_state_scan", a, st)
    return _as_operand(hi, lo), dg


def _normalizer(numa, dh, lp, w, st, want_fp32, split_lo=True):
    """hxm_mlstm_bwd_normalizer: [dnum | dden | 0 ...] rows as a bf16 split operand
    (and fp32 when asked); returns (fp32 or None, operand)."""
    bsz, nh, L, dv = dh.shape
    if dh.dtype not in (torch.float32, torch.bfloat16):
        dh = dh.float()
    if dh.stride(-1) != 1:
        dh = dh.contiguous()
    out = torch.empty(bsz, nh, lp, w, device=dh.device, dtype=torch.float32) if want_fp32 else None
    hi, lo = _bf16_pair((bsz, nh, lp, w), dh.device, split_lo)
    a = _lib.MlstmBwdNormArgs()
    a.batch, a.heads, a.seqlen, a.padded_len, a.dv, a.width = bsz, nh, L, lp, dv, w
    a.normalize, a.io_dtype = 1, dtype_code(dh)
    a.outputs, a.out, a.out_hi, a.out_lo = ptr(numa), ptr(out), ptr(hi), ptr(lo)
    a.dh, a.dh_stride = ptr(dh), dh.stride()[:3]
    _lib.call("hxm_mlstm_bwd_normalizer", a, st)
    return out, _as_operand(hi, lo)


def bwd_channels_tc(q, k, v, gi, gf, dh, c, st, split_states=None):
    """Per-channel gates (B, H, L, Dqk): the separable chunk scaling of
    hxm_mlstm_bwd_prepare with c-step chunks; prepare writes the gate-scaled q, k
    straight as split operands, the chunk-state scans and the normalizer write
    theirs (split_states=False keeps only their high parts as GEMM operands);
    the adjoint scan also forms the chunk gradients dg = <Y_k, X_{k+1}>."""
    split_states = SPLIT_STATES if split_states is None else split_states
    bsz, nh, L, dqk = q.shape
    dv = v.shape[-1]
    dev = q.device
    f32 = dict(device=dev, dtype=torch.float32)
    nch = (L + c - 1) // c
    Lp = nch * c
    G = bsz * nh * nch
    w = (dv + 1 + 7) // 8 * 8

    planes = torch.empty(8, bsz, nh, Lp, dqk, device=dev, dtype=torch.bfloat16)
    rho, erho, eg = (torch.empty(bsz, nh, nch, dqk, **f32) for _ in range(3))
    a = _lib.MlstmBwdArgs()
    a.batch, a.heads, a.seqlen, a.dqk, a.chunk, a.gate_mode = bsz, nh, L, dqk, c, 1
    a.io_dtype = dtype_code(q)
    a.q, a.q_stride = ptr(q), q.stride()[:3]
    a.k, a.k_stride = ptr(k), k.stride()[:3]
    a.log_i, a.i_stride = ptr(gi), gi.stride()[:3]
    a.log_f, a.f_stride = ptr(gf), gf.stride()[:3]
    a.rho, a.e_rho, a.e_g, a.split_planes = ptr(rho), ptr(erho), ptr(eg), ptr(planes)
    _lib.call("hxm_mlstm_bwd_prepare", a, st)
    # Qs, Ks and the decayed Qr = q e^b, Kr = i k e^(g-b) as split operands (G, c, dqk)
    Qc, Kc, Qr, Kr = (Split(planes[2 * u].view(G, c, dqk), planes[2 * u + 1].view(G, c, dqk)) for u in range(4))
    Vc = _values(v, L, Lp, w, G, c)

    # states entering each chunk X (fp32, for dg) and their e^rho row-scaled copy Xs
    X = torch.empty(bsz, nh, nch, dqk, w, **f32)
    mm([(Kr, 1, Vc, 0)], dqk, w, out=X.view(G, dqk, w))
    Xs5, _ = _scan_split(X, eg, False, st, erho)  # (the low part always: the chunk gradients read it)
    del X
    Xs = _view(Xs5, G, dqk, w) if split_states else Xs5.hi.view(G, dqk, w)
    _, S = mm([(Qc, 0, Kc, 1)], c, c, want_split=True, mask=True)
    numa = torch.empty(bsz, nh, nch, c, w, **f32)
    mm([(Qc, 0, Xs, 0), (S, 0, Vc, 0)], c, w, out=numa.view(G, c, w))
    dNa = _view(_normalizer(numa, dh, Lp, w, st, False, split_states)[1], G, c, w)
    del numa
    # adjoints leaving each chunk Y and their e^rho row-scaled copy Ys
    Y = torch.empty(bsz, nh, nch, dqk, w, **f32)
    mm([(Qr, 1, dNa, 0)], dqk, w, out=Y.view(G, dqk, w))
    Ys, dg = _scan_split(Y, eg, True, st, erho, split_states, dot=(Xs5, erho))
    del Y
    Ys = _view(Ys, G, dqk, w)
    _, dS = mm([(dNa, 0, Vc, 1)], c, c, want_split=True, mask=True)
    dQs = torch.empty(bsz, nh, Lp, dqk, **f32)
    mm([(dS, 0, Kc, 0), (dNa, 0, Xs, 1)], c, dqk, out=dQs.view(G, c, dqk))
    dKs = torch.empty(bsz, nh, Lp, dqk, **f32)
    mm([(dS, 1, Qc, 0), (Vc, 0, Ys, 1)], c, dqk, out=dKs.view(G, c, dqk))
    dVo = torch.empty(bsz, nh, Lp, dv, **f32)
    mm([(S, 1, dNa[:, :, :dv], 0), (Kc, 0, Ys[:, :, :dv], 0)], c, dv, out=dVo.view(G, c, dv))
    del S, dS, Xs, Ys, dNa, Qc, Kc, Qr, Kr

    dq, dk, dli, dlf, di = (torch.empty(bsz, nh, L, dqk, **f32) for _ in range(5))
    a.dq_scaled, a.dk_scaled, a.chunk_dg = ptr(dQs), ptr(dKs), ptr(dg)
    a.dq, a.dk, a.dlog_i, a.dlog_f, a.d_i = ptr(dq), ptr(dk), ptr(dli), ptr(dlf), ptr(di)
    _lib.call("hxm_mlstm_bwd_finalize", a, st)  # reads q_scaled / k_scaled from the split planes
    del planes
    return dq, dk, dVo[:, :, :L], dli, dlf, di


def bwd_heads_tc(q, k, v, li, lf, dout, per_channel_out, st, c=128, split_states=None):
    """Per-head gates (B, H, L): the exact decay-matrix form of tfla_bwd's
    _bwd_heads: S = causal(Q (i k)^T) * e^(b_t - b_s) and dS = dL/dS *
    e^(b_t - b_s) straight from the GEMM epilogue, the inter-chunk factors
    e^b and e^(g - b) (all at most 1) folded into the split operands."""
    split_states = SPLIT_STATES if split_states is None else split_states
    bsz, nh, L, dqk = q.shape
    dv = v.shape[-1]
    dev = q.device
    f32 = dict(device=dev, dtype=torch.float32)
    nch = (L + c - 1) // c
    Lp = nch * c
    G = bsz * nh * nch
    w = (dv + 1 + 7) // 8 * 8

    Q = torch.zeros(bsz, nh, Lp, dqk, **f32)
    Q[:, :, :L] = q
    K = torch.zeros(bsz, nh, Lp, dqk, **f32)
    K[:, :, :L] = k
    Q, K = Q.view(bsz, nh, nch, c, dqk), K.view(bsz, nh, nch, c, dqk)
    Vc = _values(v, L, Lp, w, G, c)
    lip = torch.full((bsz, nh, Lp), float("-inf"), **f32)
    lip[:, :, :L] = li
    lfp = torch.zeros(bsz, nh, Lp, **f32)
    lfp[:, :, :L] = lf
    b = lfp.view(bsz, nh, nch, c).cumsum(-1)
    g = b[..., -1:]
    ig = torch.exp(lip).view(bsz, nh, nch, c)
    Kp = K * ig.unsqueeze(-1)
    eb = torch.exp(b).unsqueeze(-1)
    egb = torch.exp(g - b).unsqueeze(-1)
    eg = torch.exp(g[..., 0]).unsqueeze(-1).expand(bsz, nh, nch, dqk).contiguous()
    Kd = Kp * egb
    g3 = lambda t, n: t.reshape(G, c, n)  # noqa: E731
    # bf16 operands straight from q, k (B*H, L, dqk): q itself (exact), i k, i k e^(g - b), q e^b
    q3, k3 = q.reshape(bsz * nh, L, dqk), k.reshape(bsz * nh, L, dqk)
    rowv = lambda t: t.reshape(bsz * nh, Lp, 1)  # noqa: E731
    Qb = _view(scale_split(q3, None, Lp, dqk, keep_lo=False), G, c, dqk)
    Kps, Kds, Qes = (_view(scale_split(x3, rowv(sc), Lp, dqk), G, c, dqk)
                     for x3, sc in ((k3, ig), (k3, ig * egb[..., 0]), (q3, eb[..., 0])))
    bdec = b.reshape(G, c)

    X = torch.empty(bsz, nh, nch, dqk, w, **f32)        # increments -> states entering each chunk
    mm([(Kds, 1, Vc, 0)], dqk, w, out=X.view(G, dqk, w))
    Xs5, _ = _scan_split(X, eg, False, st)  # (the low part always: the chunk gradients read it)
    del X
    Xs = _view(Xs5, G, dqk, w) if split_states else Xs5.hi.view(G, dqk, w)
    S, Ssp = mm([(Qb, 0, Kps, 1)], c, c, out=torch.empty(G, c, c, **f32), want_split=True, mask=True, decay=bdec)
    QX, _ = mm([(Qes, 0, Xs, 0)], c, w)
    numa = QX.clone()
    mm([(Ssp, 0, Vc, 0)], c, w, out=numa, accumulate=True)
    dNa, dNs = _normalizer(numa, dout, Lp, w, st, True, split_states)
    dNa, dNs = dNa.view(G, c, w), _view(dNs, G, c, w)
    del numa
    Y = torch.empty(bsz, nh, nch, dqk, w, **f32)        # increments -> adjoints leaving each chunk
    mm([(Qes, 1, dNs, 0)], dqk, w, out=Y.view(G, dqk, w))
    Ys, dg = _scan_split(Y, eg, True, st, None, split_states, dot=(Xs5, None))
    del Y
    Ys = _view(Ys, G, dqk, w)
    dSf, _ = mm([(dNs, 0, Vc, 1)], c, c, out=torch.empty(G, c, c, **f32), mask=True)  # dL/dS (causal part)
    _, dSs = mm([(dNs, 0, Vc, 1)], c, c, want_split=True, mask=True, decay=bdec)        # dL/d(Q (i k)^T)
    VY, _ = mm([(Vc, 0, Ys, 1)], c, dqk)
    dNes = split(dNa * g3(eb, 1)) if split_states else (dNa * g3(eb, 1)).to(torch.bfloat16)
    dQ = torch.empty(bsz, nh, nch, c, dqk, **f32)
    mm([(dSs, 0, Kps, 0), (dNes, 0, Xs, 1)], c, dqk, out=dQ.view(G, c, dqk))
    dKp = torch.empty(bsz, nh, nch, c, dqk, **f32)
    mm([(dSs, 1, Qb, 0)], c, dqk, out=dKp.view(G, c, dqk))
    VY = VY.view(bsz, nh, nch, c, dqk)
    dKp.add_(egb * VY)
    dVa = torch.empty(bsz, nh, Lp, dv, **f32)
    mm([(Ssp, 1, dNs[:, :, :dv], 0), (Kds, 0, Ys[:, :, :dv], 0)], c, dv, out=dVa.view(G, c, dv))
    del Ssp, dSs, dNes, dNs, Xs, Ys, Qb, Kps, Kds, Qes

    un = lambda t: t.reshape(bsz, nh, Lp, *t.shape[4:])[:, :, :L]  # noqa: E731
    dk = ig.unsqueeze(-1) * dKp
    di_c = K * dKp                                       # per channel: k . d(i k)
    if per_channel_out:  # the gate identity per channel, in-chunk part
        db = Q * dQ - Kp * dKp
    else:
        di_c = di_c.sum(-1)
        W = dSf.mul_(S).view(bsz, nh, nch, c, c)
        W.diagonal(dim1=-2, dim2=-1).zero_()  # in both sums: its net term is exactly zero
        dNa5, QX5 = dNa.view(bsz, nh, nch, c, w), QX.view(bsz, nh, nch, c, w)
        db = W.sum(-1) - W.sum(-2) + (dNa5 * QX5).sum(-1) - (Kd * VY).sum(-1)
        dg = dg.sum(-1)
    dlf = db.flip(3).cumsum(3).flip(3).add_(dg.unsqueeze(3))
    dlf = dlf.reshape(bsz, nh, Lp, *dlf.shape[4:])[:, :, :L]
    dlf[:, :, 0] = 0.0  # f at the first step multiplies the zero state
    di = di_c.reshape(bsz, nh, Lp, *di_c.shape[4:])[:, :, :L]
    igL = torch.exp(li.float())
    dli = di * (igL.unsqueeze(-1) if per_channel_out else igL)
    return un(dQ), un(dk), dVa[:, :, :L], dli, dlf, di
