"""Chunkwise SSD backward with the chunk contractions on the tensor cores.

Same algebra as ssd._ssd_bwd_shared (the chunkwise backward of the SSD
recurrence, whose arithmetic is the reference's Euler selective scan,
hybrid_xmamba/kernels/selective_scan/scan_interface.py:103-152, with channel
d = (head, p) and B, C shared by the heads); every chunk GEMM runs as
hxm_chunk_gemm (tcgen05, bf16 operands, fp32 accumulation):
  * bf16 inputs x, B, C (and dy when it is bf16) are exact operands;
  * the gate-weighted alpha x, beta dy, the chunk states Z and adjoints Y, and
    the intra-chunk S_h, M are bf16 high / low split operands (precise, the
    default: gradient error ~1e-5 against float64) or high parts only
    (precise=False: ~1e-3, as TF32 GEMMs);
  * the state scans run in the row mode of hxm_chunk_state_scan (split output,
    chunk gradients <Y_k, Z_{k+1}> fused into the adjoint scan);
  * the per-head c x c terms stay with hxm_ssd_bwd_intra, the row assembly
    with hxm_ssd_bwd_rows.
"""
from __future__ import annotations

import torch

from .tfla.tfla_bwd_tc import _scan_split, _view, mm, scale_split, split


def _op(t: torch.Tensor, exact: bool, precise: bool):
    """A GEMM operand: the bf16 tensor when exact, else a Split (or its high part)."""
    if exact:
        return t.to(torch.bfloat16)
    return split(t) if precise else t.to(torch.bfloat16)


def ssd_bwd_shared_tc(x, de, Af, Bm, Cm, dy, c, st, D=None, precise=True):
    """As ssd._ssd_bwd_shared (same arguments and returns), tensor-core GEMMs."""
    from .ssd import _intra, _rows
    bsz, L, nh, p = x.shape
    n = Bm.shape[-1]
    dev = x.device
    f32 = dict(device=dev, dtype=torch.float32)
    nch = (L + c - 1) // c
    Lp = nch * c
    nf = L // c
    hp = nh * p
    G2, G3 = bsz * nch, bsz * nch * nh

    def pad(t, *tail):
        out = torch.zeros(bsz, Lp, *tail, **f32)
        out[:, :L] = t
        return out

    def pad_heads(t):  # (B, L, H, P) -> head-major chunks (B, nch, H, c, P), zero past L
        out = torch.zeros(bsz, nch, nh, c, p, **f32)
        if nf:
            out[:, :nf].copy_(t[:, :nf * c].reshape(bsz, nf, c, nh, p).permute(0, 1, 3, 2, 4))
        if L > nf * c:
            out[:, nf, :, :L - nf * c].copy_(t[:, nf * c:].permute(0, 2, 1, 3))
        return out

    bf = torch.bfloat16
    xh = pad_heads(x)
    dyh = pad_heads(dy)
    dec = pad(de, nh).view(bsz, nch, c, nh)               # 0 past the sequence: no input there
    b = (dec * Af).cumsum(2)                              # (B, nch, c, H)
    g = b[:, :, -1:]
    beta = torch.exp(b)
    egb = torch.exp(g - b)
    alpha = dec * egb
    eg_rows = torch.exp(g[:, :, 0]).unsqueeze(-1).expand(bsz, nch, nh, p).reshape(bsz, nch, hp).contiguous()
    # alpha x and beta dy in the (step, head * p) layout of x, dy, B and C padded: split operands in one pass each
    axs = _view(scale_split(x.reshape(bsz, L, hp), alpha.view(bsz, Lp, nh), Lp, p, precise), G2, c, hp)
    bdys = _view(scale_split(dy.reshape(bsz, L, hp), beta.view(bsz, Lp, nh), Lp, p, precise), G2, c, hp)
    Bb = _view(scale_split(Bm, None, Lp, n, Bm.dtype != bf and precise), G2, c, n)
    Cb = _view(scale_split(Cm, None, Lp, n, Cm.dtype != bf and precise), G2, c, n)
    xb = _op(xh.view(G3, c, p), x.dtype == bf, precise)
    dyb = _op(dyh.view(G3, c, p), dy.dtype == bf, precise)

    # states entering each chunk (rows (h, p), columns n) and adjoints leaving each chunk
    Z = torch.empty(bsz, 1, nch, hp, n, **f32)
    mm([(axs, 1, Bb, 0)], hp, n, out=Z.view(G2, hp, n))
    Z5, _ = _scan_split(Z, eg_rows, False, st)            # (the low part always: the chunk gradients read it)
    del Z
    Zs = _view(Z5, G2, hp, n) if precise else Z5.hi.view(G2, hp, n)
    Y = torch.empty(bsz, 1, nch, hp, n, **f32)
    mm([(bdys, 1, Cb, 0)], hp, n, out=Y.view(G2, hp, n))
    Ys, dg = _scan_split(Y, eg_rows, True, st, None, precise, dot=(Z5, None))
    del Y
    Ys = _view(Ys, G2, hp, n)

    # per-head c x c terms (hxm_ssd_bwd_intra: one block per (batch, chunk), the head sum on chip)
    Gm = torch.empty(bsz, nch, nh, c, c, **f32)
    mm([(dyb, 0, xb, 1)], c, c, out=Gm.view(G3, c, c))   # dL/dS_h = dy_h x_h^T
    cb = torch.empty(bsz, nch, c, c, **f32)
    mm([(Cb, 0, Bb, 1)], c, c, out=cb.view(G2, c, c))    # C B^T
    S, M, di, db = _intra(cb, b, dec, Gm, st)
    del Gm
    Ss = _op(S.view(G3, c, c), False, precise)
    Ms = _op(M.view(G2, c, c), False, precise)
    del S, M
    dxi = torch.empty(bsz, nch, nh, c, p, **f32)
    mm([(Ss, 1, dyb, 0)], c, p, out=dxi.view(G3, c, p))  # intra-chunk dx, head-major
    # shared-operand GEMMs (heads folded into the inner dimension)
    dC = torch.empty(bsz, nch, c, n, **f32)
    mm([(Ms, 0, Bb, 0), (bdys, 0, Zs, 0)], c, n, out=dC.view(G2, c, n))
    dB = torch.empty(bsz, nch, c, n, **f32)
    mm([(Ms, 1, Cb, 0), (axs, 0, Ys, 0)], c, n, out=dB.view(G2, c, n))
    BY = torch.empty(bsz, nch, c, hp, **f32)
    mm([(Bb, 0, Ys, 1)], c, hp, out=BY.view(G2, c, hp))
    CZ = torch.empty(bsz, nch, c, hp, **f32)
    mm([(Cb, 0, Zs, 1)], c, hp, out=CZ.view(G2, c, hp))
    del Ss, Ms, Zs, Ys, Z5, axs, bdys
    Df = None if D is None else D.float().contiguous()
    dx, xby, dycz, dyx = _rows(xh, dyh, dxi, BY, CZ, alpha, Df, L, st)
    di = di.permute(0, 1, 3, 2).add_(egb * xby)
    db = db.permute(0, 1, 3, 2).add_(beta * dycz).sub_(alpha * xby)
    dg = dg.view(bsz, nch, nh, p).sum(-1)
    dlf = db.flip(2).cumsum(2).flip(2).add_(dg.unsqueeze(2)).reshape(bsz, Lp, nh)[:, :L]
    dlf[:, 0] = 0.0  # f at the first step multiplies the zero state
    un = lambda t: t.reshape(bsz, Lp, *t.shape[3:])[:, :L]  # noqa: E731
    dD = None if D is None else dyx.sum((0, 1, 2))
    return dx, un(di), dlf, un(dB), un(dC), dD
