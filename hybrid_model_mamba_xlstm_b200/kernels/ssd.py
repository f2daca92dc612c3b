"""Mamba-2 SSD chunked scan (ngroups = 1) over the hxm C ABI.

The reference has no SSD kernel; its arithmetic is the reference's Euler
selective scan (hybrid_xmamba/kernels/selective_scan/scan_interface.py:
103-152) with channel d = (head, p), per-head A and dt, and B, C shared by
all heads:  h[p,n] = exp(dt*A) h[p,n] + dt*x[p]*B[n];  y[p] = C.h[p,:] + D*x[p].
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib
from ._common import dtype_code, ptr, require_cuda, stream_of

__all__ = ["ssd_chunk_scan", "ssd_chunk_scan_bwd", "SSDChunkScanFunction", "ssd_chunk_scan_fn"]


def ssd_chunk_scan(x, dt, A, B, C, D=None, *, dt_bias=None, dt_softplus=False, chunk=128, initial_state=None,
                   return_final_state=True, error_flag=None, wait_limit_cycles=0):
    """x (B, L, H, P) bf16; dt (B, L, H) fp32; A (H,) fp32 (negative);
    B, C (B, L, N) bf16; D, dt_bias (H,) fp32; initial_state (B, H, P, N) fp32.
    Returns y (B, L, H, P) [and the final state (B, H, P, N) fp32].
    chunk: the kernel's time chunk, 128 (or 0 for the same); the chunkwise
    result does not depend on it and other values raise.  error_flag: a
    device int32 tensor set to 1 if a bounded device wait gave up (the
    outputs are then not written); wait_limit_cycles: that bound in SM
    cycles (0 = about 2 s)."""
    who = "ssd_chunk_scan"
    dev = require_cuda(x, dt, A, B, C, D, dt_bias, initial_state, who=who)
    if x.dim() != 4:
        raise ValueError(f"{who}: x must be (B, L, H, P)")
    bsz, L, nh, p = x.shape
    n = B.shape[-1]
    if dt.shape != (bsz, L, nh) or A.shape != (nh,) or B.shape != (bsz, L, n) or C.shape != (bsz, L, n):
        raise ValueError(f"{who}: shape mismatch x{tuple(x.shape)} dt{tuple(dt.shape)} A{tuple(A.shape)} "
                         f"B{tuple(B.shape)} C{tuple(C.shape)}")
    io = torch.bfloat16
    xc, Bc, Cc = (t.to(io).contiguous() for t in (x, B, C))
    dtc = dt.float().contiguous()
    f32 = lambda t: None if t is None else t.float().contiguous()
    A, D, dt_bias, h0 = f32(A), f32(D), f32(dt_bias), f32(initial_state)
    y = torch.empty((bsz, L, nh, p), device=dev, dtype=io)
    hT = torch.empty((bsz, nh, p, n), device=dev, dtype=torch.float32) if return_final_state else None
    a = _lib.SsdArgs()
    a.batch, a.seqlen, a.heads, a.headdim, a.dstate, a.chunk = bsz, L, nh, p, n, chunk
    a.io_dtype = dtype_code(xc)
    a.x, a.dt, a.A, a.B, a.C = ptr(xc), ptr(dtc), ptr(A), ptr(Bc), ptr(Cc)
    a.D, a.dt_bias, a.dt_softplus = ptr(D), ptr(dt_bias), int(bool(dt_softplus))
    a.y, a.h0, a.hT = ptr(y), ptr(h0), ptr(hT)
    a.struct_size = ctypes.sizeof(a)
    ws_bytes = int(_lib.lib().hxm_ssd_workspace_size(a))
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8) if ws_bytes else None
    a.workspace, a.workspace_bytes = ptr(ws), ws_bytes
    a.error_flag, a.wait_limit_cycles = ptr(error_flag), int(wait_limit_cycles)
    _lib.call("hxm_ssd_chunk_scan_fwd", a, stream_of(dev))
    return (y, hT) if return_final_state else y


def _dt_eff(dt, dt_bias, dt_softplus):
    z = dt.float() + (dt_bias.float() if dt_bias is not None else 0.0)
    return (torch.nn.functional.softplus(z) if dt_softplus else z), z


def _intra(cb, bcum, dt, G, st):
    """hxm_ssd_bwd_intra: (S_h, M, dL/d dt, dL/d b) of the per-head c x c terms."""
    bsz, nch, c, nh = bcum.shape
    S = torch.empty_like(G)
    M = torch.empty_like(cb)
    ddt, db = (torch.empty(bsz, nch, nh, c, device=G.device, dtype=torch.float32) for _ in range(2))
    a = _lib.SsdBwdIntraArgs()
    a.batch, a.nchunks, a.heads, a.chunk = bsz, nch, nh, c
    a.cb, a.bcum, a.dt, a.dS = ptr(cb), ptr(bcum), ptr(dt), ptr(G)
    a.S, a.M, a.ddt, a.db = ptr(S), ptr(M), ptr(ddt), ptr(db)
    _lib.call("hxm_ssd_bwd_intra", a, st)
    return S, M, ddt, db


def _rows(xh, dyh, dxi, BY, CZ, alpha, D, L, st):
    """hxm_ssd_bwd_rows: dx (B, L, H, P) and the per-row x.BY, dy.CZ, dy.x."""
    bsz, nch, nh, c, p = xh.shape
    dx = torch.empty(bsz, L, nh, p, device=xh.device, dtype=torch.float32)
    xby, dycz, dyx = (torch.empty(bsz, nch, c, nh, device=xh.device, dtype=torch.float32) for _ in range(3))
    a = _lib.SsdBwdRowsArgs()
    a.batch, a.nchunks, a.chunk, a.heads, a.headdim, a.seqlen = bsz, nch, c, nh, p, L
    a.xh, a.dyh, a.dxi, a.BY, a.CZ, a.alpha, a.D = ptr(xh), ptr(dyh), ptr(dxi), ptr(BY), ptr(CZ), ptr(alpha), ptr(D)
    a.dx, a.xby, a.dycz, a.dyx = ptr(dx), ptr(xby), ptr(dycz), ptr(dyx)
    _lib.call("hxm_ssd_bwd_rows", a, st)
    return dx, xby, dycz, dyx


def _ssd_bwd_shared(x, de, Af, Bm, Cm, dy, c, st, D=None):
    """Chunkwise SSD backward with B, C shared by the heads (ngroups = 1).

    Per head h and chunk (b = in-chunk prefix sum of log f = dt A, g its total,
    beta = e^b, alpha = dt e^(g - b)):
        state entering chunk k, rows (h, p), columns n:
            Z_{k+1} = e^g Z_k + (alpha x)^T B          (one GEMM over all heads)
        adjoint leaving chunk k:
            Y_k = e^g Y_{k+1} + (beta dy)^T C
        intra-chunk weights S_h = (C B^T) * e^(b_t - b_s) * dt_s (causal)
    so the state-side GEMMs fold the heads into their inner dimension
    ((c x N) x (N x H*P) per chunk) and only the c x c decay matrices are per
    head (hxm_ssd_bwd_intra forms them with the head sum on chip; x and dy are
    laid out head-major once so the per-head GEMMs read them in place).
    hxm_ssd_bwd_rows assembles dx (+ D dy) and the per-row dot products of the
    dt / log-decay / D gradients.  Returns (dx (B, L, H, P), dL/d dt through
    the input gate and dL/dlog f (B, L, H), dB, dC (B, L, N), dD or None); the
    gate identity is formed as in the per-head mLSTM path (rowsum - colsum of
    W = dL/dS * S without its diagonal, the two inter-chunk terms, and
    <Y_k, Z_{k+1}> per chunk)."""
    from .tfla.tfla_bwd import _chunk_dg, _scan
    if c not in (32, 64):
        raise ValueError(f"ssd_chunk_scan_bwd: chunk must be 32 or 64 (got {c})")
    bsz, L, nh, p = x.shape
    n = Bm.shape[-1]
    f32 = dict(device=x.device, dtype=torch.float32)
    nch = (L + c - 1) // c
    Lp = nch * c
    nf = L // c

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

    xh = pad_heads(x)
    dyh = pad_heads(dy)
    Bc = pad(Bm, n).view(bsz, nch, c, n)
    Cc = pad(Cm, n).view(bsz, nch, c, n)
    dec = pad(de, nh).view(bsz, nch, c, nh)               # 0 past the sequence: no input there
    b = (dec * Af).cumsum(2)                              # (B, nch, c, H)
    g = b[:, :, -1:]
    beta = torch.exp(b)
    egb = torch.exp(g - b)
    alpha = dec * egb
    eg_rows = torch.exp(g[:, :, 0]).unsqueeze(-1).expand(bsz, nch, nh, p).reshape(bsz, nch, nh * p).contiguous()
    ax = torch.empty(bsz, nch, c, nh, p, **f32)
    torch.mul(xh.permute(0, 1, 3, 2, 4), alpha.unsqueeze(-1), out=ax)
    ax = ax.view(bsz, nch, c, nh * p)
    bdy = torch.empty(bsz, nch, c, nh, p, **f32)
    torch.mul(dyh.permute(0, 1, 3, 2, 4), beta.unsqueeze(-1), out=bdy)
    bdy = bdy.view(bsz, nch, c, nh * p)
    Z = torch.matmul(ax.transpose(-1, -2), Bc)            # increments -> states entering each chunk
    _scan(Z.unsqueeze(1), eg_rows, False, st)
    Yz = torch.matmul(bdy.transpose(-1, -2), Cc)          # increments -> adjoints leaving each chunk
    _scan(Yz.unsqueeze(1), eg_rows, True, st)

    # per-head c x c terms (hxm_ssd_bwd_intra: one block per (batch, chunk), the head sum on chip)
    G = torch.matmul(dyh, xh.transpose(-1, -2))           # dL/dS_h = dy_h x_h^T
    cb = torch.matmul(Cc, Bc.transpose(-1, -2))           # C B^T (B, nch, c, c)
    S, M, di, db = _intra(cb, b, dec, G, st)
    del G
    dxi = torch.matmul(S.transpose(-1, -2), dyh)          # intra-chunk dx, head-major
    del S
    # shared-operand GEMMs (heads folded into the inner dimension)
    dC = torch.matmul(M, Bc).add_(torch.matmul(bdy, Z))
    dB = torch.matmul(M.transpose(-1, -2), Cc).add_(torch.matmul(ax, Yz))
    BY = torch.matmul(Bc, Yz.transpose(-1, -2))           # (B, nch, c, H*P)
    CZ = torch.matmul(Cc, Z.transpose(-1, -2))
    Df = None if D is None else D.float().contiguous()
    dx, xby, dycz, dyx = _rows(xh, dyh, dxi, BY, CZ, alpha, Df, L, st)
    di = di.permute(0, 1, 3, 2).add_(egb * xby)
    db = db.permute(0, 1, 3, 2).add_(beta * dycz).sub_(alpha * xby)
    dg = _chunk_dg(Yz.unsqueeze(1), Z.unsqueeze(1), (-1,)).view(bsz, nch, nh, p).sum(-1)
    dlf = db.flip(2).cumsum(2).flip(2).add_(dg.unsqueeze(2)).reshape(bsz, Lp, nh)[:, :L]
    dlf[:, 0] = 0.0  # f at the first step multiplies the zero state
    un = lambda t: t.reshape(bsz, Lp, *t.shape[3:])[:, :L]
    dD = None if D is None else dyx.sum((0, 1, 2))
    return dx, un(di), dlf, un(dB), un(dC), dD


def ssd_chunk_scan_bwd(x, dt, A, B, C, D, dy, *, dt_bias=None, dt_softplus=False, chunk=64, tf32=None,
                       tensor_cores=None, precise=True):
    """Gradients of y = ssd_chunk_scan(x, dt, A, B, C, D, dt_bias, dt_softplus)
    from a zero state, for dy (B, L, H, P).  Returns fp32
    (dx, ddt, dA, dB, dC, dD, ddt_bias) (dD / ddt_bias None when D / dt_bias are).

    Per head the SSD recurrence is the mLSTM state recurrence without its
    normalizer: q = C, k = B (shared by the heads), v = x[:, :, head], input
    gate i = dt and forget gate f = exp(dt A).  The chunkwise backward
    (_ssd_bwd_shared: exact decay matrix, chunk-state scans on the GPU,
    batched chunk GEMMs with the heads folded in where B, C are shared) gives
    dx, dB, dC, dL/di and dL/dlog f; then ddt = dL/di + A dL/dlog f,
    dA = sum dt dL/dlog f, and softplus / bias chain on.  tensor_cores (default
    for bf16 x, as from the bf16 forward): the chunk GEMMs run as hxm_chunk_gemm
    (tcgen05; ssd_bwd_tc), with bf16 high / low split operands (precise, ~1e-5
    against float64) or high parts only (precise=False, ~1e-3); otherwise cuBLAS
    (torch.matmul), on TF32 tensor cores when tf32 (default: bf16 x) or in full
    fp32."""
    from .tfla.tfla_bwd import _gemm_precision
    who = "ssd_chunk_scan_bwd"
    dev = require_cuda(x, dt, A, B, C, D, dy, dt_bias, who=who)
    bsz, L, nh, p = x.shape
    n = B.shape[-1]
    de, z = _dt_eff(dt, dt_bias, dt_softplus)                      # (B, L, H)
    Af = A.float()
    use_tc = (x.dtype == torch.bfloat16) if tensor_cores is None else bool(tensor_cores)
    if use_tc and (p % 8 or n % 8 or n > 640):
        if tensor_cores:
            raise ValueError(f"{who}: tensor_cores needs headdim and dstate multiples of 8, dstate <= 640")
        use_tc = False
    with torch.no_grad(), _gemm_precision(x.dtype == torch.bfloat16 if tf32 is None else tf32):
        if use_tc:
            from .ssd_bwd_tc import ssd_bwd_shared_tc
            if int(chunk) not in (32, 64):
                raise ValueError(f"ssd_chunk_scan_bwd: chunk must be 32 or 64 (got {chunk})")
            dx, di, dlf, dBm, dCm, dD = ssd_bwd_shared_tc(x, de, Af, B, C, dy, int(chunk), stream_of(dev), D,
                                                          precise=precise)
        else:
            dx, di, dlf, dBm, dCm, dD = _ssd_bwd_shared(x, de, Af, B, C, dy, int(chunk), stream_of(dev), D)
        dde = di + Af * dlf
        dA = (de * dlf).sum((0, 1))
        ddt = dde * torch.sigmoid(z) if dt_softplus else dde
        ddb = ddt.sum((0, 1)) if dt_bias is not None else None
    return dx, ddt, dA, dBm, dCm, dD, ddb


class SSDChunkScanFunction(torch.autograd.Function):
    """y = ssd_chunk_scan(...) with the chunkwise backward of ssd_chunk_scan_bwd."""

    @staticmethod
    def forward(ctx, x, dt, A, B, C, D, dt_bias, dt_softplus, chunk):
        ctx.save_for_backward(x, dt, A, B, C, D, dt_bias)
        ctx.dt_softplus = dt_softplus
        return ssd_chunk_scan(x, dt, A, B, C, D, dt_bias=dt_bias, dt_softplus=dt_softplus, chunk=chunk,
                              return_final_state=False)

    @staticmethod
    def backward(ctx, dy):
        x, dt, A, B, C, D, dt_bias = ctx.saved_tensors
        dx, ddt, dA, dB, dC, dD, ddb = ssd_chunk_scan_bwd(x, dt, A, B, C, D, dy, dt_bias=dt_bias,
                                                          dt_softplus=ctx.dt_softplus)
        cast = lambda g, t: None if g is None or t is None else g.to(t.dtype)
        return (cast(dx, x), cast(ddt, dt), cast(dA, A), cast(dB, B), cast(dC, C), cast(dD, D), cast(ddb, dt_bias),
                None, None)


def ssd_chunk_scan_fn(x, dt, A, B, C, D=None, *, dt_bias=None, dt_softplus=False, chunk=128):
    """Differentiable y = ssd_chunk_scan(x, dt, A, B, C, D, ...) (zero initial state)."""
    return SSDChunkScanFunction.apply(x, dt, A, B, C, D, dt_bias, dt_softplus, chunk)
