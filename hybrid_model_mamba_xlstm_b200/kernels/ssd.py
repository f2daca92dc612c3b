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


def ssd_chunk_scan(x, dt, A, B, C, D=None, *, dt_bias=None, dt_softplus=False, chunk=256, initial_state=None,
                   return_final_state=True):
    """x (B, L, H, P) bf16; dt (B, L, H) fp32; A (H,) fp32 (negative);
    B, C (B, L, N) bf16; D, dt_bias (H,) fp32; initial_state (B, H, P, N) fp32.
    Returns y (B, L, H, P) [and the final state (B, H, P, N) fp32]."""
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
    _lib.call("hxm_ssd_chunk_scan_fwd", a, stream_of(dev))
    return (y, hT) if return_final_state else y


def _dt_eff(dt, dt_bias, dt_softplus):
    z = dt.float() + (dt_bias.float() if dt_bias is not None else 0.0)
    return (torch.nn.functional.softplus(z) if dt_softplus else z), z


def ssd_chunk_scan_bwd(x, dt, A, B, C, D, dy, *, dt_bias=None, dt_softplus=False, chunk=64, tf32=None):
    """Gradients of y = ssd_chunk_scan(x, dt, A, B, C, D, dt_bias, dt_softplus)
    from a zero state, for dy (B, L, H, P).  Returns fp32
    (dx, ddt, dA, dB, dC, dD, ddt_bias) (dD / ddt_bias None when D / dt_bias are).

    Per head the SSD recurrence is the mLSTM state recurrence without its
    normalizer: q = C, k = B (shared by the heads), v = x[:, :, head], input
    gate i = dt and forget gate f = exp(dt A).  The chunkwise backward of the
    per-head mLSTM path (exact decay matrix, chunk-state scans on the GPU,
    batched fp32 chunk GEMMs) gives dq, dk, dv, dL/di and dL/dlog f; then
    ddt = dL/di + A dL/dlog f, dA = sum dt dL/dlog f, the shared B, C sum
    over heads, and softplus / bias chain on.  tf32: chunk GEMMs on TF32
    tensor cores (default when x is bf16, as from the bf16 forward) or in full
    fp32."""
    from .tfla.tfla_bwd import _bwd_heads, _gemm_precision
    who = "ssd_chunk_scan_bwd"
    dev = require_cuda(x, dt, A, B, C, D, dy, dt_bias, who=who)
    bsz, L, nh, p = x.shape
    n = B.shape[-1]
    de, z = _dt_eff(dt, dt_bias, dt_softplus)                      # (B, L, H)
    Af = A.float()
    with torch.no_grad(), _gemm_precision(x.dtype == torch.bfloat16 if tf32 is None else tf32):
        q = C.float().unsqueeze(1).expand(bsz, nh, L, n)
        k = B.float().unsqueeze(1).expand(bsz, nh, L, n)
        v = x.float().permute(0, 2, 1, 3)
        li = torch.log(de).permute(0, 2, 1)
        lf = (de * Af).permute(0, 2, 1)
        dyh = dy.float().permute(0, 2, 1, 3)
        dq, dk, dv, _, dlf, di = _bwd_heads(q, k, v, li, lf, dyh, int(chunk), False, False, stream_of(dev))
        dlf, di = dlf.permute(0, 2, 1), di.permute(0, 2, 1)        # (B, L, H)
        dde = di + Af * dlf
        dA = (de * dlf).sum((0, 1))
        dx = dv.permute(0, 2, 1, 3)
        dD = None
        if D is not None:
            dx = dx + D.float().view(1, 1, nh, 1) * dy.float()
            dD = (dy.float() * x.float()).sum((0, 1, 3))
        ddt = dde * torch.sigmoid(z) if dt_softplus else dde
        ddb = ddt.sum((0, 1)) if dt_bias is not None else None
    return dx, ddt, dA, dk.sum(1), dq.sum(1), dD, ddb


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


def ssd_chunk_scan_fn(x, dt, A, B, C, D=None, *, dt_bias=None, dt_softplus=False, chunk=256):
    """Differentiable y = ssd_chunk_scan(x, dt, A, B, C, D, ...) (zero initial state)."""
    return SSDChunkScanFunction.apply(x, dt, A, B, C, D, dt_bias, dt_softplus, chunk)
