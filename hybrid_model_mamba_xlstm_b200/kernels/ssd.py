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

__all__ = ["ssd_chunk_scan"]


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
