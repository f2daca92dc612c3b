"""RMSNorm, optionally fused with the residual add before it, over the hxm C ABI.

Replaces RMSNorm.forward (hybrid_xmamba/layers/normalization.py:32-34) and
the residual add + following pre-norm of HybridBlock.forward
(hybrid_xmamba/layers/hybrid_block.py:122-130) with one HBM pass.
"""
from __future__ import annotations

import torch

from .. import _lib
from ._common import dtype_code, f32_param, ptr, require_cuda, stream_of

__all__ = ["rmsnorm"]


def _rows(t, who):
    if t.stride(-1) != 1:
        raise ValueError(f"{who}: the last dim must be contiguous")
    lead = t.shape[:-1]
    # row stride: all leading dims must collapse onto one stride
    r = t.reshape(-1, t.shape[-1]) if t.is_contiguous() else None
    if r is None:
        try:
            r = t.view(-1, t.shape[-1])
        except RuntimeError:
            raise ValueError(f"{who}: leading dims must flatten to rows without a copy") from None
    return r, lead


def rmsnorm(x, weight=None, eps=1e-6, *, residual=None, return_sum=False, out=None):
    """out = weight * s / sqrt(mean(s^2, -1) + eps) with s = x (+ residual,
    rounded to x's dtype).  Returns out [and s when ``return_sum``]."""
    who = "rmsnorm"
    dev = require_cuda(x, weight, residual, out, who=who)
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"{who}: x must be fp32 or bf16, got {x.dtype}")
    if residual is not None and (residual.shape != x.shape or residual.dtype != x.dtype):
        raise ValueError(f"{who}: residual must match x")
    if return_sum and residual is None:
        raise ValueError(f"{who}: return_sum needs a residual")
    dim = x.shape[-1]
    w = f32_param(weight)
    if w is not None and w.shape != (dim,):
        raise ValueError(f"{who}: weight must be ({dim},)")
    xr, lead = _rows(x, who)
    rr = None if residual is None else _rows(residual, who)[0]
    y = torch.empty_like(x, memory_format=torch.contiguous_format) if out is None else out
    yr = _rows(y, who)[0]
    s = torch.empty_like(y) if return_sum else None
    sr = None if s is None else _rows(s, who)[0]
    a = _lib.RmsnormArgs()
    a.rows, a.dim, a.io_dtype = xr.shape[0], dim, dtype_code(x)
    a.x, a.x_row_stride = ptr(xr), xr.stride(0)
    if rr is not None:
        a.residual, a.residual_row_stride = ptr(rr), rr.stride(0)
    if sr is not None:
        a.sum_out, a.sum_row_stride = ptr(sr), sr.stride(0)
    a.weight, a.eps = ptr(w), float(eps)
    a.out, a.out_row_stride = ptr(yr), yr.stride(0)
    _lib.call("hxm_rmsnorm_fwd", a, stream_of(dev))
    return (y, s) if return_sum else y
