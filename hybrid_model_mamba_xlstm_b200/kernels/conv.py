"""Causal depthwise conv1d (+ bias, + SiLU) over the hxm C ABI.

Replaces the Mamba pre-scan convolution of the reference
(hybrid_xmamba/layers/mamba_block.py:101-104): ``rearrange`` to
(B, D, L), ``nn.Conv1d(D, D, width, groups=D, padding=width-1)``, trim to the
first L outputs, ``rearrange`` back and SiLU — here one pass over the
(B, L, D) activations, which may be a strided view (e.g. the x half of one
in_proj output).
"""
from __future__ import annotations

import torch

from .. import _lib
from ._common import dtype_code, f32_param, ptr, require_cuda, stream_of

__all__ = ["causal_conv1d"]

_ACT = {None: 0, "silu": 1, "swish": 1}


def causal_conv1d(x, weight, bias=None, activation=None, *, initial_state=None, return_final_state=False, out=None):
    """x (B, L, D) bf16 / fp32 (any batch / time strides, unit channel stride
    for the fast kernel); weight (D, width) or nn.Conv1d's (D, 1, width);
    bias (D,); initial_state (B, D, width-1): the inputs before t = 0.
    Returns out (B, L, D) in x's dtype [and the final state (B, D, width-1)]."""
    who = "causal_conv1d"
    dev = require_cuda(x, weight, bias, initial_state, out, who=who)
    if x.dim() != 3:
        raise ValueError(f"{who}: x must be (batch, seqlen, channels); got {tuple(x.shape)}")
    bsz, L, d = x.shape
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"{who}: x must be fp32 or bf16, got {x.dtype}")
    w = f32_param(weight).reshape(weight.shape[0], weight.shape[-1])
    if w.shape[0] != d:
        raise ValueError(f"{who}: weight must be ({d}, width); got {tuple(weight.shape)}")
    width = w.shape[1]
    if activation not in _ACT:
        raise ValueError(f"{who}: activation must be None or 'silu'")
    b = f32_param(bias)
    if b is not None and b.shape != (d,):
        raise ValueError(f"{who}: bias must be ({d},)")
    init = None
    if initial_state is not None:
        init = initial_state.to(x.dtype).contiguous()
        if init.shape != (bsz, d, width - 1):
            raise ValueError(f"{who}: initial_state must be {(bsz, d, width - 1)}")
    y = torch.empty((bsz, L, d), device=dev, dtype=x.dtype) if out is None else out
    fin = torch.empty((bsz, d, width - 1), device=dev, dtype=x.dtype) if return_final_state else None
    a = _lib.ConvArgs()
    a.batch, a.seqlen, a.channels, a.width = bsz, L, d, width
    a.io_dtype = dtype_code(x)
    a.x, a.x_stride = ptr(x), x.stride()
    a.weight, a.bias = ptr(w), ptr(b)
    a.out, a.out_stride = ptr(y), y.stride()
    a.init_state, a.final_state = ptr(init), ptr(fin)
    a.activation = _ACT[activation]
    _lib.call("hxm_causal_conv1d_fwd", a, stream_of(dev))
    return (y, fin) if return_final_state else y
