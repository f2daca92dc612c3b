"""sLSTM recurrence over the hxm C ABI.

Replaces the inline loop of sLSTMBlock.forward (hybrid_xmamba/layers/
slstm_block.py:91-127): gate activations (i = exp or sigmoid, f, o =
sigmoid, c~ = tanh), c = f*c + i*c~, h = o * tanh(RMSNorm_hd(c)), plus an
optional block-diagonal recurrent term R[head]^T h_{t-1} added to the gate
pre-activations (absent in the reference; R=None reproduces it).
"""
from __future__ import annotations

import torch

from .. import _lib
from ._common import dtype_code, f32_param, ptr, require_cuda, stream_of

__all__ = ["slstm_scan"]


def slstm_scan(gates_pre, norm_weight, *, R=None, eps=1e-6, exponential_gate=True, h0=None, c0=None,
               return_state=True, error_flag=None, wait_limit_cycles=0):
    """gates_pre (B, L, H, 4, hd) — gate_proj output viewed per head, blocks
    [i | f | o | c~]; norm_weight (hd,); R (H, hd, 4*hd) or None;
    h0, c0 (B, H, hd) fp32: the true hidden / cell state (the reference's
    cache['h'], cache['c']).  error_flag: a device int32 tensor set to 1 if a
    bounded cross-CTA wait gave up; wait_limit_cycles: that bound in SM
    cycles (0 = about 2 s).
    Returns h_seq (B, L, H, hd) in gates_pre's dtype [and (h, c) fp32]."""
    who = "slstm_scan"
    dev = require_cuda(gates_pre, norm_weight, R, h0, c0, who=who)
    if gates_pre.dim() != 5 or gates_pre.shape[3] != 4:
        raise ValueError(f"{who}: gates_pre must be (B, L, H, 4, hd); got {tuple(gates_pre.shape)}")
    bsz, L, nh, _, hd = gates_pre.shape
    io = gates_pre.dtype if gates_pre.dtype in (torch.float32, torch.bfloat16) else torch.float32
    g = gates_pre.to(io).contiguous()
    w = f32_param(norm_weight)
    if w.shape != (hd,):
        raise ValueError(f"{who}: norm_weight must be ({hd},)")
    Rb = None
    if R is not None:
        if R.shape != (nh, hd, 4 * hd):
            raise ValueError(f"{who}: R must be {(nh, hd, 4 * hd)}; got {tuple(R.shape)}")
        Rb = R.to(torch.bfloat16).contiguous()
    f32 = lambda t: None if t is None else t.float().contiguous()
    h0, c0 = f32(h0), f32(c0)
    out = torch.empty((bsz, L, nh, hd), device=dev, dtype=io)
    st = None
    if return_state:
        st = (torch.empty((bsz, nh, hd), device=dev, dtype=torch.float32),
              torch.empty((bsz, nh, hd), device=dev, dtype=torch.float32))
    a = _lib.SlstmArgs()
    a.batch, a.seqlen, a.heads, a.head_dim = bsz, L, nh, hd
    a.io_dtype = dtype_code(g)
    a.gates_pre, a.R, a.norm_weight = ptr(g), ptr(Rb), ptr(w)
    a.eps, a.exponential_gate = float(eps), int(bool(exponential_gate))
    a.h_out = ptr(out)
    a.h0, a.c0 = ptr(h0), ptr(c0)
    if st is not None:
        a.hT, a.cT = ptr(st[0]), ptr(st[1])
    a.error_flag, a.wait_limit_cycles = ptr(error_flag), int(wait_limit_cycles)
    _lib.call("hxm_slstm_scan_fwd", a, stream_of(dev))
    return (out, st) if return_state else out
