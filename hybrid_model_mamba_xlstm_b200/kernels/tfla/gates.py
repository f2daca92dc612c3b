"""mLSTM gate prologue / epilogue over the hxm C ABI: the element-wise work of
mLSTMBlock.forward around the recurrence (hybrid_xmamba/layers/mlstm_block.py:
117-119,138-141), one HBM pass each."""
from __future__ import annotations

import torch

from ... import _lib
from .._common import dtype_code, ptr, require_cuda, stream_of

__all__ = ["mlstm_gate_prologue", "mlstm_gate_epilogue"]


def _rows(t, who):
    """(..., dim) with unit last stride whose leading dims flatten onto one row stride."""
    if t.stride(-1) != 1:
        raise ValueError(f"{who}: the last dim must be unit-stride")
    try:
        r = t.view(-1, t.shape[-1])
    except RuntimeError:
        raise ValueError(f"{who}: leading dims must flatten to rows without a copy") from None
    return r


def _args(dim, rows, io):
    a = _lib.MlstmGatesArgs()
    a.rows, a.dim, a.io_dtype = rows, dim, io
    return a


def mlstm_gate_prologue(i_pre, f_pre):
    """log_i = i_pre and log_f = logsigmoid(f_pre) as fp32 tensors of i_pre's
    shape: the log-space gates of mlstm_chunkwise_fwd (i = exp(i_pre))."""
    who = "mlstm_gate_prologue"
    dev = require_cuda(i_pre, f_pre, who=who)
    if f_pre.shape != i_pre.shape or f_pre.dtype != i_pre.dtype:
        raise ValueError(f"{who}: i_pre and f_pre must match")
    ir, fr = _rows(i_pre, who), _rows(f_pre, who)
    li = torch.empty(i_pre.shape, device=dev, dtype=torch.float32)
    lf = torch.empty(i_pre.shape, device=dev, dtype=torch.float32)
    a = _args(i_pre.shape[-1], ir.shape[0], dtype_code(i_pre))
    a.i_pre, a.i_row_stride = ptr(ir), ir.stride(0)
    a.f_pre, a.f_row_stride = ptr(fr), fr.stride(0)
    a.log_i, a.log_i_row_stride = ptr(li), li.shape[-1]
    a.log_f, a.log_f_row_stride = ptr(lf), lf.shape[-1]
    _lib.call("hxm_mlstm_gate_prologue", a, stream_of(dev))
    return li, lf


def mlstm_gate_epilogue(h, o_pre, x_gate):
    """h * sigmoid(o_pre) * sigmoid(x_gate), in h's dtype and shape."""
    who = "mlstm_gate_epilogue"
    dev = require_cuda(h, o_pre, x_gate, who=who)
    if o_pre.shape != h.shape or x_gate.shape != h.shape or len({h.dtype, o_pre.dtype, x_gate.dtype}) != 1:
        raise ValueError(f"{who}: h, o_pre and x_gate must match in shape and dtype")
    hr, orr, xr = _rows(h, who), _rows(o_pre, who), _rows(x_gate, who)
    out = torch.empty(h.shape, device=dev, dtype=h.dtype)
    a = _args(h.shape[-1], hr.shape[0], dtype_code(h))
    a.h, a.h_row_stride = ptr(hr), hr.stride(0)
    a.o_pre, a.o_row_stride = ptr(orr), orr.stride(0)
    a.x_gate, a.x_gate_row_stride = ptr(xr), xr.stride(0)
    a.out, a.out_row_stride = ptr(out), h.shape[-1]
    _lib.call("hxm_mlstm_gate_epilogue", a, stream_of(dev))
    return out
