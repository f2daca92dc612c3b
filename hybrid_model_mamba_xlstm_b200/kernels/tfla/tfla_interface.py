"""Chunkwise mLSTM ("TFLA") on B200: the reference's interface over the C ABI.

Mirrors hybrid_xmamba/kernels/tfla/tfla_interface.py:
  * ``apply_tfla(q, k, v, i_gate, f_gate)`` — same signature and semantics as
    the reference (:142-163): activated gates (i = exp(.), f = sigmoid(.)) of
    shape (B, H, L, D); the recurrence of ``tfla_forward_pytorch`` (:84-139)
    C = f*C + i*k v^T, n = f*n + i*k, h = q C / max(q.n, 1).  Gates that are
    per-head scalars broadcast over D (an ``expand``ed view, stride 0 on D)
    take the scalar-gate kernel without being materialised.
  * ``TFLAFunction`` — autograd Function with the reference's name (:18-81);
    its backward is the chunkwise one of ``tfla_bwd`` (the reference re-runs
    the step loop under autograd, :52-81).
  * ``mlstm_chunkwise_fwd(q, k, v, log_i, log_f, ...)`` — the extended entry:
    gates in log space (log_i = input-gate pre-activation, log_f =
    logsigmoid(forget pre-activation)), per head (B, H, L) or per channel
    (B, H, L, Dqk), optional initial state and the final stabilized state
    (C, n, m) with the true state equal to exp(m) * (C, n).
"""
from __future__ import annotations

import ctypes

import torch

from ... import _lib
from .._common import dtype_code, ptr, require_cuda, stream_of
from .tfla_bwd import mlstm_chunkwise_bwd

__all__ = ["apply_tfla", "mlstm_chunkwise_fwd", "mlstm_chunkwise_bwd", "TFLAFunction"]


def _unit_last(t):
    """(B, H, L, D) views pass as they are (any b / h / t strides) when D is unit-stride."""
    return t if t.stride(-1) == 1 or t.shape[-1] == 1 else t.contiguous()


def mlstm_chunkwise_fwd(q, k, v, log_i, log_f, C0=None, n0=None, m0=None, *, chunk=128, return_state=False,
                        out=None, error_flag=None, wait_limit_cycles=0):
    """h (B, H, L, Dv) [, (C, n, m)] of the mLSTM recurrence with log-space gates.

    chunk: the time chunk of the tensor-core kernels, 128 (or 0 for the same);
    the chunkwise result does not depend on it and other values raise.
    error_flag: a device int32 tensor set to 1 if a bounded device wait of
    the tensor-core kernels gave up (their outputs are then not written);
    wait_limit_cycles: that bound in SM cycles (0 = about 2 s).

    q, k: (B, H, L, Dqk); v: (B, H, L, Dv) — bf16 runs the tcgen05 chunkwise
    kernel, fp32 runs the exact fp32 recurrent kernel.  log_i, log_f: fp32
    (B, H, L) (per-head gates) or (B, H, L, Dqk) (per-channel gates).
    C0 (B, H, Dqk, Dv), n0 (B, H, Dqk), m0 (B, H): stabilized initial state.
    """
    who = "mlstm_chunkwise_fwd"
    dev = require_cuda(q, k, v, log_i, log_f, C0, n0, m0, who=who)
    if q.dim() != 4 or k.shape != q.shape or v.shape[:3] != q.shape[:3]:
        raise ValueError(f"{who}: q, k (B,H,L,Dqk) and v (B,H,L,Dv) expected; got "
                         f"{tuple(q.shape)} {tuple(k.shape)} {tuple(v.shape)}")
    bsz, nh, L, dqk = q.shape
    dv = v.shape[-1]
    if log_i.shape == (bsz, nh, L) and log_f.shape == (bsz, nh, L):
        gate_mode = 0
    elif log_i.shape == (bsz, nh, L, dqk) and log_f.shape == (bsz, nh, L, dqk):
        gate_mode = 1
    else:
        raise ValueError(f"{who}: gates must be (B,H,L) or (B,H,L,Dqk); got {tuple(log_i.shape)} {tuple(log_f.shape)}")
    io = q.dtype if q.dtype in (torch.float32, torch.bfloat16) else torch.float32
    q, k, v = (_unit_last(t if t.dtype == io else t.to(io)) for t in (q, k, v))
    gi, gf = log_i.float(), log_f.float()
    if gate_mode == 1:  # per-channel gates: unit channel stride; (b, h, t) strides free
        gi, gf = _unit_last(gi), _unit_last(gf)
    h = torch.empty((bsz, nh, L, dv), device=dev, dtype=io) if out is None else out
    if h.shape != (bsz, nh, L, dv) or h.dtype != io or h.stride(-1) != 1:
        raise ValueError(f"{who}: out must be a ({bsz}, {nh}, {L}, {dv}) {io} view with unit last stride")
    st = None
    if return_state:
        st = (torch.empty((bsz, nh, dqk, dv), device=dev, dtype=torch.float32),
              torch.empty((bsz, nh, dqk), device=dev, dtype=torch.float32),
              torch.empty((bsz, nh), device=dev, dtype=torch.float32))
    c32 = lambda t: None if t is None else t.float().contiguous()
    C0, n0, m0 = c32(C0), c32(n0), c32(m0)
    a = _lib.MlstmArgs()
    a.batch, a.heads, a.seqlen, a.dqk, a.dv = bsz, nh, L, dqk, dv
    a.chunk, a.gate_mode, a.io_dtype = chunk, gate_mode, dtype_code(q)
    a.q, a.q_stride = ptr(q), q.stride()[:2]
    a.k, a.k_stride = ptr(k), k.stride()[:2]
    a.v, a.v_stride = ptr(v), v.stride()[:2]
    a.log_i, a.i_stride = ptr(gi), gi.stride()[:2]
    a.log_f, a.f_stride = ptr(gf), gf.stride()[:2]
    a.h, a.h_stride = ptr(h), h.stride()[:2]
    a.q_tstride, a.k_tstride, a.v_tstride, a.h_tstride = q.stride(2), k.stride(2), v.stride(2), h.stride(2)
    a.i_tstride, a.f_tstride = gi.stride(2), gf.stride(2)
    a.C0, a.n0, a.m0 = ptr(C0), ptr(n0), ptr(m0)
    if st is not None:
        a.CT, a.nT, a.mT = ptr(st[0]), ptr(st[1]), ptr(st[2])
    a.struct_size = ctypes.sizeof(a)
    ws_bytes = _lib.lib().hxm_mlstm_workspace_size(a)
    ws = torch.empty(max(int(ws_bytes), 1), device=dev, dtype=torch.uint8) if ws_bytes else None
    a.workspace, a.workspace_bytes = ptr(ws), int(ws_bytes)
    a.error_flag, a.wait_limit_cycles = ptr(error_flag), int(wait_limit_cycles)
    _lib.call("hxm_mlstm_chunkwise_fwd", a, stream_of(dev))
    return (h, st) if return_state else h


def _gate_logs(i_gate, f_gate):
    """log-space gates; per-head when the gates are broadcast views over D."""
    if i_gate.dim() == 4 and i_gate.stride(-1) == 0 and f_gate.stride(-1) == 0:
        return torch.log(i_gate[..., 0].float()), torch.log(f_gate[..., 0].float())
    return torch.log(i_gate.float()), torch.log(f_gate.float())


class TFLAFunction(torch.autograd.Function):
    """Autograd wrapper with the reference's name (tfla_interface.py:18-81).

    The reference's backward re-runs the step loop under autograd (:52-81);
    this one is the chunkwise backward of ``tfla_bwd.mlstm_chunkwise_bwd``
    (same gradients, fp32 arithmetic).  Gates given as expanded per-head
    views get their per-channel gradients; autograd sums them over D."""

    @staticmethod
    def forward(ctx, q, k, v, i_gate, f_gate):
        ctx.save_for_backward(q, k, v, i_gate, f_gate)
        log_i, log_f = _gate_logs(i_gate, f_gate)
        return mlstm_chunkwise_fwd(q, k, v, log_i, log_f)

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, i_gate, f_gate = ctx.saved_tensors
        log_i, log_f = _gate_logs(i_gate, f_gate)
        dq, dk, dv, _, dlog_f, di = mlstm_chunkwise_bwd(q, k, v, log_i, log_f, grad_output, chunk=64,
                                                        gate_grads="channel")
        df = dlog_f / f_gate.float()
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), di.to(i_gate.dtype), df.to(f_gate.dtype)


def apply_tfla(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, i_gate: torch.Tensor,
               f_gate: torch.Tensor) -> torch.Tensor:
    """Drop-in for hybrid_xmamba.kernels.tfla.apply_tfla (tfla_interface.py:142-163).

    q, k, v, i_gate, f_gate: (B, H, L, D); i_gate > 0 and f_gate > 0 (as
    mLSTMBlock produces them: exp and sigmoid)."""
    return TFLAFunction.apply(q, k, v, i_gate, f_gate)
