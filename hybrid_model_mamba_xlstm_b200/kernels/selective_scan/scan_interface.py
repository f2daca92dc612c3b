"""Selective scan on B200: the reference's interface over the hxm C ABI.

Mirrors hybrid_xmamba/kernels/selective_scan/scan_interface.py:
  * ``selective_scan(x, dt, A, B, C, D, z=None)`` — same signature, layout
    (batch, seqlen, dim) and semantics as the reference (:155-180): Euler
    discretisation as in ``selective_scan_pytorch`` (:103-152) and a plain
    ``y * z`` gate (:57-58).
  * ``SelectiveScanFunction`` — autograd Function with the reference's name
    (:17-100).  Forward is the CUDA kernel; backward recomputes the forward
    under autograd with torch ops, as the reference's backward does (:62-100).
  * ``selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None,
    delta_softplus=False, return_last_state=False, discretization="euler",
    initial_state=None)`` — the fused entry in (batch, dim, seqlen) layout
    with ``y * silu(z)``, softplus(delta + bias) and the final state.

Inputs of any strides are accepted; the kernel stages whichever of the time
or channel axes is unit-stride with 16-byte async copies.
"""
from __future__ import annotations

from typing import Optional

import torch

from ... import _lib
from .._common import dtype_code, ptr, require_cuda, stream_of

__all__ = ["selective_scan", "selective_scan_fn", "SelectiveScanFunction", "selective_scan_raw"]

_ZMODE = {None: 0, "mul": 1, "silu": 2}
_DISC = {"euler": 0, "zoh": 1}


def selective_scan_raw(u, delta, A, B, C, D=None, z=None, *, z_mode=None, delta_bias=None, delta_softplus=False,
                       discretization="euler", h0=None, return_last_state=False, out=None):
    """Launch hxm_selective_scan_fwd on tensors in (batch, seqlen, dim) LOGICAL layout.

    u, delta, z: (Bt, L, Dm); A: (Dm, N) fp32; B, C: (Bt, L, N); D, delta_bias: (Dm,) fp32;
    h0: (Bt, Dm, N) fp32.  Returns y (Bt, L, Dm) in u's dtype, and the final state if asked.
    Strides are passed through as they are (views need no copy).
    """
    who = "selective_scan"
    dev = require_cuda(u, delta, A, B, C, D, z, delta_bias, h0, who=who)
    if u.dim() != 3 or delta.shape != u.shape:
        raise ValueError(f"{who}: u and delta must be (batch, seqlen, dim); got {tuple(u.shape)}, {tuple(delta.shape)}")
    bt, L, dm = u.shape
    if A.dim() != 2 or A.shape[0] != dm:
        raise ValueError(f"{who}: A must be (dim, dstate); got {tuple(A.shape)}")
    n = A.shape[1]
    for name, t in (("B", B), ("C", C)):
        if t.shape != (bt, L, n):
            raise ValueError(f"{who}: {name} must be {(bt, L, n)}; got {tuple(t.shape)}")
    io = u.dtype if u.dtype in (torch.float32, torch.bfloat16) else torch.float32
    cast = lambda t: None if t is None else (t if t.dtype == io else t.to(io))
    u, delta, B, C, z = cast(u), cast(delta), cast(B), cast(C), cast(z)
    f32 = lambda t: None if t is None else t.float()
    A, D, delta_bias = f32(A), f32(D), f32(delta_bias)
    if z is not None and z.shape != u.shape:
        raise ValueError(f"{who}: z must be {tuple(u.shape)}; got {tuple(z.shape)}")
    if D is not None:
        D = D.contiguous()
        if D.shape != (dm,):
            raise ValueError(f"{who}: D must be ({dm},)")
    if delta_bias is not None:
        delta_bias = delta_bias.contiguous()
    y = torch.empty((bt, L, dm), device=dev, dtype=io) if out is None else out
    hT = torch.empty((bt, dm, n), device=dev, dtype=torch.float32) if return_last_state else None
    if h0 is not None:
        h0 = h0.float().contiguous()
        if h0.shape != (bt, dm, n):
            raise ValueError(f"{who}: initial state must be {(bt, dm, n)}")
    a = _lib.ScanArgs()
    a.batch, a.seqlen, a.dim, a.dstate = bt, L, dm, n
    a.io_dtype = dtype_code(u)
    a.u, a.u_stride = ptr(u), u.stride()
    a.delta, a.delta_stride = ptr(delta), delta.stride()
    a.A, a.A_stride = ptr(A), A.stride()
    a.B, a.B_stride = ptr(B), B.stride()
    a.C, a.C_stride = ptr(C), C.stride()
    a.D = ptr(D)
    if z is not None:
        a.z, a.z_stride = ptr(z), z.stride()
    a.delta_bias = ptr(delta_bias)
    a.y, a.y_stride = ptr(y), y.stride()
    a.h0, a.hT = ptr(h0), ptr(hT)
    a.z_mode = _ZMODE[z_mode if z is not None else None]
    a.delta_softplus = int(bool(delta_softplus))
    a.discretization = _DISC[discretization]
    _lib.call("hxm_selective_scan_fwd", a, stream_of(dev))
    return (y, hT) if return_last_state else y


def _scan_torch(x, dt, A, B, C, D):
    """Differentiable torch restatement of the forward, used only by backward
    (the reference's backward recomputes its loop the same way, :62-100)."""
    bsz, L, dm = x.shape
    h = torch.zeros(bsz, dm, A.shape[1], device=x.device, dtype=torch.float32)
    ys = []
    for t in range(L):
        dt_t = dt[:, t].float()
        h = torch.exp(A[None] * dt_t[..., None]) * h + (dt_t * x[:, t].float())[..., None] * B[:, t, None].float()
        ys.append((h * C[:, t, None].float()).sum(-1) + D[None].float() * x[:, t].float())
    return torch.stack(ys, 1)


class SelectiveScanFunction(torch.autograd.Function):
    """Autograd wrapper with the reference's name and argument order
    (scan_interface.py:17-100).  Forward runs hxm_selective_scan_fwd."""

    @staticmethod
    def forward(ctx, x, dt, A, B, C, D, z=None):
        ctx.save_for_backward(x, dt, A, B, C, D, z)
        return selective_scan_raw(x, dt, A, B, C, D, z, z_mode="mul" if z is not None else None)

    @staticmethod
    def backward(ctx, grad_output):
        x, dt, A, B, C, D, z = ctx.saved_tensors
        with torch.enable_grad():
            ins = [t.detach().requires_grad_(True) for t in (x, dt, A, B, C, D)]
            y = _scan_torch(*ins)
            zc = None
            if z is not None:
                zc = z.detach().requires_grad_(True)
                y = y * zc.float()
            y.backward(grad_output.float())
        grads = [t.grad.to(o.dtype) if t.grad is not None else None for t, o in zip(ins, (x, dt, A, B, C, D))]
        return (*grads, (zc.grad.to(z.dtype) if zc is not None else None))


def selective_scan(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor, C: torch.Tensor,
                   D: torch.Tensor, z: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Drop-in for hybrid_xmamba.kernels.selective_scan.selective_scan
    (scan_interface.py:155-180): x, dt (B, L, D); A (D, N); B, C (B, L, N);
    D (D,); optional z (B, L, D) multiplies the output."""
    return SelectiveScanFunction.apply(x, dt, A, B, C, D, z)


def selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                      return_last_state=False, discretization="euler", initial_state=None):
    """Fused selective scan in (batch, dim, seqlen) layout.

    u, delta, z: (B, D, L); B, C: (B, N, L); A: (D, N); D, delta_bias: (D,).
    Computes softplus(delta + delta_bias) (if requested), the scan, + D*u and
    y * silu(z).  Returns y (B, D, L) [and the final state (B, D, N) fp32].
    """
    t = lambda a: None if a is None else a.transpose(1, 2)
    y_bld = torch.empty((u.shape[0], u.shape[1], u.shape[2]), device=u.device,
                        dtype=u.dtype if u.dtype in (torch.float32, torch.bfloat16) else torch.float32)
    res = selective_scan_raw(t(u), t(delta), A, t(B), t(C), D, t(z), z_mode="silu" if z is not None else None,
                             delta_bias=delta_bias, delta_softplus=delta_softplus, discretization=discretization,
                             h0=initial_state, return_last_state=return_last_state, out=y_bld.transpose(1, 2))
    if return_last_state:
        return y_bld, res[1]
    return y_bld
