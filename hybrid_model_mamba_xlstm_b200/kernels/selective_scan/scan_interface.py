"""Selective scan on B200: the reference's interface over the hxm C ABI.

Mirrors hybrid_xmamba/kernels/selective_scan/scan_interface.py:
  * ``selective_scan(x, dt, A, B, C, D, z=None)`` — same signature, layout
    (batch, seqlen, dim) and semantics as the reference (:155-180): Euler
    discretisation as in ``selective_scan_pytorch`` (:103-152) and a plain
    ``y * z`` gate (:57-58).
  * ``SelectiveScanFunction`` — autograd Function with the reference's name
    (:17-100).  Forward and backward are CUDA kernels (the reference's backward
    recomputes its loop under autograd, :62-100; the gradients are the same).
  * ``selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None,
    delta_softplus=False, return_last_state=False, discretization="euler",
    initial_state=None)`` — the fused entry in (batch, dim, seqlen) layout
    with ``y * silu(z)``, softplus(delta + bias) and the final state.

Inputs of any strides are accepted; the kernel stages whichever of the time
or channel axes is unit-stride with 16-byte async copies.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from ... import _lib
from .._common import dtype_code, ptr, require_cuda, stream_of

__all__ = ["selective_scan", "selective_scan_fn", "SelectiveScanFunction", "SelectiveScanFnFunction",
           "selective_scan_raw", "selective_scan_bwd"]

_ZMODE = {None: 0, "mul": 1, "silu": 2}
_DISC = {"euler": 0, "zoh": 1}


def _prepare(u, delta, A, B, C, D, z, z_mode, delta_bias, delta_softplus, discretization, h0, who):
    """Checks, dtype casts and the hxm_scan_args of a request in (batch, seqlen, dim)
    LOGICAL layout.  Returns (args, tensors kept alive, device, io dtype)."""
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
    if h0 is not None:
        h0 = h0.float().contiguous()
        if h0.shape != (bt, dm, n):
            raise ValueError(f"{who}: initial state must be {(bt, dm, n)}")
    a = _lib.ScanArgs()
    a.struct_size = ctypes.sizeof(a)
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
    a.h0 = ptr(h0)
    a.z_mode = _ZMODE[z_mode if z is not None else None]
    a.delta_softplus = int(bool(delta_softplus))
    a.discretization = _DISC[discretization]
    return a, (u, delta, A, B, C, D, z, delta_bias, h0), dev, io


def selective_scan_raw(u, delta, A, B, C, D=None, z=None, *, z_mode=None, delta_bias=None, delta_softplus=False,
                       discretization="euler", h0=None, return_last_state=False, out=None):
    """Launch hxm_selective_scan_fwd on tensors in (batch, seqlen, dim) LOGICAL layout.

    u, delta, z: (Bt, L, Dm); A: (Dm, N) fp32; B, C: (Bt, L, N); D, delta_bias: (Dm,) fp32;
    h0: (Bt, Dm, N) fp32.  Returns y (Bt, L, Dm) in u's dtype, and the final state if asked.
    Strides are passed through as they are (views need no copy).
    """
    a, keep, dev, io = _prepare(u, delta, A, B, C, D, z, z_mode, delta_bias, delta_softplus, discretization, h0,
                                "selective_scan")
    bt, L, dm = u.shape
    y = torch.empty((bt, L, dm), device=dev, dtype=io) if out is None else out
    hT = torch.empty((bt, dm, A.shape[1]), device=dev, dtype=torch.float32) if return_last_state else None
    a.y, a.y_stride = ptr(y), y.stride()
    a.hT = ptr(hT)
    # scratch for the time segments the library runs when the grid would not fill the GPU
    ws_bytes = int(_lib.lib().hxm_selective_scan_workspace_size(a))
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8) if ws_bytes else None
    a.workspace, a.workspace_bytes = ptr(ws), ws_bytes
    _lib.call("hxm_selective_scan_fwd", a, stream_of(dev))
    return (y, hT) if return_last_state else y


def selective_scan_bwd(dout, u, delta, A, B, C, D=None, z=None, *, z_mode=None, delta_bias=None,
                       delta_softplus=False, h0=None):
    """Gradients of ``selective_scan_raw``'s y (Euler) with respect to every input,
    from hxm_selective_scan_bwd; fp32 tensors in the inputs' logical shapes:
    dict(u, delta, A, B, C, D, z, delta_bias, h0) (entries of absent inputs are None)."""
    a, keep, dev, io = _prepare(u, delta, A, B, C, D, z, z_mode, delta_bias, delta_softplus, "euler", h0,
                                "selective_scan_bwd")
    bt, L, dm = u.shape
    n = A.shape[1]
    g = dout if dout.dtype == io else dout.to(io)
    f32 = dict(device=dev, dtype=torch.float32)
    out = {"u": torch.empty(bt, L, dm, **f32), "delta": torch.empty(bt, L, dm, **f32),
           "A": torch.empty(dm, n, **f32), "B": torch.empty(bt, L, n, **f32), "C": torch.empty(bt, L, n, **f32),
           "D": torch.empty(dm, **f32) if D is not None else None,
           "z": torch.empty(bt, L, dm, **f32) if z is not None else None,
           "delta_bias": torch.empty(dm, **f32) if delta_bias is not None else None,
           "h0": torch.empty(bt, dm, n, **f32) if h0 is not None else None}
    b = _lib.ScanBwdArgs()
    b.fwd = a
    b.struct_size = ctypes.sizeof(b)
    b.dout, b.dout_stride = ptr(g), g.stride()
    b.du, b.ddelta, b.dz = ptr(out["u"]), ptr(out["delta"]), ptr(out["z"])
    b.dA, b.dB, b.dC, b.dD = ptr(out["A"]), ptr(out["B"]), ptr(out["C"]), ptr(out["D"])
    b.ddelta_bias, b.dh0 = ptr(out["delta_bias"]), ptr(out["h0"])
    ws_bytes = int(_lib.lib().hxm_selective_scan_bwd_workspace_size(b))
    ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
    b.workspace, b.workspace_bytes = ptr(ws), ws_bytes
    _lib.call("hxm_selective_scan_bwd", b, stream_of(dev))
    return out


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
        g = selective_scan_bwd(grad_output, x, dt, A, B, C, D, z, z_mode="mul" if z is not None else None)
        cast = lambda t, o: None if t is None else t.to(o.dtype)
        return (cast(g["u"], x), cast(g["delta"], dt), cast(g["A"], A), cast(g["B"], B), cast(g["C"], C),
                cast(g["D"], D), cast(g["z"], z) if z is not None else None)


class SelectiveScanFnFunction(torch.autograd.Function):
    """Autograd of ``selective_scan_fn`` ((batch, dim, seqlen) layout, softplus(delta + bias),
    y * silu(z), optional initial state h0): forward and backward both on the hxm kernels
    (the backward kernel also returns dL/dh0)."""

    @staticmethod
    def forward(ctx, u, delta, A, B, C, D, z, delta_bias, delta_softplus, h0):
        t = lambda a: None if a is None else a.transpose(1, 2)
        ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, h0)
        ctx.delta_softplus = delta_softplus
        y = torch.empty(u.shape, device=u.device,
                        dtype=u.dtype if u.dtype in (torch.float32, torch.bfloat16) else torch.float32)
        selective_scan_raw(t(u), t(delta), A, t(B), t(C), D, t(z), z_mode="silu" if z is not None else None,
                           delta_bias=delta_bias, delta_softplus=delta_softplus, h0=h0, out=y.transpose(1, 2))
        return y

    @staticmethod
    def backward(ctx, grad_output):
        u, delta, A, B, C, D, z, delta_bias, h0 = ctx.saved_tensors
        t = lambda a: None if a is None else a.transpose(1, 2)
        g = selective_scan_bwd(t(grad_output), t(u), t(delta), A, t(B), t(C), D, t(z),
                               z_mode="silu" if z is not None else None, delta_bias=delta_bias,
                               delta_softplus=ctx.delta_softplus, h0=h0)
        cast = lambda x, o: None if (x is None or o is None) else x.to(o.dtype)
        return (cast(t(g["u"]), u), cast(t(g["delta"]), delta), cast(g["A"], A), cast(t(g["B"]), B),
                cast(t(g["C"]), C), cast(g["D"], D), cast(t(g["z"]), z), cast(g["delta_bias"], delta_bias), None,
                cast(g["h0"], h0))


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
    Differentiable (Euler) through y, into every input and initial_state; the
    final state is not differentiable, so asking for it (or for the ZOH rule)
    while gradients are needed raises instead of silently dropping them.
    """
    needs_grad = torch.is_grad_enabled() and any(
        x is not None and x.requires_grad for x in (u, delta, A, B, C, D, z, delta_bias, initial_state))
    if needs_grad:
        if discretization != "euler":
            raise NotImplementedError("selective_scan_fn: the backward covers the Euler rule only")
        if return_last_state:
            raise NotImplementedError("selective_scan_fn: the final state is not differentiable; call with "
                                      "return_last_state=False under autograd (or under torch.no_grad())")
        return SelectiveScanFnFunction.apply(u, delta, A, B, C, D, z, delta_bias, delta_softplus, initial_state)
    t = lambda a: None if a is None else a.transpose(1, 2)
    y_bld = torch.empty((u.shape[0], u.shape[1], u.shape[2]), device=u.device,
                        dtype=u.dtype if u.dtype in (torch.float32, torch.bfloat16) else torch.float32)
    res = selective_scan_raw(t(u), t(delta), A, t(B), t(C), D, t(z), z_mode="silu" if z is not None else None,
                             delta_bias=delta_bias, delta_softplus=delta_softplus, discretization=discretization,
                             h0=initial_state, return_last_state=return_last_state, out=y_bld.transpose(1, 2))
    if return_last_state:
        return y_bld, res[1]
    return y_bld
