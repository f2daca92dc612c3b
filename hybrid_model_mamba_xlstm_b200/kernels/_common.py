"""Torch-side plumbing shared by the op wrappers: dtype codes, stream, checks."""
from __future__ import annotations

import torch

from .. import _lib

_DTYPE = {torch.float32: _lib.HXM_F32, torch.bfloat16: _lib.HXM_BF16, torch.float16: _lib.HXM_F16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def require_cuda(*tensors, who: str):
    """The kernels run only on a CUDA device; there is no CPU fallback."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{who}: tensors must be on a CUDA device (got {t.device}); "
                               "this package has no CPU path")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{who}: tensors on different devices ({dev} vs {t.device})")
    return dev


def stream_of(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t):
    return None if t is None else t.data_ptr()


def strides(t, n):
    return (0,) * n if t is None else tuple(t.stride())


def f32_param(t):
    """``t`` as a contiguous fp32 tensor, for small parameters (weights, biases) that the
    kernels read in fp32.  A bf16 parameter's fp32 copy is kept on the tensor and reused while
    the tensor is unchanged (same storage and version), so inference calls launch no cast
    kernel; with autograd recording for ``t`` the cast is a fresh differentiable op, and a copy
    first made during a CUDA-graph capture is not kept."""
    if t is None:
        return None
    if t.dtype == torch.float32 and t.is_contiguous():
        return t
    if torch.is_grad_enabled() and t.requires_grad:
        return t.float().contiguous()
    key = (t.data_ptr(), t._version, tuple(t.shape), t.stride())
    hit = getattr(t, "_hxm_f32", None)
    if hit is not None and hit[0] == key:
        return hit[1]
    v = t.detach().float().contiguous()
    if t.is_cuda and torch.cuda.is_current_stream_capturing():
        return v  # a copy made inside a graph capture only holds data once the graph runs
    try:
        t._hxm_f32 = (key, v)
    except (AttributeError, RuntimeError):
        pass
    return v
