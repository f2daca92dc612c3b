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
