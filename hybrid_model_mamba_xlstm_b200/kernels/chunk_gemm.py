"""Batched chunk GEMMs on the tensor cores (hxm_chunk_gemm) for the chunkwise
backward passes: per group g, D = alpha * sum_p op(A_p) op(B_p) with bf16
operands and fp32 accumulation, then the causal mask / decay weighting of a
chunk's step matrix, accumulation and fp32 / bf16 stores in one epilogue.

These are the intra-chunk contractions of the chunkwise backward that
replaces the reference's recompute-under-autograd backward
(hybrid_xmamba/kernels/tfla/tfla_interface.py:52-81).
"""
from __future__ import annotations

import torch

from .. import _lib
from ._common import ptr, require_cuda, stream_of

__all__ = ["chunk_gemm"]


def _operand(o: _lib.GemmOperand, t: torch.Tensor, trans: bool, who: str):
    if t.dtype != torch.bfloat16 or t.dim() != 3 or t.stride(-1) != 1:
        raise ValueError(f"{who}: operands must be bf16 (groups, rows, cols) with unit column stride")
    o.ptr = t.data_ptr()
    o.group_stride, o.row_stride = t.stride(0), t.stride(1)
    o.rows, o.cols = t.shape[1], t.shape[2]
    o.trans = int(bool(trans))


def chunk_gemm(products, *, out=None, out_bf16=None, out_bf16_lo=None, alpha: float = 1.0, mask: bool = False,
               decay=None, accumulate: bool = False, error_flag=None, wait_limit_cycles: int = 0):
    """products: one to four (A, trans_a, B, trans_b), A / B bf16 (groups, rows, cols);
    op(A) is m x K, op(B) K x n.  out: fp32 (groups, m, n) and / or out_bf16: bf16
    (groups, m, n) (views with unit column stride).  mask: zero D[r, c] for c > r;
    decay: fp32 (groups, m) cumulative log gate b, D[r, c] *= exp(b_r - b_c) on the kept
    entries.  accumulate: out += D (every output then holds the sum).  out_bf16_lo: the
    bf16 low part D - bf16(D), laid out like out_bf16 (which it needs): high + low is a
    split operand of ~16 mantissa bits.  Returns (out, out_bf16)."""
    who = "chunk_gemm"
    if not 1 <= len(products) <= 4:
        raise ValueError(f"{who}: one to four products")
    ts = [t for pr in products for t in (pr[0], pr[2])]
    dev = require_cuda(*ts, out, out_bf16, out_bf16_lo, decay, error_flag, who=who)
    a = _lib.ChunkGemmArgs()
    a.groups = ts[0].shape[0]
    A0, ta0, B0, tb0 = products[0]
    a.m = A0.shape[2] if ta0 else A0.shape[1]
    a.n = B0.shape[1] if tb0 else B0.shape[2]
    a.nprod = len(products)
    for i, (A, ta, B, tb) in enumerate(products):
        if A.shape[0] != a.groups or B.shape[0] != a.groups:
            raise ValueError(f"{who}: operands with different group counts")
        _operand(a.a[i], A, ta, who)
        _operand(a.b[i], B, tb, who)
    if out_bf16_lo is not None and (out_bf16 is None or out_bf16_lo.stride() != out_bf16.stride()):
        raise ValueError(f"{who}: out_bf16_lo needs out_bf16 with the same strides")
    for t, dt in ((out, torch.float32), (out_bf16, torch.bfloat16), (out_bf16_lo, torch.bfloat16)):
        if t is not None and (t.dtype != dt or t.shape != (a.groups, a.m, a.n) or t.stride(-1) != 1):
            raise ValueError(f"{who}: outputs must be ({a.groups}, {a.m}, {a.n}) {dt} with unit column stride")
    if out is None and out_bf16 is None:
        out = torch.empty(a.groups, a.m, a.n, device=dev, dtype=torch.float32)
    a.alpha, a.mask, a.accumulate = float(alpha), int(bool(mask)), int(bool(accumulate))
    if decay is not None:
        if decay.dtype != torch.float32 or decay.shape != (a.groups, a.m) or decay.stride(-1) != 1:
            raise ValueError(f"{who}: decay must be fp32 (groups, m) with unit step stride")
        a.decay, a.decay_stride = decay.data_ptr(), decay.stride(0)
    if out is not None:
        a.out, a.out_group_stride, a.out_row_stride = out.data_ptr(), out.stride(0), out.stride(1)
    if out_bf16 is not None:
        a.out_bf16, a.outb_group_stride, a.outb_row_stride = out_bf16.data_ptr(), out_bf16.stride(0), out_bf16.stride(1)
    a.out_bf16_lo = ptr(out_bf16_lo)
    a.error_flag, a.wait_limit_cycles = ptr(error_flag), int(wait_limit_cycles)
    _lib.call("hxm_chunk_gemm", a, stream_of(dev))
    return out, out_bf16
