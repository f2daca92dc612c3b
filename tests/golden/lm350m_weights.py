"""Deterministic weights for the hybrid-350M parity check, chosen by parameter name.

The reference's ``HybridLanguageModel`` (hybrid_xmamba/models/hybrid_lm.py) and
this package's ``HybridLanguageModel`` use the same parameter names, so both
can be filled from this one function without ever storing the ~611 M weights:
every tensor is drawn from its own generator, seeded by the CRC-32 of its name,
so the values depend on the name and shape only (not on module order).

Rules (fp32 draws, then cast by the caller):
  *.A_log            log(1..N) per row (the S4D-real initialization, mamba_block.py)
  *.D                ones
  *.dt_proj.bias     softplus^-1(dt), dt log-uniform in [1e-3, 1e-1]
  1-D *norm*.weight  1 + 0.05 N(0, 1)
  other 1-D *.bias   0.02 N(0, 1)
  everything else    0.02 N(0, 1)
"""
from __future__ import annotations

import math
import zlib

import torch


def value(name: str, shape) -> torch.Tensor:
    g = torch.Generator().manual_seed(zlib.crc32(name.encode()) & 0x7FFFFFFF)
    shape = tuple(shape)
    if name.endswith("A_log"):
        return torch.log(torch.arange(1, shape[1] + 1, dtype=torch.float32)).repeat(shape[0], 1)
    if name.endswith(".D") and len(shape) == 1:
        return torch.ones(shape)
    if name.endswith("dt_proj.bias"):
        dt = torch.exp(torch.rand(shape, generator=g) * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3))
        return dt + torch.log(-torch.expm1(-dt))
    if len(shape) == 1 and "norm" in name and name.endswith("weight"):
        return 1.0 + 0.05 * torch.randn(shape, generator=g)
    return 0.02 * torch.randn(shape, generator=g)


def fill_(module: torch.nn.Module, skip=()) -> list:
    """Overwrite every parameter of `module` by `value(name)` (tied parameters
    once, under their first name); returns the names filled."""
    seen, names = set(), []
    with torch.no_grad():
        for name, p in module.named_parameters(remove_duplicate=False):
            if p.data_ptr() in seen or any(name.endswith(s) for s in skip):
                continue
            seen.add(p.data_ptr())
            p.copy_(value(name, p.shape).to(p.dtype))
            names.append(name)
    return names
