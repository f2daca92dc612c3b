"""Seeded synthetic inputs with the value distributions of the benchmark workloads.

Every generator draws on the host with ``torch.Generator().manual_seed(seed)``
in fp32 (so a workload is identical on every machine), then casts and moves.
Large inputs can be generated directly on the device (``on_device=True``)
with a CUDA generator — same distributions, different bits — which is what
the benchmark does for multi-GB inputs.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


def _gen(seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def softplus_inv(x):
    return x + torch.log(-torch.expm1(-x))


@dataclass
class ScanInputs:
    """Selective-scan inputs in (batch, dim, seqlen) layout (the kernel's
    fast layout): u, delta_raw, z (B, D, L); B, C (B, N, L); A (D, N);
    D, delta_bias (D,).  delta = softplus(delta_raw + delta_bias)."""
    u: torch.Tensor
    delta: torch.Tensor
    z: torch.Tensor
    A: torch.Tensor
    B: torch.Tensor
    C: torch.Tensor
    D: torch.Tensor
    delta_bias: torch.Tensor

    def bytes_moved(self) -> int:
        """Algorithmic HBM bytes of one fused scan pass (inputs read once,
        y written once, final state written once)."""
        bt, dm, L = self.u.shape
        n = self.A.shape[1]
        es = self.u.element_size()
        return (bt * L * dm * 4 * es          # u, delta, z, y
                + 2 * bt * L * n * es         # B, C
                + (dm * n + 2 * dm) * 4       # A, D, delta_bias
                + bt * dm * n * 4)            # final state


def scan_inputs(batch, seqlen, dim, dstate=16, dtype=torch.float32, seed=0, device="cpu", on_device=False):
    """u, z ~ N(0,1); delta_raw ~ N(0, 0.5^2); delta_bias = softplus^-1(dt),
    dt log-uniform in [1e-3, 1e-1] per channel; A = -(1..N) per channel
    (S4D-real); B, C ~ N(0,1); D = 1."""
    gdev = device if on_device else "cpu"
    g = _gen(seed, gdev)
    f = dict(generator=g, device=gdev, dtype=torch.float32)
    u = torch.randn(batch, dim, seqlen, **f)
    z = torch.randn(batch, dim, seqlen, **f)
    raw = torch.randn(batch, dim, seqlen, **f).mul_(0.5)
    dt0 = torch.exp(torch.rand(dim, **f) * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3))
    bias = softplus_inv(dt0)
    A = -torch.arange(1, dstate + 1, dtype=torch.float32, device=gdev).repeat(dim, 1)
    B = torch.randn(batch, dstate, seqlen, **f)
    C = torch.randn(batch, dstate, seqlen, **f)
    D = torch.ones(dim, device=gdev)
    cast = lambda t: t.to(device=device, dtype=dtype)
    return ScanInputs(cast(u), cast(raw), cast(z), A.to(device), cast(B), cast(C), D.to(device), bias.to(device))


@dataclass
class MlstmInputs:
    """q, k, v (B, H, L, d); log_i = input-gate pre-activation (i = exp),
    log_f = logsigmoid(forget pre-activation); gates (B, H, L) fp32."""
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    log_i: torch.Tensor
    log_f: torch.Tensor

    def flops(self, chunk) -> float:
        """Algorithmic chunkwise FLOPs: per chunk 2c^2 d (QK^T) + 2c^2 d (.V)
        + 2 c d^2 (Q.C) + 2 c d^2 (K^T V)."""
        b, h, L, d = self.q.shape
        nc = L / chunk
        return b * h * nc * (2 * chunk * chunk * d * 2 + 2 * chunk * d * d * 2)

    def bytes_moved(self) -> int:
        b, h, L, d = self.q.shape
        es = self.q.element_size()
        return 4 * b * h * L * d * es + 2 * b * h * L * 4


def mlstm_inputs(batch, heads, seqlen, d, dtype=torch.bfloat16, seed=0, device="cpu", on_device=False):
    """q, k, v ~ N(0,1) with q scaled by 1/sqrt(d); input-gate pre-activation
    ~ N(0,1) (used as exp); forget pre-activation ~ N(3,1) (used as logsigmoid)."""
    gdev = device if on_device else "cpu"
    g = _gen(seed, gdev)
    f = dict(generator=g, device=gdev, dtype=torch.float32)
    q = torch.randn(batch, heads, seqlen, d, **f).mul_(1.0 / math.sqrt(d))
    k = torch.randn(batch, heads, seqlen, d, **f)
    v = torch.randn(batch, heads, seqlen, d, **f)
    ipre = torch.randn(batch, heads, seqlen, **f)
    fpre = torch.randn(batch, heads, seqlen, **f).add_(3.0)
    cast = lambda t: t.to(device=device, dtype=dtype)
    return MlstmInputs(cast(q), cast(k), cast(v), ipre.to(device), torch.nn.functional.logsigmoid(fpre).to(device))


@dataclass
class SsdInputs:
    x: torch.Tensor   # (B, L, H, P)
    dt: torch.Tensor  # (B, L, H) fp32, already softplus'ed
    A: torch.Tensor   # (H,)
    B: torch.Tensor   # (B, L, N)
    C: torch.Tensor   # (B, L, N)
    D: torch.Tensor   # (H,)

    def flops(self, chunk) -> float:
        b, L, h, p = self.x.shape
        n = self.B.shape[-1]
        nc = L / chunk
        return b * nc * 2 * chunk * chunk * n + b * h * nc * (2 * chunk * chunk * p + 4 * chunk * n * p)

    def bytes_moved(self) -> int:
        b, L, h, p = self.x.shape
        n = self.B.shape[-1]
        return 2 * b * L * h * p * 2 + 2 * b * L * n * 2 + b * L * h * 4 + b * h * p * n * 4


def ssd_inputs(batch, seqlen, heads, headdim, dstate, seed=0, device="cpu", on_device=False):
    """x, B, C ~ N(0,1) bf16; dt = softplus(N(0,0.5^2) + softplus^-1(U_log[1e-3,1e-1])) fp32;
    A = -U[1,16] per head; D = 1."""
    gdev = device if on_device else "cpu"
    g = _gen(seed, gdev)
    f = dict(generator=g, device=gdev, dtype=torch.float32)
    x = torch.randn(batch, seqlen, heads, headdim, **f)
    Bm = torch.randn(batch, seqlen, dstate, **f)
    Cm = torch.randn(batch, seqlen, dstate, **f)
    dt0 = torch.exp(torch.rand(heads, **f) * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3))
    dt = torch.nn.functional.softplus(torch.randn(batch, seqlen, heads, **f) * 0.5 + softplus_inv(dt0))
    A = -(1.0 + 15.0 * torch.rand(heads, **f))
    D = torch.ones(heads, device=gdev)
    bf = lambda t: t.to(device=device, dtype=torch.bfloat16)
    return SsdInputs(bf(x), dt.to(device), A.to(device), bf(Bm), bf(Cm), D.to(device))


def scan_rows(rows, seqlen, dim, dstate=16, dtype=torch.bfloat16, seed=0, device="cpu"):
    """Batch rows ``rows`` (a range) of one global selective-scan workload, so
    that ranks holding different rows — and a checker regenerating one row —
    see the same numbers: the per-channel parameters (A, D, delta_bias) come
    from ``seed`` and row b's u, delta, z, B, C from seed * 1000 + 1 + b, each
    drawn on ``device``.  Distributions as ``scan_inputs``."""
    g = _gen(seed, device)
    f = dict(generator=g, device=device, dtype=torch.float32)
    dt0 = torch.exp(torch.rand(dim, **f) * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3))
    bias = softplus_inv(dt0)
    A = -torch.arange(1, dstate + 1, dtype=torch.float32, device=device).repeat(dim, 1)
    D = torch.ones(dim, device=device)
    parts = {k: [] for k in ("u", "delta", "z", "B", "C")}
    for b in rows:
        gr = _gen(seed * 1000 + 1 + b, device)
        fr = dict(generator=gr, device=device, dtype=torch.float32)
        parts["u"].append(torch.randn(1, dim, seqlen, **fr).to(dtype))
        parts["z"].append(torch.randn(1, dim, seqlen, **fr).to(dtype))
        parts["delta"].append(torch.randn(1, dim, seqlen, **fr).mul_(0.5).to(dtype))
        parts["B"].append(torch.randn(1, dstate, seqlen, **fr).to(dtype))
        parts["C"].append(torch.randn(1, dstate, seqlen, **fr).to(dtype))
    cat = {k: torch.cat(v, 0) for k, v in parts.items()}
    return ScanInputs(cat["u"], cat["delta"], cat["z"], A, cat["B"], cat["C"], D, bias)


def mlstm_rows(rows, heads, seqlen, d, dtype=torch.bfloat16, seed=0, device="cpu"):
    """Batch rows ``rows`` of one global mLSTM workload with per-head gates,
    row b drawn from seed * 1000 + 1 + b on ``device`` (distributions as
    ``mlstm_inputs``), so any rank or checker can regenerate any row."""
    parts = {k: [] for k in ("q", "k", "v", "li", "lf")}
    for b in rows:
        g = _gen(seed * 1000 + 1 + b, device)
        f = dict(generator=g, device=device, dtype=torch.float32)
        parts["q"].append(torch.randn(1, heads, seqlen, d, **f).mul_(1.0 / math.sqrt(d)).to(dtype))
        parts["k"].append(torch.randn(1, heads, seqlen, d, **f).to(dtype))
        parts["v"].append(torch.randn(1, heads, seqlen, d, **f).to(dtype))
        parts["li"].append(torch.randn(1, heads, seqlen, **f))
        parts["lf"].append(torch.nn.functional.logsigmoid(torch.randn(1, heads, seqlen, **f).add_(3.0)))
    cat = {k: torch.cat(v, 0) for k, v in parts.items()}
    return MlstmInputs(cat["q"], cat["k"], cat["v"], cat["li"], cat["lf"])
