"""The reference's layer callers of the recurrent hot path, wired to the B200 kernels.

Module and parameter names follow hybrid_xmamba/layers so a reference
state_dict loads unchanged:
  RMSNorm        layers/normalization.py:8-34
  MambaBlock     layers/mamba_block.py:17-133
  mLSTMBlock     layers/mlstm_block.py:19-146
  sLSTMBlock     layers/slstm_block.py:18-143 (+ optional block-diagonal
                 recurrent weights ``recurrent_weight`` (H, hd, 4*hd); zero
                 reproduces the reference, which has none)
  HybridBlock    layers/hybrid_block.py:20-147

The projections are plain GEMMs (torch / cuBLAS); the recurrences and the
Mamba causal conv + SiLU are the hxm kernels.  Activations stay in the GEMMs'
(batch, seqlen, features) layout: the kernels read strided column views of
the projection outputs in place, so no transpose or copy runs between them,
and softplus(dt + dt_proj.bias) and y * silu(z) happen inside the scan.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..kernels.conv import causal_conv1d
from ..kernels.norm import rmsnorm
from ..kernels.selective_scan.scan_interface import selective_scan_raw
from ..kernels.slstm import slstm_scan
from ..kernels.tfla.gates import mlstm_gate_epilogue, mlstm_gate_prologue
from ..kernels.tfla.tfla_interface import mlstm_chunkwise_fwd


class RMSNorm(nn.Module):
    """w * x / sqrt(mean(x^2) + eps) over the last dim (normalization.py:8-34),
    one pass of the hxm RMSNorm kernel."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x, residual=None):
        """RMSNorm(x), or with ``residual``: (RMSNorm(x + residual), x + residual)."""
        if residual is None:
            return rmsnorm(x, self.weight, self.eps)
        return rmsnorm(x, self.weight, self.eps, residual=residual, return_sum=True)


class MambaBlock(nn.Module):
    """Mamba mixer (mamba_block.py:29-133): in_proj -> causal depthwise conv +
    SiLU -> x_proj -> dt_proj -> fused selective scan (Euler, softplus(dt+bias),
    + D*u, * silu(z)) -> out_proj."""

    def __init__(self, dim, state_size=16, conv_size=4, expand_factor=2, dt_rank=None, use_fast_path=True):
        super().__init__()
        self.dim, self.state_size, self.conv_size = dim, state_size, conv_size
        self.inner_dim = dim * expand_factor
        self.dt_rank = max(1, dim // 16) if dt_rank is None else dt_rank
        self.use_fast_path = use_fast_path
        self.in_proj = nn.Linear(dim, self.inner_dim * 2, bias=False)
        self.conv1d = nn.Conv1d(self.inner_dim, self.inner_dim, conv_size, padding=conv_size - 1,
                                groups=self.inner_dim, bias=True)
        self.x_proj = nn.Linear(self.inner_dim, self.dt_rank + 2 * state_size, bias=False)
        self.dt_proj = nn.Linear(self.dt_rank, self.inner_dim, bias=True)
        A = torch.arange(1, state_size + 1, dtype=torch.float32).repeat(self.inner_dim, 1)
        self.A_log = nn.Parameter(torch.log(A))
        self.D = nn.Parameter(torch.ones(self.inner_dim))
        self.out_proj = nn.Linear(self.inner_dim, dim, bias=False)

    def forward(self, x, cache=None):
        # Everything stays in (B, L, .) layout: the x / z halves of in_proj and
        # the dt / B / C columns of x_proj are strided views that the conv and
        # scan kernels read in place (unit channel stride), so no transpose or
        # copy kernel runs between the GEMMs.
        di, n, r = self.inner_dim, self.state_size, self.dt_rank
        xz = self.in_proj(x)                                     # (B, L, 2*di)
        x_in, z = xz[..., :di], xz[..., di:]
        # with a cache (dict): continue from / update the conv inputs and the scan state
        conv0 = cache.get("conv") if cache is not None else None
        ssm0 = cache.get("ssm") if cache is not None else None
        conv = causal_conv1d(x_in, self.conv1d.weight, self.conv1d.bias, activation="silu", initial_state=conv0,
                             return_final_state=cache is not None)
        u, conv_state = conv if cache is not None else (conv, None)                          # (B, L, di)
        dbc = self.x_proj(u)                                     # (B, L, r + 2n)
        dt_low, Bm, Cm = dbc[..., :r], dbc[..., r:r + n], dbc[..., r + n:]
        delta = F.linear(dt_low, self.dt_proj.weight)            # (B, L, di); bias folded into the scan
        A, D, dt_bias = self._scan_params()
        res = selective_scan_raw(u, delta, A, Bm, Cm, D, z, z_mode="silu", delta_bias=dt_bias, delta_softplus=True,
                                 h0=ssm0, return_last_state=cache is not None)             # (B, L, di)
        if cache is not None:
            y, cache["ssm"] = res
            cache["conv"] = conv_state
        else:
            y = res
        return self.out_proj(y)

    def _scan_params(self):
        """fp32 A = -exp(A_log), D and dt_proj.bias; cached while the parameters
        are unchanged and no gradient is being recorded (inference)."""
        params = (self.A_log, self.D, self.dt_proj.bias)
        derive = lambda: (-torch.exp(self.A_log.float()), self.D.float(), self.dt_proj.bias.float())
        if torch.is_grad_enabled() and any(p.requires_grad for p in params):
            return derive()
        key = tuple((p.data_ptr(), p._version, p.device) for p in params)
        if getattr(self, "_scan_key", None) != key:
            with torch.no_grad():
                self._scan_val = derive()
            self._scan_key = key
        return self._scan_val


class mLSTMBlock(nn.Module):
    """mLSTM mixer (mlstm_block.py:32-146): projections, per-head RMSNorm of
    q and k, i = exp, f = sigmoid, o = sigmoid per channel, the mLSTM
    recurrence, h*o*sigmoid(x_gate), out_proj."""

    def __init__(self, dim, head_dim=64, num_heads=None, use_tfla=True, proj_factor=2):
        super().__init__()
        self.dim, self.head_dim = dim, head_dim
        self.num_heads = max(1, dim // head_dim) if num_heads is None else num_heads
        self.inner_dim = self.num_heads * head_dim
        self.use_tfla, self.proj_factor = use_tfla, proj_factor
        self.in_proj = nn.Linear(dim, self.inner_dim * proj_factor, bias=False)
        self.q_proj = nn.Linear(self.inner_dim, self.inner_dim, bias=False)
        self.k_proj = nn.Linear(self.inner_dim, self.inner_dim, bias=False)
        self.v_proj = nn.Linear(self.inner_dim, self.inner_dim, bias=False)
        self.i_gate_proj = nn.Linear(self.inner_dim, self.inner_dim, bias=True)
        self.f_gate_proj = nn.Linear(self.inner_dim, self.inner_dim, bias=True)
        self.o_gate_proj = nn.Linear(self.inner_dim, self.inner_dim, bias=True)
        self.q_norm = RMSNorm(head_dim)
        self.k_norm = RMSNorm(head_dim)
        self.out_proj = nn.Linear(self.inner_dim, dim, bias=False)
        self.register_buffer("eps", torch.tensor(1e-6))

    def forward(self, x, cache=None):
        bsz, L, _ = x.shape
        nh, hd = self.num_heads, self.head_dim
        inner = self.inner_dim
        if self.proj_factor == 2:
            # the two halves of in_proj as two GEMMs: contiguous x_inner feeds the next GEMMs
            w = self.in_proj.weight
            x_inner, x_gate = F.linear(x, w[:inner]), F.linear(x, w[inner:])
        else:
            x_inner = x_gate = self.in_proj(x)
        # (B, L, H, hd) memory throughout; the mLSTM kernels take the (B, H, L, hd)
        # views with their time stride, so no transpose copy runs.
        split = lambda t: t.view(bsz, L, nh, hd)
        heads = lambda t: split(t).transpose(1, 2)                  # (B, H, L, hd) view
        q = self.q_norm(split(self.q_proj(x_inner))).transpose(1, 2)
        k = self.k_norm(split(self.k_proj(x_inner))).transpose(1, 2)
        v = heads(self.v_proj(x_inner))
        # i, f, o gate projections as one GEMM with the bias in its epilogue
        w_ifo, b_ifo = self._gate_params()
        ifo = F.linear(x_inner, w_ifo, b_ifo)                       # (B, L, 3*inner)
        # log_i = i_pre (i = exp), log_f = logsigmoid(f_pre): one fused pass
        log_i, log_f = mlstm_gate_prologue(ifo[..., :inner], ifo[..., inner:2 * inner])
        log_i, log_f = heads(log_i), heads(log_f)
        h = torch.empty(bsz, L, nh, hd, device=x.device, dtype=q.dtype)
        if cache is None:
            mlstm_chunkwise_fwd(q, k, v, log_i, log_f, out=h.transpose(1, 2))
        else:  # continue from / update the stabilized state (C, n, m)
            _, st = mlstm_chunkwise_fwd(q, k, v, log_i, log_f, cache.get("C"), cache.get("n"), cache.get("m"),
                                        out=h.transpose(1, 2), return_state=True)
            cache["C"], cache["n"], cache["m"] = st
        # h * sigmoid(o_pre) * sigmoid(x_gate): one fused pass
        h = mlstm_gate_epilogue(h.view(bsz, L, nh * hd), ifo[..., 2 * inner:], x_gate)
        return self.out_proj(h)


    def _gate_params(self):
        """[W_i; W_f; W_o] and [b_i; b_f; b_o] stacked; cached while the
        parameters are unchanged and no gradient is being recorded."""
        mods = (self.i_gate_proj, self.f_gate_proj, self.o_gate_proj)
        params = [m.weight for m in mods] + [m.bias for m in mods]
        derive = lambda: (torch.cat([m.weight for m in mods]), torch.cat([m.bias for m in mods]))
        if torch.is_grad_enabled() and any(p.requires_grad for p in params):
            return derive()
        key = tuple((p.data_ptr(), p._version, p.device, p.dtype) for p in params)
        if getattr(self, "_gate_key", None) != key:
            with torch.no_grad():
                self._gate_val = derive()
            self._gate_key = key
        return self._gate_val


class sLSTMBlock(nn.Module):
    """sLSTM mixer (slstm_block.py:30-143) with the recurrence in the hxm
    kernel.  ``recurrent_weight`` (H, hd, 4*hd) adds R[head]^T h_{t-1} to the
    gate pre-activations (zero-initialised: the reference block has no R)."""

    def __init__(self, dim, hidden_dim=None, num_heads=4, use_exponential_gate=True, recurrent=False):
        super().__init__()
        self.dim = dim
        self.hidden_dim = hidden_dim or dim
        self.num_heads = num_heads
        self.use_exponential_gate = use_exponential_gate
        assert self.hidden_dim % num_heads == 0
        self.head_dim = self.hidden_dim // num_heads
        self.in_proj = nn.Linear(dim, self.hidden_dim, bias=False)
        self.gate_proj = nn.Linear(self.hidden_dim, self.hidden_dim * 4, bias=True)
        self.h_norm = RMSNorm(self.head_dim)
        self.out_proj = nn.Linear(self.hidden_dim, dim, bias=False)
        self.register_buffer("eps", torch.tensor(1e-6))
        self.recurrent_weight = (nn.Parameter(torch.zeros(num_heads, self.head_dim, 4 * self.head_dim))
                                 if recurrent else None)

    def forward(self, x, cache=None):
        bsz, L, _ = x.shape
        gates = self.gate_proj(self.in_proj(x)).view(bsz, L, self.num_heads, 4, self.head_dim)
        h0 = c0 = None
        if cache is not None and "h" in cache and "c" in cache:
            h0, c0 = cache["h"], cache["c"]
        h_seq, (h, c) = slstm_scan(gates, self.h_norm.weight, R=self.recurrent_weight, eps=self.h_norm.eps,
                                   exponential_gate=self.use_exponential_gate, h0=h0, c0=c0)
        if cache is not None:  # fp32 true states (the reference keeps them in x's dtype)
            cache["h"], cache["c"] = h, c
        return self.out_proj(h_seq.reshape(bsz, L, self.hidden_dim))


class HybridBlock(nn.Module):
    """Pre-norm mixer + residual, optional pre-norm GELU MLP + residual
    (hybrid_block.py:38-134), with the reference's kwarg routing (:58-88)."""

    def __init__(self, dim, layer_type="mamba", norm_type="rms", use_mlp=True, mlp_ratio=4.0, **kw):
        super().__init__()
        self.dim, self.layer_type, self.use_mlp = dim, layer_type.lower(), use_mlp
        norm = (lambda: RMSNorm(dim)) if norm_type.lower() == "rms" else (lambda: nn.LayerNorm(dim))
        self.norm1 = norm()
        if self.layer_type == "mamba":
            keys = {"state_size", "conv_size", "expand_factor", "dt_rank", "use_fast_path"}
            self.mixer = MambaBlock(dim, **{k: v for k, v in kw.items() if k in keys})
        elif self.layer_type == "mlstm":
            keys = {"head_dim", "num_heads", "use_tfla", "proj_factor"}
            self.mixer = mLSTMBlock(dim, **{k: v for k, v in kw.items() if k in keys})
        elif self.layer_type == "slstm":
            sk = {}
            for k, v in kw.items():
                if k.startswith("slstm_"):
                    name = k[len("slstm_"):]
                    if name in ("hidden_dim", "num_heads", "use_exponential_gate", "recurrent"):
                        sk[name] = v
                elif k in ("num_heads", "use_exponential_gate"):
                    sk[k] = v
            self.mixer = sLSTMBlock(dim, **sk)
        else:
            raise ValueError(f"Unknown layer type: {layer_type}")
        if use_mlp:
            self.norm2 = norm()
            self.mlp = nn.Sequential(nn.Linear(dim, int(dim * mlp_ratio), bias=False), nn.GELU(),
                                     nn.Linear(int(dim * mlp_ratio), dim, bias=False))
        else:
            self.norm2 = self.mlp = None

    def forward(self, x, cache=None):
        out, pending = self.forward_pending(x, None, cache=cache)
        return out + pending if pending is not None else out

    def forward_pending(self, x, pending, cache=None):
        """The block with its last residual add left pending: returns (x, d)
        with the block output = x + d (d None when nothing is pending).  A
        pending add from the previous block is fused into norm1, and the mixer's
        residual add into norm2 (one RMSNorm kernel pass each)."""
        fused = isinstance(self.norm1, RMSNorm)
        if pending is not None:
            if fused:
                h, x = self.norm1(pending, residual=x)
            else:
                x = x + pending
                h = self.norm1(x)
        else:
            h = self.norm1(x)
        m = self.mixer(h, cache=cache)
        if not self.use_mlp:
            return x, m
        if fused:
            h2, x = self.norm2(m, residual=x)
        else:
            x = x + m
            h2 = self.norm2(x)
        return x, self.mlp(h2)
