"""Generate golden input/output vectors by running the REFERENCE itself.

Run where a checkout of the reference exists and name its root in the
environment variable HXM_REFERENCE_ROOT (the directory that holds the
``hybrid_xmamba`` package).  The reference is imported read-only and executed
in float64 on CPU; the fixtures (small .npz files in this directory) are
committed so that the tests never need the reference at run time.

What each fixture pins (reference file:line of the code that produced it):
  scan_*.npz     selective_scan_pytorch / selective_scan
                 (hybrid_xmamba/kernels/selective_scan/scan_interface.py:103-180)
  scan_zoh.npz   the ZOH / Taylor discretization of MambaBlock._selective_scan_pytorch
                 (hybrid_xmamba/layers/mamba_block_v2.py:280-351)
  tfla_*.npz     tfla_forward_pytorch (hybrid_xmamba/kernels/tfla/tfla_interface.py:84-139)
  slstm_*.npz    sLSTMBlock.forward with a correctly shaped cache
                 (hybrid_xmamba/layers/slstm_block.py:64-143); gate_proj output and
                 the out_proj input are captured with forward hooks
  mamba_block.npz, mlstm_block.npz   layer forwards (mamba_block.py:80-133,
                 mlstm_block.py:77-146) with their state_dicts
  conv_block.npz the Mamba conv + SiLU (mamba_block.py:97-104), captured with a
                 forward hook on the block's SiLU module
  hybrid_lm.npz  HybridLanguageModel.forward (hybrid_xmamba/models/hybrid_lm.py:145-209)
                 at a tiny size; sLSTM blocks get the correctly shaped zero cache
                 (the reference crashes without it, slstm_block.py:109-112)
  hybrid_lm350m.npz  the same forward at the hybrid-350M architecture, batch 1 x 256,
                 with name-seeded weights (lm350m_weights.py); logit slices and sums

Usage:  python tests/golden/make_golden.py [fixture-function ...]
        (no argument: all fixtures; e.g. ``make_conv`` regenerates one)
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("HXM_REFERENCE_ROOT", "")


def _import_reference():
    if not REF or not os.path.isdir(os.path.join(REF, "hybrid_xmamba")):
        sys.exit("set HXM_REFERENCE_ROOT to the reference checkout (the directory holding hybrid_xmamba/)")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    from hybrid_xmamba.kernels.selective_scan import scan_interface
    from hybrid_xmamba.kernels.tfla import tfla_interface
    from hybrid_xmamba.layers import slstm_block, mamba_block, mlstm_block
    from hybrid_xmamba.models import hybrid_lm, configuration_hybrid
    return scan_interface, tfla_interface, slstm_block, mamba_block, mlstm_block, hybrid_lm, configuration_hybrid


def scan_inputs_cfg1(gen, bsz, L, dm, n):
    """BASELINE config-1 value distributions (S4D-real A, log-uniform dt bias)."""
    u = torch.randn(bsz, dm, L, generator=gen)
    z = torch.randn(bsz, dm, L, generator=gen)
    raw = 0.5 * torch.randn(bsz, dm, L, generator=gen)
    dt0 = torch.exp(torch.rand(dm, generator=gen) * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3))
    bias = dt0 + torch.log(-torch.expm1(-dt0))  # softplus^-1(dt0)
    A = -torch.arange(1, n + 1, dtype=torch.float32).repeat(dm, 1)
    Bm = torch.randn(bsz, n, L, generator=gen)
    Cm = torch.randn(bsz, n, L, generator=gen)
    D = torch.ones(dm)
    return u, z, raw, bias, A, Bm, Cm, D


def make_scan(si):
    gen = torch.Generator().manual_seed(0)
    # (1) the reference test's shapes and distributions (tests/test_kernels.py:63-70)
    bsz, L, dm, n = 2, 64, 128, 16
    x = torch.randn(bsz, L, dm, generator=gen)
    dt = torch.nn.functional.softplus(torch.randn(bsz, L, dm, generator=gen))
    A = -torch.randn(dm, n, generator=gen).exp()
    Bm = torch.randn(bsz, L, n, generator=gen)
    Cm = torch.randn(bsz, L, n, generator=gen)
    D = torch.randn(dm, generator=gen)
    z = torch.randn(bsz, L, dm, generator=gen)
    d64 = lambda t: t.to(torch.float64)
    y = si.selective_scan_pytorch(d64(x), d64(dt), d64(A), d64(Bm), d64(Cm), d64(D))
    yz = si.selective_scan(d64(x), d64(dt), d64(A), d64(Bm), d64(Cm), d64(D), z=d64(z))
    np.savez_compressed(os.path.join(HERE, "scan_small.npz"), x=x.numpy(), dt=dt.numpy(), A=A.numpy(),
                        B=Bm.numpy(), C=Cm.numpy(), D=D.numpy(), z=z.numpy(), y=y.numpy(), y_z=yz.numpy())
    # (2) config-1 distributions on a channel slice at full seqlen 512 (B=2, D=48 of 1536)
    bsz, L, dm, n = 2, 512, 48, 16
    u, zz, raw, bias, A, Bm, Cm, D = scan_inputs_cfg1(gen, bsz, L, dm, n)
    delta = torch.nn.functional.softplus(d64(raw) + d64(bias)[None, :, None])
    ref = si.selective_scan_pytorch(d64(u).transpose(1, 2), delta.transpose(1, 2), d64(A),
                                    d64(Bm).transpose(1, 2), d64(Cm).transpose(1, 2), d64(D))
    y = ref * torch.nn.functional.silu(d64(zz).transpose(1, 2))
    np.savez_compressed(os.path.join(HERE, "scan_cfg1_slice.npz"), u=u.numpy(), z=zz.numpy(), raw=raw.numpy(),
                        bias=bias.numpy(), A=A.numpy(), B=Bm.numpy(), C=Cm.numpy(), D=D.numpy(),
                        y=y.transpose(1, 2).numpy())


def make_tfla(ti):
    gen = torch.Generator().manual_seed(1)
    for name, (b, h, L, d) in {"tfla_1x2x16x8": (1, 2, 16, 8), "tfla_2x4x32x16": (2, 4, 32, 16),
                               "tfla_2x4x64x32": (2, 4, 64, 32)}.items():
        q = torch.randn(b, h, L, d, generator=gen)
        k = torch.randn(b, h, L, d, generator=gen)
        v = torch.randn(b, h, L, d, generator=gen)
        ipre = torch.randn(b, h, L, d, generator=gen)
        fpre = torch.randn(b, h, L, d, generator=gen)
        out = ti.tfla_forward_pytorch(q.double(), k.double(), v.double(), ipre.double().exp(),
                                      torch.sigmoid(fpre.double()))
        np.savez_compressed(os.path.join(HERE, name + ".npz"), q=q.numpy(), k=k.numpy(), v=v.numpy(),
                            i_pre=ipre.numpy(), f_pre=fpre.numpy(), h=out.numpy())
    # config-2 distributions (scalar gates broadcast over d), reduced size
    b, h, L, d = 1, 2, 192, 64
    q = torch.randn(b, h, L, d, generator=gen) / math.sqrt(d)
    k = torch.randn(b, h, L, d, generator=gen)
    v = torch.randn(b, h, L, d, generator=gen)
    ipre = torch.randn(b, h, L, generator=gen)
    fpre = 3.0 + torch.randn(b, h, L, generator=gen)
    ig = ipre.double().exp()[..., None].expand(b, h, L, d)
    fg = torch.sigmoid(fpre.double())[..., None].expand(b, h, L, d)
    out = ti.tfla_forward_pytorch(q.double(), k.double(), v.double(), ig, fg)
    np.savez_compressed(os.path.join(HERE, "tfla_scalar_gates.npz"), q=q.numpy(), k=k.numpy(), v=v.numpy(),
                        i_pre=ipre.numpy(), f_pre=fpre.numpy(), h=out.numpy())


def make_slstm(sb):
    gen = torch.Generator().manual_seed(2)
    torch.manual_seed(2)
    bsz, L, dim, hidden, nh = 2, 40, 32, 64, 4
    blk = sb.sLSTMBlock(dim, hidden_dim=hidden, num_heads=nh).double()
    with torch.no_grad():
        blk.h_norm.weight.copy_(1.0 + 0.1 * torch.randn(hidden // nh, generator=gen))
        blk.gate_proj.bias.copy_(0.1 * torch.randn(4 * hidden, generator=gen))
    x = torch.randn(bsz, L, dim, generator=gen, dtype=torch.float64)
    cap = {}
    blk.gate_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("gates", o.detach().clone()))
    blk.out_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("h_seq", i[0].detach().clone()))
    hd = hidden // nh
    cache = {"h": torch.zeros(bsz, nh, hd, dtype=torch.float64), "c": torch.zeros(bsz, nh, hd, dtype=torch.float64)}
    out = blk(x, cache=cache)
    np.savez_compressed(os.path.join(HERE, "slstm_block.npz"), x=x.numpy(),
                        gates=cap["gates"].numpy(), h_seq=cap["h_seq"].numpy(), out=out.detach().numpy(),
                        h=cache["h"].detach().numpy(), c=cache["c"].detach().numpy(), norm_w=blk.h_norm.weight.detach().numpy(),
                        heads=nh, head_dim=hd,
                        **{"sd_" + k: v.detach().numpy() for k, v in blk.state_dict().items()})


def make_layers(mb, lb):
    gen = torch.Generator().manual_seed(3)
    torch.manual_seed(3)
    blk = mb.MambaBlock(64, state_size=16).double()
    with torch.no_grad():
        blk.dt_proj.bias.copy_(torch.log(torch.expm1(torch.full((128,), 0.01, dtype=torch.float64))))
    x = torch.randn(2, 48, 64, generator=gen, dtype=torch.float64)
    out = blk(x)
    np.savez_compressed(os.path.join(HERE, "mamba_block.npz"), x=x.numpy(), out=out.detach().numpy(),
                        **{"sd_" + k: v.detach().numpy() for k, v in blk.state_dict().items()})
    torch.manual_seed(4)
    blk = lb.mLSTMBlock(64, head_dim=32, num_heads=2).double()
    x = torch.randn(2, 48, 64, generator=gen, dtype=torch.float64)
    out = blk(x)
    np.savez_compressed(os.path.join(HERE, "mlstm_block.npz"), x=x.numpy(), out=out.detach().numpy(),
                        **{"sd_" + k: v.detach().numpy() for k, v in blk.state_dict().items() if k != "eps"})


def make_conv(mb):
    """The reference MambaBlock's conv + SiLU output (mamba_block.py:101-104),
    captured at the first call of its SiLU module, and the conv input
    (the x half of in_proj, mamba_block.py:97-98)."""
    gen = torch.Generator().manual_seed(5)
    torch.manual_seed(5)
    blk = mb.MambaBlock(32, state_size=8, conv_size=4).double()
    x = torch.randn(2, 40, 32, generator=gen, dtype=torch.float64)
    seen = []
    h = blk.activation.register_forward_hook(lambda m, i, o: seen.append(o.detach().clone()))
    with torch.no_grad():
        blk(x)
        x_inner = blk.in_proj(x).chunk(2, dim=-1)[0]
    h.remove()
    np.savez_compressed(os.path.join(HERE, "conv_block.npz"), x_inner=x_inner.numpy(), conv_silu=seen[0].numpy(),
                        weight=blk.conv1d.weight.detach().numpy(), bias=blk.conv1d.bias.detach().numpy())


def make_lm(hl, cfgmod, sb):
    orig = sb.sLSTMBlock.forward

    def fwd_with_cache(self, x, cache=None):
        if cache is None:
            z = torch.zeros(x.shape[0], self.num_heads, self.head_dim, dtype=x.dtype)
            cache = {"h": z.clone(), "c": z.clone()}
        return orig(self, x, cache=cache)

    sb.sLSTMBlock.forward = fwd_with_cache
    try:
        torch.manual_seed(5)
        cfg = cfgmod.HybridConfig(vocab_size=97, dim=64, num_layers=4,
                                  layer_pattern=["mamba", "mamba", "mlstm", "slstm"],
                                  state_size=16, conv_size=4, expand_factor=2, head_dim=32, num_heads=2,
                                  slstm_num_heads=4, dropout=0.0)
        model = hl.HybridLanguageModel(cfg).double().eval()
        ids = torch.randint(0, 97, (2, 24), generator=torch.Generator().manual_seed(6))
        logits = model(ids).logits
        np.savez_compressed(os.path.join(HERE, "hybrid_lm.npz"), ids=ids.numpy(), logits=logits.detach().numpy(),
                            **{"sd_" + k: v.detach().numpy() for k, v in model.state_dict().items()
                               if not k.endswith(".eps")})
    finally:
        sb.sLSTMBlock.forward = orig


def make_lm350m(hl, cfgmod, sb):
    """HybridLanguageModel.forward (hybrid_lm.py:145-209) at the hybrid-350M
    architecture (d 1024, 24 layers of [Mamba, Mamba, mLSTM, sLSTM], Mamba
    expand 2 / d_state 16 / conv 4, mLSTM 4 heads x 512, sLSTM 4 heads, vocab
    50304, the reference's default MLP), float64, batch 1 x 256 tokens, with
    the name-seeded weights of lm350m_weights.py (the reference has no sLSTM
    recurrent weights: R = 0).  Stored: slices of the logits (every position
    over the first 512 vocabulary entries, five positions over all of it), the
    sum / sum of squares of all logits, and how far the reference's own fp32
    run lands from its float64 run on the same slices (the model amplifies
    rounding late in the sequence, so that is the scale an fp32 port is judged
    against)."""
    sys.path.insert(0, HERE)
    import lm350m_weights as W
    orig = sb.sLSTMBlock.forward

    def fwd_with_cache(self, x, cache=None):
        if cache is None:
            z = torch.zeros(x.shape[0], self.num_heads, self.head_dim, dtype=x.dtype)
            cache = {"h": z.clone(), "c": z.clone()}
        return orig(self, x, cache=cache)

    sb.sLSTMBlock.forward = fwd_with_cache
    try:
        cfg = cfgmod.HybridConfig(vocab_size=50304, dim=1024, num_layers=24,
                                  layer_pattern=["mamba", "mamba", "mlstm", "slstm"], state_size=16, conv_size=4,
                                  expand_factor=2, head_dim=512, num_heads=4, slstm_num_heads=4, dropout=0.0)
        model = hl.HybridLanguageModel(cfg)
        names = W.fill_(model)
        model = model.eval()
        ids = torch.randint(0, 50304, (1, 256), generator=torch.Generator().manual_seed(8))
        pos = np.array([0, 63, 127, 191, 255])
        with torch.no_grad():
            l32 = model(ids).logits[0].double()  # the reference's own fp32 run
            logits = model.double()(ids).logits[0]
        rel = lambda a, b: float(torch.linalg.norm(a - b) / torch.linalg.norm(b))
        np.savez_compressed(os.path.join(HERE, "hybrid_lm350m.npz"), ids=ids.numpy(),
                            logits_head=logits[:, :512].float().numpy(), positions=pos,
                            logits_rows=logits[pos].float().numpy(), logit_sum=float(logits.sum()),
                            logit_sumsq=float((logits * logits).sum()), n_filled=len(names),
                            n_params=sum(p.numel() for p in model.parameters()),
                            ref_fp32_err_head=rel(l32[:, :512], logits[:, :512]),
                            ref_fp32_err_rows=rel(l32[pos], logits[pos]))
    finally:
        sb.sLSTMBlock.forward = orig


def make_zoh():
    """MambaBlock._selective_scan_pytorch of the v2 block (mamba_block_v2.py:280-351):
    Bbar = (exp(dA) - 1) / A * B, or dt * B where |dA| < 0.01 (its Taylor branch).
    The method uses no module state, so it is called unbound.  delta spans both
    branches: softplus(N(0, 0.5^2) + softplus^-1(dt0)), dt0 log-uniform in
    [1e-3, 1e-1], against A = -(1..16)."""
    from hybrid_xmamba.layers import mamba_block_v2 as mb2
    gen = torch.Generator().manual_seed(7)
    bsz, L, dm, n = 2, 48, 24, 16
    x = torch.randn(bsz, L, dm, generator=gen, dtype=torch.float64)
    dt0 = torch.exp(torch.rand(dm, generator=gen, dtype=torch.float64) * (math.log(1e-1) - math.log(1e-3))
                    + math.log(1e-3))
    raw = 0.5 * torch.randn(bsz, L, dm, generator=gen, dtype=torch.float64)
    delta = torch.nn.functional.softplus(raw + dt0 + torch.log(-torch.expm1(-dt0)))
    A = -torch.arange(1, n + 1, dtype=torch.float64).repeat(dm, 1)
    Bm = torch.randn(bsz, L, n, generator=gen, dtype=torch.float64)
    Cm = torch.randn(bsz, L, n, generator=gen, dtype=torch.float64)
    D = torch.randn(dm, generator=gen, dtype=torch.float64)
    y = mb2.MambaBlock._selective_scan_pytorch(None, x, delta, A, Bm, Cm, D)
    taylor = float(((delta[..., None] * A).abs() < 0.01).double().mean())
    np.savez_compressed(os.path.join(HERE, "scan_zoh.npz"), x=x.numpy(), delta=delta.numpy(), A=A.numpy(),
                        B=Bm.numpy(), C=Cm.numpy(), D=D.numpy(), y=y.numpy(), taylor_fraction=taylor)


def main():
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    si, ti, sb, mb, lb, hl, cfgmod = _import_reference()
    if len(sys.argv) > 1:
        args = {"make_scan": (si,), "make_tfla": (ti,), "make_slstm": (sb,), "make_layers": (mb, lb),
                "make_conv": (mb,), "make_lm": (hl, cfgmod, sb), "make_zoh": (),
                "make_lm350m": (hl, cfgmod, sb)}
        for name in sys.argv[1:]:
            globals()[name](*args[name])
        return
    make_scan(si)
    make_tfla(ti)
    make_slstm(sb)
    make_layers(mb, lb)
    make_conv(mb)
    make_lm(hl, cfgmod, sb)
    make_zoh()
    make_lm350m(hl, cfgmod, sb)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f"{f:28s} {os.path.getsize(os.path.join(HERE, f)) / 1024:8.1f} KiB")


if __name__ == "__main__":
    main()
