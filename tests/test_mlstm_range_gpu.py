"""mLSTM over the whole gate range, forward and backward, against the float64 oracle.

Strong forget gates push the key-streaming kernel's chunk factors e^(|g|/2)
past the fp32 range (logsigmoid of N(-1.5, 1), N(-2, 1) and N(-4, 1)
pre-activations sum to about -230, -280 and -520 per 128 steps): the prescale
pass flags those (batch, head) pairs on the device, they are prescaled again
in 64-step chunks and run with those, and the pairs still out of range (the
N(-4, 1) case) take the exact recurrent kernel — all in the same call.  The
reference loop (tfla_interface.py:84-139) multiplies by f step by step and
has no such limit, so neither may this path.  The chunkwise backward shortens
its chunk for such gates.

Tolerances: bf16 I/O 2e-2 normwise relative error against the float64
oracle on the same bf16-rounded inputs, final states included (as
exp(m) * (C, n) against the true state); fp32 backward 1e-4 against float64
autograd of the loop.
"""
import math

import numpy as np
import pytest
import torch

from oracle import numpy_ref as R
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
TOL16 = 2e-2


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from hybrid_model_mamba_xlstm_b200.kernels.tfla import tfla_interface as ti
    return ti


def np64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def _inputs(shape, fmu, seed, per_channel=True, imu=0.0, isd=1.0):
    """Config-2 value distributions with the forget pre-activation ~ N(fmu, 1)."""
    b, h, L, d = shape
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(b, h, L, d, generator=g) / math.sqrt(d)).to("cuda", torch.bfloat16)
    k = torch.randn(b, h, L, d, generator=g).to("cuda", torch.bfloat16)
    v = torch.randn(b, h, L, d, generator=g).to("cuda", torch.bfloat16)
    gs = (b, h, L, d) if per_channel else (b, h, L)
    li = (torch.randn(*gs, generator=g) * isd + imu).cuda()
    lf = torch.nn.functional.logsigmoid(torch.randn(*gs, generator=g) + fmu).cuda()
    return q, k, v, li, lf


def _check(ops, q, k, v, li, lf):
    out, (C, n, m) = ops.mlstm_chunkwise_fwd(q, k, v, li, lf, return_state=True)
    ref, Cr, nr = R.tfla_recurrent(np64(q), np64(k), np64(v), np.exp(np64(li)), np.exp(np64(lf)))
    assert np.isfinite(np64(out)).all()
    assert rel_err(np64(out), ref) < TOL16
    em = np.exp(np64(m))
    assert rel_err(np64(C) * em[..., None, None], Cr) < TOL16
    assert rel_err(np64(n) * em[..., None], nr) < TOL16
    return out


@pytest.mark.parametrize("d", [128, 256, 512])
@pytest.mark.parametrize("fmu", [-1.5, -2.0, -4.0])
def test_strong_channel_forget_gates(ops, d, fmu):
    """Per-channel gates (mLSTMBlock) with strong forgetting, lengths that are
    not a multiple of the 128- or 64-step chunk."""
    _check(ops, *_inputs((1, 2, 300, d), fmu, seed=int(-10 * fmu) + d))


def test_64_step_chunks_long_and_segmented(ops):
    """Every pair in the 64-step range (forget pre-activation N(-1.5, 1)),
    700 steps, with an initial state: the state carried across a split of
    the sequence and across the 64-step chunks matches one pass."""
    q, k, v, li, lf = _inputs((2, 2, 700, 256), -1.5, seed=47)
    out = _check(ops, q, k, v, li, lf)
    s = 333
    a, st = ops.mlstm_chunkwise_fwd(q[:, :, :s], k[:, :, :s], v[:, :, :s], li[:, :, :s], lf[:, :, :s],
                                    return_state=True)
    b2, _ = ops.mlstm_chunkwise_fwd(q[:, :, s:], k[:, :, s:], v[:, :, s:], li[:, :, s:], lf[:, :, s:], *st,
                                    return_state=True)
    assert rel_err(np64(torch.cat([a, b2], 2)), np64(out)) < TOL16


@pytest.mark.parametrize("d", [256, 512])
def test_strong_head_forget_gates(ops, d):
    """Per-head gates with strong forgetting: d = 512 runs the key-streaming
    kernel (its per-head prescale), d = 256 the tcgen05 chunkwise kernel."""
    _check(ops, *_inputs((2, 2, 333, d), -4.0, seed=d, per_channel=False))


def test_mixed_heads_stream_and_fallback(ops):
    """One call where (batch, head) pairs take all three routes — 128-step
    chunks, 64-step chunks, the exact recurrence: each pair is run by exactly
    one kernel and the outputs and states of every kind match the oracle."""
    q, k, v, li, lf = _inputs((2, 3, 260, 128), 3.0, seed=41)
    g = torch.Generator().manual_seed(42)
    strong = torch.nn.functional.logsigmoid(torch.randn(260, 128, generator=g) - 4.0).cuda()
    medium = torch.nn.functional.logsigmoid(torch.randn(260, 128, generator=g) - 1.5).cuda()
    lf[0, 1] = strong
    lf[1, 2] = strong
    lf[1, 0] = medium
    out = _check(ops, q, k, v, li, lf)
    # the pairs left in range agree with a call that holds only them (no cross-talk)
    alone = ops.mlstm_chunkwise_fwd(q[:1, :1], k[:1, :1], v[:1, :1], li[:1, :1], lf[:1, :1])
    assert torch.equal(alone, out[:1, :1])


def test_forget_gate_zero_steps(ops):
    """f = 0 on some steps (log f = -inf, e.g. sigmoid underflow): the state
    restarts there, as in the reference's multiply by f."""
    q, k, v, li, lf = _inputs((1, 2, 200, 128), 1.0, seed=43)
    lf[:, :, 50] = float("-inf")
    lf[0, 1, 170, :64] = float("-inf")
    _check(ops, q, k, v, li, lf)


def test_large_input_gates_in_range(ops):
    """Input gates exp(N(10, 2)) with moderate forgetting: the bound counts
    log i as well as the forget gates (the state grows with i)."""
    _check(ops, *_inputs((1, 2, 256, 128), 0.0, seed=44, imu=10.0, isd=2.0))


# ------------------------------------------------------------------ backward --
def _loop(q, k, v, ig, fg):
    """float64 restatement of tfla_forward_pytorch (tfla_interface.py:84-139)."""
    bsz, nh, L, d = q.shape
    C = torch.zeros(bsz, nh, d, v.shape[-1], dtype=q.dtype)
    n = torch.zeros(bsz, nh, d, dtype=q.dtype)
    hs = []
    for t in range(L):
        C = fg[:, :, t, :, None] * C + ig[:, :, t, :, None] * (k[:, :, t, :, None] * v[:, :, t, None, :])
        n = fg[:, :, t] * n + ig[:, :, t] * k[:, :, t]
        num = torch.einsum("bhd,bhde->bhe", q[:, :, t], C)
        den = torch.clamp(torch.einsum("bhd,bhd->bh", q[:, :, t], n), min=1.0)[..., None]
        hs.append(num / den)
    return torch.stack(hs, 2)


@pytest.mark.parametrize("d,dtype", [(128, torch.float32), (128, torch.bfloat16), (512, torch.bfloat16)])
@pytest.mark.parametrize("fmu", [-2.0, -4.0])
def test_strong_channel_forget_gates_backward(ops, d, dtype, fmu):
    """Every gradient of apply_tfla with strong per-channel forget gates vs
    float64 autograd of the loop; the chunkwise backward shortens its chunk."""
    from hybrid_model_mamba_xlstm_b200.kernels.tfla import tfla_bwd
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        g = torch.Generator().manual_seed(int(-fmu) * 7 + d)
        b, h, L = 1, 2, 150
        q = (torch.randn(b, h, L, d, generator=g) / math.sqrt(d)).to(dtype)
        k = torch.randn(b, h, L, d, generator=g).to(dtype)
        v = torch.randn(b, h, L, d, generator=g).to(dtype)
        ig = torch.exp(torch.randn(b, h, L, d, generator=g) * 0.5)
        fg = torch.sigmoid(torch.randn(b, h, L, d, generator=g) + fmu)
        dh = torch.randn(b, h, L, d, generator=g).to(dtype)
        c = tfla_bwd._channel_chunk(torch.log(ig).cuda(), torch.log(fg).cuda(), 64)
        assert c < 64  # the 64-step chunk is out of range for these gates
        leaves = [t.cuda().requires_grad_(True) for t in (q, k, v, ig, fg)]
        out = ops.apply_tfla(*leaves)
        out.backward(dh.cuda())
        ref = [t.detach().double().requires_grad_(True) for t in (q, k, v, ig, fg)]
        rout = _loop(*ref)
        rout.backward(dh.double())
        tol = 1e-4 if dtype == torch.float32 else TOL16
        assert rel_err(np64(out), rout.detach().numpy()) < (1e-5 if dtype == torch.float32 else TOL16)
        for name, a, r in zip(("dq", "dk", "dv", "di", "df"), leaves, ref):
            assert torch.isfinite(a.grad).all(), name
            assert rel_err(np64(a.grad), r.grad.numpy()) < tol, name
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def test_backward_out_of_range_raises(ops):
    """Forget gates of exactly 0 cannot be split into chunk factors at any
    length: the backward says so instead of returning non-finite gradients."""
    from hybrid_model_mamba_xlstm_b200.kernels.tfla import tfla_bwd
    q, k, v, li, lf = _inputs((1, 1, 64, 128), 1.0, seed=45)
    lf[:, :, 10] = float("-inf")
    with pytest.raises(RuntimeError, match="out of range"):
        tfla_bwd.mlstm_chunkwise_bwd(q, k, v, li, lf, torch.randn_like(v))


# ------------------------------------------------------- long-context workload --
@pytest.mark.slow
def test_long_context_workload_sampled_heads(ops):
    """batch 8, heads 8, seqlen 32768, d_qk = d_v = 512, per-head gates with
    the config-2 distributions, bf16: all 64 (b, h) pairs run in one call;
    four of them are checked over the full 32768 steps against the fp32 C
    oracle, h and the final (C, n)."""
    from hybrid_model_mamba_xlstm_b200.workloads import mlstm_inputs
    from oracle import build as OC
    inp = mlstm_inputs(8, 8, 32768, 512, torch.bfloat16, seed=0, device="cuda", on_device=True)
    out, (C, n, m) = ops.mlstm_chunkwise_fwd(inp.q, inp.k, inp.v, inp.log_i, inp.log_f, return_state=True)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    pairs = [(0, 0), (3, 5), (6, 2), (7, 7)]
    sel = lambda t: torch.stack([t[b, h] for b, h in pairs])[None]  # (1, 4, ...)
    q, k, v = (np64(sel(t)).astype(np.float32) for t in (inp.q, inp.k, inp.v))
    ig = np.exp(np64(sel(inp.log_i))).astype(np.float32)
    fg = np.exp(np64(sel(inp.log_f))).astype(np.float32)
    hr, Cr, nr = OC.mlstm(q, k, v, ig, fg)
    em = np.exp(np64(sel(m)))
    for i, (b, h) in enumerate(pairs):
        assert rel_err(np64(out[b, h]), hr[0, i]) < TOL16, (b, h)
        assert rel_err(np64(C[b, h]) * em[0, i], Cr[0, i]) < TOL16, (b, h)
        assert rel_err(np64(n[b, h]) * em[0, i], nr[0, i]) < TOL16, (b, h)
