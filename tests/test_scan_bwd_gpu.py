"""Selective-scan backward kernel vs autograd of the reference loop.

The reference's backward (scan_interface.py:62-100) re-runs
selective_scan_pytorch (:103-152) under autograd; the check here does the
same in float64 on the same inputs and compares every gradient.  Tolerances
(normwise relative error): fp32 I/O 1e-4 (fp32 state and sums in the kernel,
atomics in a different order); bf16 I/O 2e-2.
"""
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def S():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from hybrid_model_mamba_xlstm_b200.kernels.selective_scan import scan_interface as si
    return si


def _loop(x, dt, A, B, C, D, z=None, z_mode="mul", bias=None, softplus=False):
    """float64 restatement of selective_scan_pytorch (+ the fused softplus / gate options)."""
    bsz, L, dm = x.shape
    if bias is not None:
        dt = dt + bias
    if softplus:
        dt = torch.nn.functional.softplus(dt)
    h = torch.zeros(bsz, dm, A.shape[1], dtype=x.dtype, device=x.device)
    ys = []
    for t in range(L):
        h = torch.exp(A[None] * dt[:, t, :, None]) * h + (dt[:, t] * x[:, t])[..., None] * B[:, t, None]
        ys.append((h * C[:, t, None]).sum(-1) + D * x[:, t])
    y = torch.stack(ys, 1)
    if z is not None:
        y = y * z if z_mode == "mul" else y * z * torch.sigmoid(z)
    return y


def np64(t):
    return t.detach().double().cpu().numpy()


def _inputs(b, L, dm, n, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(b, L, dm, generator=g)
    dt = torch.nn.functional.softplus(torch.randn(b, L, dm, generator=g) - 2.0)
    A = -torch.exp(torch.randn(dm, n, generator=g) * 0.5)
    B = torch.randn(b, L, n, generator=g)
    C = torch.randn(b, L, n, generator=g)
    D = torch.randn(dm, generator=g)
    z = torch.randn(b, L, dm, generator=g)
    go = torch.randn(b, L, dm, generator=g)
    return [t.to(dtype) for t in (x, dt)] + [A] + [t.to(dtype) for t in (B, C)] + [D, z.to(dtype), go.to(dtype)]


# (2, 24, 4790, 16): a grid of at least one CTA per SM at two lanes per channel, so the
# kernel keeps 64-channel CTAs (the smaller shapes run four lanes per channel); ragged dim
@pytest.mark.parametrize("shape", [(2, 37, 70, 16), (1, 64, 128, 8), (3, 5, 33, 16), (2, 24, 4790, 16)])
@pytest.mark.parametrize("with_z", [False, True])
def test_reference_api_gradients_fp32(S, shape, with_z):
    x, dt, A, B, C, D, z, go = _inputs(*shape, seed=sum(shape), dtype=torch.float32)
    z = z if with_z else None
    ins = [t.cuda().requires_grad_(True) for t in (x, dt, A, B, C, D)]
    zc = z.cuda().requires_grad_(True) if with_z else None
    y = S.selective_scan(*ins, z=zc)
    y.backward(go.cuda())
    ref_ins = [t.double().requires_grad_(True) for t in (x, dt, A, B, C, D)]
    zr = z.double().requires_grad_(True) if with_z else None
    yr = _loop(*ref_ins, z=zr)
    yr.backward(go.double())
    assert rel_err(np64(y), np64(yr)) < 1e-5
    for got, ref in zip(ins + ([zc] if with_z else []), ref_ins + ([zr] if with_z else [])):
        assert rel_err(np64(got.grad), np64(ref.grad)) < 1e-4


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fused_entry_gradients_softplus_bias_silu(S, dtype):
    """selective_scan_fn in (batch, dim, seqlen) layout with softplus(delta + bias)
    and y * silu(z): gradients of u, delta, A, B, C, D, z and the bias."""
    x, dt, A, B, C, D, z, go = _inputs(2, 50, 64, 16, seed=9, dtype=dtype)
    raw = (torch.log(torch.expm1(dt.float())) - 0.3).to(dtype)
    bias = torch.full((64,), 0.3)
    t = lambda a: a.transpose(1, 2).contiguous()
    ins = {"u": t(x), "delta": t(raw), "A": A, "B": t(B), "C": t(C), "D": D, "z": t(z), "delta_bias": bias}
    cu = {k: v.cuda().requires_grad_(True) for k, v in ins.items()}
    y = S.selective_scan_fn(cu["u"], cu["delta"], cu["A"], cu["B"], cu["C"], cu["D"], z=cu["z"],
                            delta_bias=cu["delta_bias"], delta_softplus=True)
    y.backward(t(go).cuda())
    rf = {k: v.double().requires_grad_(True) for k, v in ins.items()}
    tb = lambda a: a.transpose(1, 2)
    yr = _loop(tb(rf["u"]), tb(rf["delta"]), rf["A"], tb(rf["B"]), tb(rf["C"]), rf["D"], z=tb(rf["z"]),
               z_mode="silu", bias=rf["delta_bias"], softplus=True)
    yr.backward(go.double())
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    for k in ins:
        assert rel_err(np64(cu[k].grad), np64(rf[k].grad)) < tol, k


def test_empty_sequence_zero_gradients(S):
    x = torch.zeros(2, 0, 8, device="cuda", requires_grad=True)
    A = (-torch.ones(8, 4, device="cuda")).requires_grad_(True)
    B = torch.zeros(2, 0, 4, device="cuda", requires_grad=True)
    D = torch.ones(8, device="cuda", requires_grad=True)
    y = S.selective_scan(x, x, A, B, B, D)
    y.sum().backward()
    assert float(A.grad.abs().sum()) == 0.0 and float(D.grad.abs().sum()) == 0.0


def _loop_h0(x, dt, A, B, C, D, h0):
    """The loop of _loop started from a state h0 (the continuation of an earlier segment)."""
    h = h0
    ys = []
    for t in range(x.shape[1]):
        h = torch.exp(A[None] * dt[:, t, :, None]) * h + (dt[:, t] * x[:, t])[..., None] * B[:, t, None]
        ys.append((h * C[:, t, None]).sum(-1) + D * x[:, t])
    return torch.stack(ys, 1)


def test_fused_entry_initial_state_gradient(S):
    """selective_scan_fn with initial_state under autograd: the gradient of the
    initial state (and of every input) against float64 autograd of the loop."""
    x, dt, A, B, C, D, z, go = _inputs(2, 40, 32, 16, seed=13, dtype=torch.float32)
    h0 = torch.randn(2, 32, 16, generator=torch.Generator().manual_seed(14))
    t = lambda a: a.transpose(1, 2).contiguous()
    ins = {"u": t(x), "delta": t(dt), "A": A, "B": t(B), "C": t(C), "D": D, "h0": h0}
    cu = {k: v.cuda().requires_grad_(True) for k, v in ins.items()}
    y = S.selective_scan_fn(cu["u"], cu["delta"], cu["A"], cu["B"], cu["C"], cu["D"], initial_state=cu["h0"])
    y.backward(t(go).cuda())
    rf = {k: v.double().requires_grad_(True) for k, v in ins.items()}
    tb = lambda a: a.transpose(1, 2)
    yr = _loop_h0(tb(rf["u"]), tb(rf["delta"]), rf["A"], tb(rf["B"]), tb(rf["C"]), rf["D"], rf["h0"])
    yr.backward(go.double())
    for k in ins:
        assert rel_err(np64(cu[k].grad), np64(rf[k].grad)) < 1e-4, k


def test_fused_entry_refuses_what_it_cannot_differentiate(S):
    """Under autograd, asking for the (non-differentiable) final state or the
    ZOH rule raises instead of returning outputs with no gradient path."""
    x, dt, A, B, C, D, z, go = _inputs(1, 8, 32, 16, seed=15, dtype=torch.float32)
    t = lambda a: a.transpose(1, 2).contiguous().cuda()
    u = t(x).requires_grad_(True)
    with pytest.raises(NotImplementedError):
        S.selective_scan_fn(u, t(dt), A.cuda(), t(B), t(C), D.cuda(), return_last_state=True)
    with pytest.raises(NotImplementedError):
        S.selective_scan_fn(u, t(dt), A.cuda(), t(B), t(C), D.cuda(), discretization="zoh")
    with torch.no_grad():
        y, h = S.selective_scan_fn(u, t(dt), A.cuda(), t(B), t(C), D.cuda(), return_last_state=True)
    assert y.shape == u.shape and h.shape == (1, 32, 16)
