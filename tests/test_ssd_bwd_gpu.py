"""SSD chunked-scan backward vs float64 autograd of the SSD recurrence.

The reference has no SSD; its arithmetic is the Euler selective scan
(scan_interface.py:103-152) with channel d = (head, p), per-head A and dt and
B, C shared by the heads.  The check differentiates that loop in float64 on
the same (bf16-rounded) inputs and compares every gradient of
ssd_chunk_scan_fn.  Tolerance (normwise relative error): 2e-2 for the bf16
forward's gradients in fp32 arithmetic, 1e-4 for the fp32 backward entry
given the float64 loop's own cotangent (full-fp32 chunk GEMMs; the bf16
path's default TF32 GEMMs add ~1e-3).
"""
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def S():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    torch.backends.cuda.matmul.allow_tf32 = False
    from hybrid_model_mamba_xlstm_b200.kernels import ssd
    return ssd


def _loop(x, dt, A, B, C, D, dt_bias, softplus):
    """float64 SSD: h[p, n] = exp(dt A) h + dt x[p] B[n];  y[p] = C . h[p, :] + D x[p]."""
    if dt_bias is not None:
        dt = dt + dt_bias
    if softplus:
        dt = torch.nn.functional.softplus(dt)
    bsz, L, nh, p = x.shape
    h = torch.zeros(bsz, nh, p, B.shape[-1], dtype=x.dtype)
    ys = []
    for t in range(L):
        a = torch.exp(dt[:, t] * A)                                   # (b, H)
        h = a[..., None, None] * h + (dt[:, t, :, None] * x[:, t])[..., None] * B[:, t, None, None, :]
        ys.append((h * C[:, t, None, None, :]).sum(-1) + D[None, :, None] * x[:, t])
    return torch.stack(ys, 1)


def _inputs(bsz, L, nh, p, n, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(bsz, L, nh, p, generator=g).bfloat16()
    dt = torch.randn(bsz, L, nh, generator=g) * 0.5
    bias = torch.log(torch.expm1(torch.exp(torch.empty(nh).uniform_(-6.9, -2.3, generator=g))))  # softplus^-1 of dt in [1e-3, 1e-1]
    A = -torch.empty(nh).uniform_(1.0, 16.0, generator=g)
    B = torch.randn(bsz, L, n, generator=g).bfloat16()
    C = torch.randn(bsz, L, n, generator=g).bfloat16()
    D = torch.randn(nh, generator=g)
    dy = torch.randn(bsz, L, nh, p, generator=g)
    return x, dt, A, B, C, D, bias, dy


@pytest.mark.parametrize("shape", [(2, 100, 4, 32, 128), (1, 64, 2, 64, 128), (2, 7, 3, 32, 128)])
def test_ssd_grads_vs_float64_loop(S, shape):
    x, dt, A, B, C, D, bias, dy = _inputs(*shape, seed=sum(shape))
    cu = [t.cuda().requires_grad_(True) for t in (x, dt, A, B, C, D, bias)]
    y = S.ssd_chunk_scan_fn(cu[0], cu[1], cu[2], cu[3], cu[4], cu[5], dt_bias=cu[6], dt_softplus=True)
    y.backward(dy.cuda().bfloat16())
    ref = [t.detach().double().requires_grad_(True) for t in (x, dt, A, B, C, D, bias)]
    yr = _loop(*ref, True)
    yr.backward(dy.bfloat16().double())
    assert rel_err(y.detach().double().cpu().numpy(), yr.detach().numpy()) < 2e-2
    for name, a, b in zip(("dx", "ddt", "dA", "dB", "dC", "dD", "ddt_bias"), cu, ref):
        assert rel_err(a.grad.double().cpu().numpy(), b.grad.numpy()) < 2e-2, name


def test_ssd_bwd_entry_fp32_exact_and_large_decay(S):
    """ssd_chunk_scan_bwd in fp32 against the float64 loop's gradients for the
    same cotangent, with dt up to ~3 and A down to -16: per-step log decays of
    ~-50 (chunk totals far beyond any separable scaling), exact form."""
    bsz, L, nh, p, n = 1, 150, 3, 16, 32
    x, dt, A, B, C, D, _, dy = _inputs(bsz, L, nh, p, n, seed=9)
    dt = dt * 4.0
    ref = [t.double().requires_grad_(True) for t in (x, dt, A, B, C, D)]
    yr = _loop(*ref, None, True)
    yr.backward(dy.double())
    got = S.ssd_chunk_scan_bwd(x.cuda(), dt.cuda(), A.cuda(), B.cuda(), C.cuda(), D.cuda(), dy.cuda(),
                               dt_softplus=True, chunk=64, tf32=False)
    for name, a, b in zip(("dx", "ddt", "dA", "dB", "dC", "dD"), got, ref):
        assert torch.isfinite(a).all(), name
        assert rel_err(a.double().cpu().numpy(), b.grad.numpy()) < 1e-4, name


@pytest.mark.parametrize("c", [32, 64])
def test_ssd_bwd_intra_kernel_vs_formulas(S, c):
    """hxm_ssd_bwd_intra (one block per (batch, chunk), the head sum on chip)
    against the torch formulas of its outputs: S_h, M, dL/d dt and dL/d b."""
    g = torch.Generator().manual_seed(c)
    bsz, nch, nh = 2, 3, 5
    cb = torch.randn(bsz, nch, c, c, generator=g)
    bcum = (-torch.rand(bsz, nch, c, nh, generator=g)).cumsum(2)
    dt = torch.rand(bsz, nch, c, nh, generator=g)
    G = torch.randn(bsz, nch, nh, c, c, generator=g)
    got = S._intra(cb.cuda(), bcum.cuda(), dt.cuda(), G.cuda(), torch.cuda.current_stream().cuda_stream)
    bh = bcum.permute(0, 1, 3, 2)
    causal = torch.ones(c, c, dtype=torch.bool).tril()
    Lm = torch.exp((bh.unsqueeze(-1) - bh.unsqueeze(-2)).masked_fill(~causal, float("-inf")))
    ds = dt.permute(0, 1, 3, 2).unsqueeze(-2)
    V = G * Lm * cb.unsqueeze(2)
    W = V * ds * (~torch.eye(c, dtype=torch.bool))
    want = (cb.unsqueeze(2) * Lm * ds, (G * Lm * ds).sum(2), V.sum(-2), W.sum(-1) - W.sum(-2))
    for name, a, b in zip(("S", "M", "ddt", "db"), got, want):
        assert rel_err(a.double().cpu().numpy(), b.double().numpy()) < 1e-5, name


def test_ssd_bwd_chunk32_ragged_matches_chunk64(S):
    """32-step chunks (the intra kernel's other tile) on a ragged length give the
    gradients of 64-step chunks and of the float64 loop."""
    x, dt, A, B, C, D, bias, dy = _inputs(1, 77, 3, 32, 128, seed=12)
    cu = lambda t: t.cuda()
    g32 = S.ssd_chunk_scan_bwd(*map(cu, (x, dt, A, B, C, D, dy)), dt_bias=cu(bias), dt_softplus=True, chunk=32,
                               tf32=False)
    g64 = S.ssd_chunk_scan_bwd(*map(cu, (x, dt, A, B, C, D, dy)), dt_bias=cu(bias), dt_softplus=True, chunk=64,
                               tf32=False)
    ref = [t.double().requires_grad_(True) for t in (x, dt, A, B, C, D, bias)]
    _loop(*ref, True).backward(dy.double())
    for name, a, b, r in zip(("dx", "ddt", "dA", "dB", "dC", "dD", "ddt_bias"), g32, g64, ref):
        assert rel_err(a.double().cpu().numpy(), b.double().cpu().numpy()) < 1e-5, name
        assert rel_err(a.double().cpu().numpy(), r.grad.numpy()) < 1e-4, name


@pytest.mark.parametrize("precise,chunk", [(True, 64), (False, 64), (True, 32)])
def test_ssd_bwd_tensor_cores_match_library_path(S, precise, chunk):
    """The tcgen05 chunk-GEMM backward (bf16 x, B, C; split operands) against
    the fp32 library-GEMM path on the same inputs (batch 2, 300 steps, 8 heads
    x 64, dstate 128): every gradient within 1e-3 (precise; measured 2.5e-4
    on dA, a sum over every step and channel) or 2e-2 (high parts only, the
    class of TF32 GEMMs; 7e-3 measured on ddt_bias)."""
    x, dt, A, B, C, D, bias, dy = _inputs(2, 300, 8, 64, 128, seed=chunk + int(precise))
    args = [t.cuda() for t in (x, dt, A, B, C, D)] + [dy.cuda().bfloat16()]
    kw = dict(dt_bias=bias.cuda(), dt_softplus=True, chunk=chunk)
    tc = S.ssd_chunk_scan_bwd(*args, **kw, tensor_cores=True, precise=precise)
    lib = S.ssd_chunk_scan_bwd(*args, **kw, tensor_cores=False, tf32=False)
    for name, a, b in zip(("dx", "ddt", "dA", "dB", "dC", "dD", "ddt_bias"), tc, lib):
        assert torch.isfinite(a).all(), name
        assert rel_err(a.double().cpu().numpy(), b.double().cpu().numpy()) < (1e-3 if precise else 2e-2), name
