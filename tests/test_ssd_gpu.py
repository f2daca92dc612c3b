"""Mamba-2 SSD chunked scan (tcgen05) vs the oracle.

The reference has no SSD kernel; the oracle is its Euler selective-scan loop
(scan_interface.py:103-152) with head-repeated A and dt (oracle/numpy_ref.py
ssd_scan, pinned to the reference in test_oracle_golden.py).  bf16 I/O:
normwise relative error <= 2e-2 against the oracle on the same bf16 inputs.
"""
import numpy as np
import pytest
import torch

from oracle import numpy_ref as R
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
TOL16 = 2e-2


@pytest.fixture(scope="module")
def ssd():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from hybrid_model_mamba_xlstm_b200.kernels.ssd import ssd_chunk_scan
    return ssd_chunk_scan


def np64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("shape", [(1, 300, 4, 64, 128), (2, 256, 3, 128, 128), (1, 128, 2, 64, 256),
                                   (1, 77, 2, 96, 128)])
def test_ssd_parity_small(ssd, shape):
    from hybrid_model_mamba_xlstm_b200.workloads import ssd_inputs
    b, L, h, p, n = shape
    inp = ssd_inputs(b, L, h, p, n, seed=4, device="cuda")
    y, hT = ssd(inp.x, inp.dt, inp.A, inp.B, inp.C, inp.D)
    yr, hr = R.ssd_scan(np64(inp.x), np64(inp.dt), np64(inp.A), np64(inp.B), np64(inp.C), np64(inp.D))
    assert rel_err(np64(y), yr) < TOL16
    assert rel_err(np64(hT), hr) < TOL16


def test_ssd_bias_softplus_initial_state_and_strong_decay(ssd):
    """dt = softplus(raw + bias) inside the kernel, a nonzero initial state, and
    heads whose decay over one 128-step chunk spans e^-400 (the chunk-local
    exponents stay <= 0, nothing overflows)."""
    g = torch.Generator().manual_seed(8)
    b, L, h, p, n = 2, 400, 4, 64, 128
    x = torch.randn(b, L, h, p, generator=g).to("cuda", torch.bfloat16)
    Bm = torch.randn(b, L, n, generator=g).to("cuda", torch.bfloat16)
    Cm = torch.randn(b, L, n, generator=g).to("cuda", torch.bfloat16)
    raw = (torch.randn(b, L, h, generator=g) * 0.5).cuda()
    bias = torch.tensor([-4.0, -1.0, 0.5, 1.5]).cuda()
    A = -torch.tensor([1.0, 4.0, 16.0, 16.0]).cuda()
    D = torch.randn(h, generator=g).cuda()
    h0 = torch.randn(b, h, p, n, generator=g).cuda()
    y, hT = ssd(x, raw, A, Bm, Cm, D, dt_bias=bias, dt_softplus=True, initial_state=h0)
    yr, hr = R.ssd_scan(np64(x), np64(raw), np64(A), np64(Bm), np64(Cm), np64(D), dt_bias=np64(bias),
                        dt_softplus=True, h0=np64(h0))
    assert np.isfinite(np64(y)).all()
    assert rel_err(np64(y), yr) < TOL16
    assert rel_err(np64(hT), hr) < TOL16


def test_ssd_segmented_state(ssd):
    from hybrid_model_mamba_xlstm_b200.workloads import ssd_inputs
    inp = ssd_inputs(1, 512, 2, 64, 128, seed=6, device="cuda")
    y, hT = ssd(inp.x, inp.dt, inp.A, inp.B, inp.C, inp.D)
    s = 256
    y1, h1 = ssd(inp.x[:, :s], inp.dt[:, :s], inp.A, inp.B[:, :s], inp.C[:, :s], inp.D)
    y2, h2 = ssd(inp.x[:, s:], inp.dt[:, s:], inp.A, inp.B[:, s:], inp.C[:, s:], inp.D, initial_state=h1)
    assert rel_err(np64(torch.cat([y1, y2], 1)), np64(y)) < 1e-2
    assert rel_err(np64(h2), np64(hT)) < 1e-3


def test_ssd_full_workload_sampled_heads(ssd):
    """batch 8, heads 32, headdim 64, dstate 128, seqlen 4096: all heads run;
    heads 0 and 31 of batches 0 and 7 are checked against the C oracle."""
    from hybrid_model_mamba_xlstm_b200.workloads import ssd_inputs
    from oracle import build as OC
    inp = ssd_inputs(8, 4096, 32, 64, 128, seed=0, device="cuda")
    y, hT = ssd(inp.x, inp.dt, inp.A, inp.B, inp.C, inp.D)
    assert torch.isfinite(y).all()
    for bb in (0, 7):
        for hh in (0, 31):
            x = np64(inp.x[bb, :, hh]).T[None].astype(np.float32)  # (1, P, L)
            dt = np.repeat(np64(inp.dt[bb, :, hh])[None, None], 64, axis=1).astype(np.float32)
            A = np.full((64, 128), float(inp.A[hh]), np.float32)
            Bm = np64(inp.B[bb]).T[None].astype(np.float32)
            Cm = np64(inp.C[bb]).T[None].astype(np.float32)
            yr, hr = OC.scan(x, dt, A, Bm, Cm, np.ones(64, np.float32))
            assert rel_err(np64(y[bb, :, hh]).T[None], yr) < TOL16
            assert rel_err(np64(hT[bb, hh])[None], hr) < TOL16


def test_ssd_determinism(ssd):
    from hybrid_model_mamba_xlstm_b200.workloads import ssd_inputs
    inp = ssd_inputs(1, 300, 2, 64, 128, seed=1, device="cuda")
    a = ssd(inp.x, inp.dt, inp.A, inp.B, inp.C, inp.D)
    b2 = ssd(inp.x, inp.dt, inp.A, inp.B, inp.C, inp.D)
    assert torch.equal(a[0], b2[0]) and torch.equal(a[1], b2[1])
