"""sLSTM recurrence on the GPU vs the reference block's golden vectors and the oracle.

fp32 gates: normwise relative error <= 1e-5 (hd 16: one-CTA kernel) or
2e-3 (cluster kernel: the recurrent matvec runs in bf16 on the tensor cores);
bf16 gates: <= 2e-2 against the float64 oracle on the same bf16 inputs.
"""
import numpy as np
import pytest
import torch

from oracle import numpy_ref as R
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def slstm():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from hybrid_model_mamba_xlstm_b200.kernels.slstm import slstm_scan
    return slstm_scan


def np64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def test_golden_reference_block(slstm, golden):
    """Gate pre-activations captured from the reference sLSTMBlock (R absent)."""
    g = golden("slstm_block")
    nh, hd = int(g["heads"]), int(g["head_dim"])
    bsz, L, _ = g["gates"].shape
    gates = torch.as_tensor(g["gates"].reshape(bsz, L, nh, 4, hd), dtype=torch.float32).cuda()
    out, (h, c) = slstm(gates, torch.as_tensor(g["norm_w"], dtype=torch.float32).cuda())
    assert rel_err(np64(out).reshape(bsz, L, nh * hd), g["h_seq"]) < 1e-5
    assert rel_err(np64(h), g["h"]) < 1e-5
    assert rel_err(np64(c), g["c"]) < 1e-5


def _inputs(b, L, nh, hd, seed, dtype, with_R=True, scale=1.0):
    gen = torch.Generator().manual_seed(seed)
    gates = (torch.randn(b, L, nh, 4, hd, generator=gen) * scale).to("cuda", dtype)
    w = (1.0 + 0.1 * torch.randn(hd, generator=gen)).cuda()
    Rm = (torch.randn(nh, hd, 4 * hd, generator=gen) / hd ** 0.5).to("cuda", torch.bfloat16) if with_R else None
    return gates, w, Rm


@pytest.mark.parametrize("b,L,nh,hd,dtype", [(2, 64, 4, 128, torch.float32), (3, 100, 2, 256, torch.float32),
                                             (8, 256, 4, 256, torch.bfloat16), (1, 50, 1, 128, torch.bfloat16),
                                             (11, 40, 2, 128, torch.bfloat16), (2, 30, 2, 64, torch.float32)])
def test_recurrent_R_parity(slstm, b, L, nh, hd, dtype):
    """Block-diagonal recurrent weights R ~ N(0, 1/hd) (head_dim 128/256 run
    the 8-CTA cluster kernel; batch > 8 uses several clusters)."""
    gates, w, Rm = _inputs(b, L, nh, hd, 7, dtype)
    out, (h, c) = slstm(gates, w, R=Rm)
    ref, hr, cr = R.slstm_recurrent(np64(gates), np64(w), R=np64(Rm))
    tol = 2e-3 if dtype == torch.float32 and hd > 64 else (1e-5 if dtype == torch.float32 else 2e-2)
    assert rel_err(np64(out), ref) < tol
    assert rel_err(np64(h), hr) < tol
    assert rel_err(np64(c), cr) < tol


@pytest.mark.parametrize("hd", [16, 256])
def test_initial_state_and_segments(slstm, hd):
    gates, w, Rm = _inputs(2, 90, 2, hd, 3, torch.float32, with_R=hd > 16)
    out, (h, c) = slstm(gates, w, R=Rm)
    a, (h1, c1) = slstm(gates[:, :37], w, R=Rm)
    b2, (h2, c2) = slstm(gates[:, 37:], w, R=Rm, h0=h1, c0=c1)
    tol = 1e-5 if hd == 16 else 2e-3
    assert rel_err(np64(torch.cat([a, b2], 1)), np64(out)) < tol
    assert rel_err(np64(c2), np64(c)) < tol


def test_large_input_gates_stay_finite(slstm):
    """exp input gate with pre-activations ~ +60: the reference's fp32 cell
    would overflow; the per-channel stabilizer keeps h exact (RMSNorm is
    scale-invariant) and finite."""
    gates, w, _ = _inputs(1, 50, 2, 32, 4, torch.float32)
    gates[:, :, :, 0] += 60.0
    out, (h, c) = slstm(gates, w)
    ref, hr, _ = R.slstm_recurrent(np64(gates), np64(w))
    assert np.isfinite(np64(out)).all()
    assert rel_err(np64(out), ref) < 1e-5


def test_sigmoid_input_gate(slstm):
    gates, w, Rm = _inputs(2, 40, 2, 128, 5, torch.float32)
    out, _ = slstm(gates, w, R=Rm, exponential_gate=False)
    ref, _, _ = R.slstm_recurrent(np64(gates), np64(w), R=np64(Rm), exponential_gate=False)
    assert rel_err(np64(out), ref) < 2e-3


def test_prefill_sized_sampled(slstm):
    """batch 8, seqlen 2048, 4 heads x 256 (the hybrid prefill's sLSTM layer),
    checked against the C oracle on all heads of batch rows 0 and 7."""
    from oracle import build as OC
    gates, w, Rm = _inputs(8, 2048, 4, 256, 11, torch.bfloat16, scale=0.5)
    out, (h, c) = slstm(gates, w, R=Rm)
    assert torch.isfinite(out).all()
    for bb in (0, 7):
        ref, hr, cr = OC.slstm(np64(gates[bb:bb + 1]), np64(w), R=np64(Rm))
        assert rel_err(np64(out[bb:bb + 1]), ref) < 2e-2
        assert rel_err(np64(c[bb:bb + 1]), cr) < 2e-2


@pytest.mark.parametrize("b,hd,dtype", [(1, 256, torch.bfloat16), (3, 128, torch.float32), (4, 256, torch.bfloat16)])
def test_two_heads_per_cluster_matches_one(slstm, b, hd, dtype, monkeypatch):
    """Batches of at most 4 rows run two heads per 8-CTA cluster (half the SMs):
    each (head, row) slot takes the same MMA chain, norm and exchanges as with
    one head per cluster, so outputs and final states agree bitwise; both also
    match the oracle."""
    gates, w, Rm = _inputs(b, 70, 4, hd, 11, dtype)
    gen = torch.Generator().manual_seed(5)
    h0 = (0.5 * torch.randn(b, 4, hd, generator=gen)).cuda()
    c0 = torch.randn(b, 4, hd, generator=gen).cuda()
    res = []
    for hpc in ("1", "2"):
        monkeypatch.setenv("HXM_SLSTM_HPC", hpc)
        out, (h, c) = slstm(gates, w, R=Rm, h0=h0, c0=c0)
        torch.cuda.synchronize()
        res.append((out.clone(), h.clone(), c.clone()))
    for x, y in zip(*res):
        assert torch.equal(x, y)
    ref, hr, cr = R.slstm_recurrent(np64(gates), np64(w), R=np64(Rm), h0=np64(h0), c0=np64(c0))
    tol = 2e-3 if dtype == torch.float32 else 2e-2
    assert rel_err(np64(res[1][0]), ref) < tol
    assert rel_err(np64(res[1][2]), cr) < tol
