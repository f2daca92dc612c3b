"""RMSNorm (and the fused residual add + RMSNorm) on the GPU vs the oracle.

Tolerances (normwise relative error): fp32 I/O 1e-5; bf16 I/O 1e-2 against the
float64 oracle on the same bf16-rounded inputs (the bf16 sum is rounded once,
as the reference's bf16 residual stream is).
"""
import numpy as np
import pytest
import torch

from oracle import numpy_ref as R
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu

TOL32, TOL16 = 1e-5, 1e-2


@pytest.fixture(scope="module")
def norm():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from hybrid_model_mamba_xlstm_b200.kernels.norm import rmsnorm
    return rmsnorm


def np64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("dim", [8, 64, 256, 1000, 1024, 4096, 8192])
def test_rmsnorm(norm, dtype, dim):
    g = torch.Generator().manual_seed(dim)
    x = (torch.randn(3, 37, dim, generator=g) * 2).to("cuda", dtype)
    w = torch.randn(dim, generator=g).cuda()
    y = norm(x, w, 1e-6)
    ref = R.rmsnorm(np64(x), np64(w), 1e-6)
    assert rel_err(np64(y), ref) < (TOL32 if dtype == torch.float32 else TOL16)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fused_residual_add(norm, dtype):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(4, 50, 1024, generator=g).to("cuda", dtype)
    r = torch.randn(4, 50, 1024, generator=g).to("cuda", dtype)
    w = torch.randn(1024, generator=g).cuda()
    y, s = norm(x, w, 1e-6, residual=r, return_sum=True)
    assert torch.equal(s, x + r)                       # the io-dtype sum, exactly torch's add
    ref = R.rmsnorm(np64(x + r), np64(w), 1e-6)
    assert rel_err(np64(y), ref) < (TOL32 if dtype == torch.float32 else TOL16)


def test_strided_rows_and_no_weight(norm):
    """Rows of a wider buffer (row stride > dim) and weight None (ones)."""
    g = torch.Generator().manual_seed(2)
    big = torch.randn(64, 3 * 512, generator=g).cuda().to(torch.bfloat16)
    x = big[:, 512:1024]
    y = norm(x, None, 1e-5)
    ref = R.rmsnorm(np64(x), np.ones(512), 1e-5)
    assert rel_err(np64(y), ref) < TOL16


def test_module_matches_reference_formula(norm):
    """The layer module against the reference formula w * x / sqrt(mean(x^2) + eps) in fp32."""
    from hybrid_model_mamba_xlstm_b200.layers import RMSNorm
    m = RMSNorm(256).cuda()
    with torch.no_grad():
        m.weight.normal_()
    x = torch.randn(8, 10, 256, device="cuda")
    ref = m.weight * (x / torch.sqrt(torch.mean(x ** 2, dim=-1, keepdim=True) + m.eps))
    assert float((m(x) - ref).norm() / ref.norm()) < TOL32
