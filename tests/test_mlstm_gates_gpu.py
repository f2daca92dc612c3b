"""mLSTM gate prologue / epilogue kernels vs the reference's element-wise
formulas (mlstm_block.py:117-119,138-141) computed in float64 on the same inputs.

Tolerances (normwise relative error): fp32 1e-6; bf16 1e-2 (one bf16 rounding
of the epilogue output)."""
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def G():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from hybrid_model_mamba_xlstm_b200.kernels.tfla import gates
    return gates


def np64(t):
    return t.detach().double().cpu().numpy()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("dim", [1000, 2048, 7])
def test_prologue_and_epilogue_on_projection_views(G, dtype, dim):
    g = torch.Generator(device="cuda").manual_seed(dim)
    ifo = (torch.randn(2, 33, 3 * dim, device="cuda", generator=g) * 3).to(dtype)   # one fused GEMM output
    i_pre, f_pre, o_pre = ifo[..., :dim], ifo[..., dim:2 * dim], ifo[..., 2 * dim:]
    li, lf = G.mlstm_gate_prologue(i_pre, f_pre)
    assert li.dtype == torch.float32 and li.shape == (2, 33, dim)
    assert torch.equal(li, i_pre.float())
    ref_f = torch.nn.functional.logsigmoid(f_pre.double())
    assert rel_err(np64(lf), np64(ref_f)) < (1e-6 if dtype == torch.float32 else 1e-5)
    h = torch.randn(2, 33, dim, device="cuda", generator=g).to(dtype)
    xg = torch.randn(2, 33, dim, device="cuda", generator=g).to(dtype)
    out = G.mlstm_gate_epilogue(h, o_pre, xg)
    ref = h.double() * torch.sigmoid(o_pre.double()) * torch.sigmoid(xg.double())
    assert out.dtype == dtype
    assert rel_err(np64(out), np64(ref)) < (1e-6 if dtype == torch.float32 else 1e-2)


def test_empty_rows(G):
    x = torch.zeros(0, 16, device="cuda")
    li, lf = G.mlstm_gate_prologue(x, x)
    assert li.shape == (0, 16)
    assert G.mlstm_gate_epilogue(x, x, x).shape == (0, 16)
