"""Causal depthwise conv1d (+ SiLU) on the GPU vs the oracle and the reference's golden vectors.

Tolerances (normwise relative error): fp32 I/O 1e-5; bf16 I/O 1e-2 against the
float64 oracle on the same bf16-rounded inputs (one bf16 rounding of the output).
"""
import numpy as np
import pytest
import torch

from oracle import numpy_ref as R
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu

TOL32, TOL16 = 1e-5, 1e-2


@pytest.fixture(scope="module")
def conv():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from hybrid_model_mamba_xlstm_b200.kernels.conv import causal_conv1d
    return causal_conv1d


def np64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def test_golden_reference_block_fp32(conv, golden):
    g = golden("conv_block")
    x = torch.as_tensor(g["x_inner"]).cuda().float()
    out = conv(x, torch.as_tensor(g["weight"]).cuda(), torch.as_tensor(g["bias"]).cuda(), activation="silu")
    assert rel_err(np64(out), g["conv_silu"]) < TOL32


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("width", [1, 2, 3, 4])
@pytest.mark.parametrize("act", [None, "silu"])
def test_widths_and_activation(conv, dtype, width, act):
    g = torch.Generator().manual_seed(width)
    x = torch.randn(2, 100, 96, generator=g).to("cuda", dtype)
    w = torch.randn(96, 1, width, generator=g).cuda()      # nn.Conv1d weight shape
    b = torch.randn(96, generator=g).cuda()
    out = conv(x, w, b, activation=act)
    ref, _ = R.causal_conv1d(np64(x), np64(w), np64(b), activation=act)
    assert rel_err(np64(out), ref) < (TOL32 if dtype == torch.float32 else TOL16)


@pytest.mark.parametrize("layout", ["dense", "in_proj_half", "odd_channels", "time_major"])
def test_layouts(conv, layout):
    """Dense rows, the x half of an in_proj output (row stride 2*dim), channel
    counts that are not a multiple of the 16-byte vector (element kernel) and
    unit time stride (element kernel)."""
    g = torch.Generator().manual_seed(7)
    d = 130 if layout == "odd_channels" else 256
    xz = torch.randn(3, 77, 2 * d, generator=g).to("cuda", torch.bfloat16)
    x = {"dense": xz[..., :d].contiguous(), "in_proj_half": xz[..., :d], "odd_channels": xz[..., :d].contiguous(),
         "time_major": xz[..., :d].transpose(1, 2).contiguous().transpose(1, 2)}[layout]
    w = torch.randn(d, 4, generator=g).cuda()
    b = torch.randn(d, generator=g).cuda()
    out = conv(x, w, b, activation="silu")
    ref, _ = R.causal_conv1d(np64(x), np64(w), np64(b), activation="silu")
    assert rel_err(np64(out), ref) < TOL16


@pytest.mark.parametrize("L1", [0, 1, 2, 33, 64])
def test_continuation_with_state(conv, L1):
    """Two segments with the carried state give the one-pass result, and the
    final state is the last width-1 inputs (segments shorter than width-1 included)."""
    g = torch.Generator().manual_seed(11)
    x = torch.randn(2, 70, 64, generator=g).cuda()
    w = torch.randn(64, 4, generator=g).cuda()
    b = torch.randn(64, generator=g).cuda()
    whole, fin = conv(x, w, b, activation="silu", return_final_state=True)
    a, s = conv(x[:, :L1].contiguous(), w, b, activation="silu", return_final_state=True)
    c, fin2 = conv(x[:, L1:].contiguous(), w, b, activation="silu", initial_state=s, return_final_state=True)
    assert rel_err(np64(torch.cat([a, c], 1)), np64(whole)) < TOL32
    assert torch.equal(fin, fin2)
    assert torch.equal(fin, x[:, -3:].transpose(1, 2))


def test_large_matches_torch_conv(conv):
    """The hybrid-350M Mamba shape (batch 8, seqlen 2048, 2048 channels, bf16)
    against torch's own grouped conv in fp32 on the same inputs."""
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(8, 2048, 2048, device="cuda", generator=g).to(torch.bfloat16)
    w = torch.randn(2048, 1, 4, device="cuda", generator=g) * 0.5
    b = torch.randn(2048, device="cuda", generator=g) * 0.1
    out = conv(x, w, b, activation="silu")
    ref = torch.nn.functional.conv1d(x.float().transpose(1, 2), w, b, padding=3, groups=2048)[..., :2048]
    ref = torch.nn.functional.silu(ref).transpose(1, 2)
    assert float((out.float() - ref).norm() / ref.norm()) < TOL16


def test_empty_sequence_passes_state(conv):
    x = torch.zeros(2, 0, 32, device="cuda")
    w = torch.randn(32, 4, device="cuda")
    s0 = torch.randn(2, 32, 3, device="cuda")
    out, fin = conv(x, w, None, initial_state=s0, return_final_state=True)
    assert out.shape == (2, 0, 32) and torch.equal(fin, s0)
