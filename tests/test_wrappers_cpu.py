"""Host-side helpers of the kernel wrappers (no GPU needed)."""
import torch

from hybrid_model_mamba_xlstm_b200.kernels._common import f32_param


def test_f32_param_reuses_the_copy_until_the_parameter_changes():
    """A bf16 parameter's fp32 copy is made once and reused while the parameter
    is unchanged; an in-place update (a new version) or a new tensor gives a
    fresh copy; fp32 contiguous tensors pass through; with autograd recording
    for the parameter the cast is differentiable, not cached."""
    p = torch.nn.Parameter(torch.randn(64).to(torch.bfloat16), requires_grad=False)
    a = f32_param(p)
    assert a.dtype == torch.float32 and torch.equal(a, p.float())
    assert f32_param(p) is a
    with torch.no_grad():
        p.add_(1)
    b = f32_param(p)
    assert b is not a and torch.equal(b, p.float())
    f = torch.randn(8)
    assert f32_param(f) is f
    q = torch.nn.Parameter(torch.randn(8).to(torch.bfloat16))
    c = f32_param(q)
    assert c.requires_grad and c.grad_fn is not None
    assert f32_param(None) is None
