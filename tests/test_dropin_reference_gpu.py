"""The drop-in boundary: the reference's own, unmodified layers on these kernels.

``hybrid_xmamba`` is installed unmodified into ``baseline/_ref`` (pip
--target, no dependencies), which travels with the repository.  The test
rebinds the two kernel names the reference's layers bind at import time, as
INTEGRATION.md describes:
  hybrid_xmamba.layers.mamba_block.selective_scan  (mamba_block.py:13, called at :123-125)
  hybrid_xmamba.layers.mlstm_block.apply_tfla      (mlstm_block.py:14, called at :129)
and then runs the reference's MambaBlock / mLSTMBlock classes themselves on
CUDA.  Their outputs must match the golden outputs the same reference
produced on CPU in float64 (fp32: normwise relative error 1e-4), and a bf16
block on the tensor-core path must match the reference block's own float64
loop on the same bf16-rounded weights and input (2e-2).
"""
import os
import sys

import numpy as np
import pytest
import torch

from tests.conftest import ROOT, rel_err

pytestmark = pytest.mark.gpu
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


@pytest.fixture(scope="module")
def ref():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    if not os.path.isdir(os.path.join(REF_DIR, "hybrid_xmamba")):
        pytest.skip("the reference is not installed in baseline/_ref (pip install --no-deps --target baseline/_ref)")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import hybrid_xmamba.layers.mamba_block as mb
    import hybrid_xmamba.layers.mlstm_block as lb
    from hybrid_model_mamba_xlstm_b200.kernels import apply_tfla, selective_scan
    calls = {"scan": 0, "tfla": 0}

    def scan(*a, **k):
        calls["scan"] += 1
        return selective_scan(*a, **k)

    def tfla(*a, **k):
        calls["tfla"] += 1
        return apply_tfla(*a, **k)
    saved = (mb.selective_scan, lb.apply_tfla)
    mb.selective_scan, lb.apply_tfla = scan, tfla
    yield mb, lb, calls
    mb.selective_scan, lb.apply_tfla = saved


def _state(g):
    return {k[3:]: torch.as_tensor(v) for k, v in g.items() if k.startswith("sd_")}


def np64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def test_reference_mamba_block_on_hxm_scan(ref, golden):
    mb, _, calls = ref
    g = golden("mamba_block")
    torch.manual_seed(0)
    blk = mb.MambaBlock(64, state_size=16)
    blk.load_state_dict(_state(g))
    blk = blk.cuda().float()
    n0 = calls["scan"]
    with torch.no_grad():
        out = blk(torch.as_tensor(g["x"], dtype=torch.float32).cuda())
    out = out[0] if isinstance(out, tuple) else out
    assert calls["scan"] == n0 + 1  # the reference block called the rebound kernel
    assert rel_err(np64(out), g["out"]) < 1e-4


def test_reference_mlstm_block_on_hxm_tfla(ref, golden):
    _, lb, calls = ref
    g = golden("mlstm_block")
    torch.manual_seed(0)
    blk = lb.mLSTMBlock(64, head_dim=32, num_heads=2)
    blk.load_state_dict(_state(g), strict=False)
    blk = blk.cuda().float()
    n0 = calls["tfla"]
    with torch.no_grad():
        out = blk(torch.as_tensor(g["x"], dtype=torch.float32).cuda())
    assert calls["tfla"] == n0 + 1
    assert rel_err(np64(out), g["out"]) < 1e-4


def test_reference_mlstm_block_bf16_tensor_core_path(ref):
    """The reference mLSTMBlock with head_dim 128 in bf16 on CUDA: apply_tfla
    gets per-channel gates and runs the key-streaming tcgen05 kernel.  Checked
    against the same block in float64 on CPU running the reference's own loop
    (tfla_forward_pytorch), with the rebinding undone for that run."""
    _, lb, calls = ref
    torch.manual_seed(5)
    blk = lb.mLSTMBlock(256, head_dim=128, num_heads=2).double()
    with torch.no_grad():
        for p in blk.parameters():
            p.copy_(torch.randn_like(p).mul_(0.05).to(torch.bfloat16).double())
    x = torch.randn(2, 160, 256).to(torch.bfloat16).double()
    mine = lb.apply_tfla
    import hybrid_xmamba.kernels.tfla.tfla_interface as ti
    lb.apply_tfla = ti.apply_tfla  # the reference's own path, float64 on CPU
    try:
        with torch.no_grad():
            want = blk(x)
    finally:
        lb.apply_tfla = mine
    n0 = calls["tfla"]
    with torch.no_grad():
        got = blk.to("cuda", torch.bfloat16)(x.to("cuda", torch.bfloat16))
    assert calls["tfla"] == n0 + 1
    assert rel_err(np64(got), want.numpy()) < 2e-2
