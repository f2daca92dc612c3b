"""hxm_mlstm_chunkwise_fwd_noalloc: the mLSTM forward for callers that cannot
allocate device memory at call time (plugin hosts whose execute callbacks
forbid cudaMalloc, programs that own all device memory).  It takes no
workspace; its scratch is a fixed 32 MiB device array inside the library.

The GPU test calls it through the C ABI twice in a row per case (different
inputs, so the shared scratch is reused) and checks each result:
  * against the regular entry point, which gets a caller-allocated
    workspace: bitwise where both run the same kernels (the key-streaming
    kernel, and the recurrent kernel for (b, h) pairs out of its range);
  * against the float64 oracle at the bf16 tolerance used throughout
    (normwise relative error <= 2e-2), final states included — the only
    check for per-head gates at dqk 128 / 256, where the regular entry point
    takes the tcgen05 chunkwise kernel instead.
This file is collected last.
"""
import ctypes as ct

import numpy as np
import pytest
import torch

from hybrid_model_mamba_xlstm_b200 import _lib
from tests.conftest import rel_err


def _args(q, k, v, li, lf, h, CT=None, nT=None, mT=None, C0=None, n0=None, m0=None):
    a = _lib.MlstmArgs()
    b, nh, L, d = q.shape
    a.batch, a.heads, a.seqlen, a.dqk, a.dv = b, nh, L, d, v.shape[-1]
    a.chunk, a.gate_mode, a.io_dtype = 128, 1 if li.dim() == 4 else 0, _lib.HXM_BF16
    a.q, a.q_stride = q.data_ptr(), q.stride()[:2]
    a.k, a.k_stride = k.data_ptr(), k.stride()[:2]
    a.v, a.v_stride = v.data_ptr(), v.stride()[:2]
    a.log_i, a.i_stride = li.data_ptr(), li.stride()[:2]
    a.log_f, a.f_stride = lf.data_ptr(), lf.stride()[:2]
    a.h, a.h_stride = h.data_ptr(), h.stride()[:2]
    for name, t in (("CT", CT), ("nT", nT), ("mT", mT), ("C0", C0), ("n0", n0), ("m0", m0)):
        setattr(a, name, None if t is None else t.data_ptr())
    a.struct_size = ct.sizeof(a)
    return a


def test_noalloc_rejects_oversized_request_without_a_gpu():
    a = _lib.MlstmArgs()
    a.batch, a.heads, a.seqlen, a.dqk, a.dv = 8, 8, 32768, 512, 512  # needs ~1.6 GB of scratch
    a.chunk, a.gate_mode, a.io_dtype = 128, 0, _lib.HXM_BF16
    fake = 1 << 20  # aligned non-null placeholders: the size check fails before any pointer is used
    for f in ("q", "k", "v", "log_i", "log_f", "h"):
        setattr(a, f, fake)
    a.q_stride = a.k_stride = a.v_stride = a.h_stride = (8 * 32768 * 512, 32768 * 512)
    a.struct_size = ct.sizeof(a)
    st = _lib.lib().hxm_mlstm_chunkwise_fwd_noalloc(ct.byref(a), None)
    assert st == _lib.HXM_EBADARG
    assert b"32 MiB" in _lib.lib().hxm_last_error_string()


def test_noalloc_applies_the_regular_argument_checks_without_a_gpu():
    """The same checks as hxm_mlstm_chunkwise_fwd: a chunk other than the
    kernels' 128 steps, and dv above 512, are refused before any launch."""
    a = _lib.MlstmArgs()
    a.batch, a.heads, a.seqlen, a.dqk, a.dv = 1, 1, 256, 128, 128
    a.chunk, a.gate_mode, a.io_dtype = 64, 1, _lib.HXM_BF16
    a.struct_size = ct.sizeof(a)
    assert _lib.lib().hxm_mlstm_chunkwise_fwd_noalloc(ct.byref(a), None) == _lib.HXM_EUNSUPPORTED
    assert b"chunk" in _lib.lib().hxm_last_error_string()
    a.chunk, a.dv = 128, 1024
    assert _lib.lib().hxm_mlstm_chunkwise_fwd_noalloc(ct.byref(a), None) == _lib.HXM_EUNSUPPORTED
    assert b"512" in _lib.lib().hxm_last_error_string()


# (gate mode, dqk, seqlen, forget pre-activation mean, initial state, same kernels as the workspace entry)
CASES = [
    ("channel", 256, 300, 1.0, False, True),     # key-streaming kernel in both
    ("channel", 128, 200, 1.0, True, True),      # with an initial (C0, n0, m0) state
    ("channel", 128, 180, -4.0, False, True),    # out of the streaming range: recurrent kernel in both
    ("head", 512, 160, 3.0, True, True),         # dqk 512: key-streaming kernel in both
    ("head", 128, 260, 3.0, False, False),       # workspace entry: tcgen05 chunkwise kernel
    ("head", 256, 140, 3.0, True, False),
]


@pytest.mark.gpu
@pytest.mark.parametrize("mode,d,L,fmu,init,same_kernels", CASES)
def test_noalloc_matches_workspace_entry_point_twice(mode, d, L, fmu, init, same_kernels):
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from hybrid_model_mamba_xlstm_b200.kernels._common import stream_of
    from oracle import numpy_ref as R
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    np64 = lambda t: t.detach().float().cpu().numpy().astype(np.float64)
    for seed in (0, 1):
        g = torch.Generator().manual_seed(seed + 10 * d + L)
        b, nh, Ls = 2, 2, L + 37 * seed
        q = (torch.randn(b, nh, Ls, d, generator=g) / d ** 0.5).to(dev, torch.bfloat16)
        k = torch.randn(b, nh, Ls, d, generator=g).to(dev, torch.bfloat16)
        v = torch.randn(b, nh, Ls, d, generator=g).to(dev, torch.bfloat16)
        gs = (b, nh, Ls, d) if mode == "channel" else (b, nh, Ls)
        li = (0.5 * torch.randn(*gs, generator=g)).to(dev)
        lf = torch.nn.functional.logsigmoid(torch.randn(*gs, generator=g) + fmu).to(dev)
        C0 = n0 = m0 = None
        if init:
            C0 = (0.1 * torch.randn(b, nh, d, d, generator=g)).to(dev)
            n0 = torch.rand(b, nh, d, generator=g).to(dev)
            m0 = torch.randn(b, nh, generator=g).to(dev)
        outs = []
        for noalloc in (False, True):
            h = torch.empty(b, nh, Ls, d, device=dev, dtype=torch.bfloat16)
            CT = torch.empty(b, nh, d, d, device=dev)
            nT = torch.empty(b, nh, d, device=dev)
            mT = torch.empty(b, nh, device=dev)
            a = _args(q, k, v, li, lf, h, CT, nT, mT, C0, n0, m0)
            if noalloc:
                _lib.check("hxm_mlstm_chunkwise_fwd_noalloc",
                           _lib.lib().hxm_mlstm_chunkwise_fwd_noalloc(ct.byref(a), ct.c_void_p(stream_of(dev))))
            else:
                nbytes = _lib.lib().hxm_mlstm_workspace_size(ct.byref(a))
                ws = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
                a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
                _lib.check("hxm_mlstm_chunkwise_fwd",
                           _lib.lib().hxm_mlstm_chunkwise_fwd(ct.byref(a), ct.c_void_p(stream_of(dev))))
            torch.cuda.synchronize(dev)
            em = np.exp(np64(mT))
            outs.append((np64(h), np64(CT) * em[..., None, None], np64(nT) * em[..., None]))
        if same_kernels:
            for x, y in zip(outs[0], outs[1]):
                assert np.array_equal(x, y)
        s0 = np.exp(np64(m0)) if init else None
        ref = R.tfla_recurrent(np64(q), np64(k), np64(v), np.exp(np64(li)), np.exp(np64(lf)),
                               C0=None if C0 is None else np64(C0) * s0[..., None, None],
                               n0=None if n0 is None else np64(n0) * s0[..., None])
        for got in outs:
            for x, r in zip(got, ref):
                assert np.isfinite(x).all()
                assert rel_err(x, r) < 2e-2
