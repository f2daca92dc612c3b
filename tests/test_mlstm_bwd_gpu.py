"""Chunkwise mLSTM backward vs autograd of the reference loop.

The reference's backward (tfla_interface.py:52-81) re-runs the step loop
tfla_forward_pytorch (:84-139) under autograd; the check here does the same in
float64 on the same inputs and compares every gradient of apply_tfla (q, k, v,
i_gate, f_gate).  Tolerances (normwise relative error): fp32 I/O 1e-4 (fp32
chunk GEMMs and state); bf16 I/O 2e-2 against the loop on the bf16-rounded
inputs (tcgen05 chunk GEMMs on bf16 operands, ~2e-3).
"""
import ctypes as ct
import math

import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
TOL32, TOL16 = 1e-4, 2e-2


@pytest.fixture(scope="module")
def T():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    torch.backends.cuda.matmul.allow_tf32 = False
    from hybrid_model_mamba_xlstm_b200.kernels import tfla
    return tfla


def _loop(q, k, v, ig, fg):
    """float64 restatement of tfla_forward_pytorch (tfla_interface.py:84-139)."""
    bsz, nh, L, d = q.shape
    C = torch.zeros(bsz, nh, d, v.shape[-1], dtype=q.dtype)
    n = torch.zeros(bsz, nh, d, dtype=q.dtype)
    hs = []
    for t in range(L):
        C = fg[:, :, t, :, None] * C + ig[:, :, t, :, None] * (k[:, :, t, :, None] * v[:, :, t, None, :])
        n = fg[:, :, t] * n + ig[:, :, t] * k[:, :, t]
        num = torch.einsum("bhd,bhde->bhe", q[:, :, t], C)
        den = torch.clamp(torch.einsum("bhd,bhd->bh", q[:, :, t], n), min=1.0)[..., None]
        hs.append(num / den)
    return torch.stack(hs, 2)


def _d64(t):
    return t.detach().double().cpu()


def _case(shape, dv, per_channel, fmu, seed, dtype, qscale=None):
    bsz, nh, L, d = shape
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(bsz, nh, L, d, generator=g) * (qscale if qscale is not None else 1 / math.sqrt(d))
    k = torch.randn(bsz, nh, L, d, generator=g)
    v = torch.randn(bsz, nh, L, dv, generator=g)
    gs = (bsz, nh, L, d) if per_channel else (bsz, nh, L, 1)
    ipre = torch.randn(*gs, generator=g) * 0.5
    fpre = torch.randn(*gs, generator=g) + fmu
    dh = torch.randn(bsz, nh, L, dv, generator=g)
    q, k, v, dh = (t.to(dtype) for t in (q, k, v, dh))
    return q, k, v, torch.exp(ipre), torch.sigmoid(fpre), dh


def _grads_gpu(T, q, k, v, ig, fg, dh, expand):
    leaves = [t.cuda().requires_grad_(True) for t in (q, k, v, ig, fg)]
    igx, fgx = leaves[3], leaves[4]
    if expand:
        igx, fgx = igx.expand(*q.shape), fgx.expand(*q.shape)
    out = T.apply_tfla(leaves[0], leaves[1], leaves[2], igx, fgx)
    out.backward(dh.cuda())
    return out, [t.grad for t in leaves]


def _grads_ref(q, k, v, ig, fg, dh, expand):
    leaves = [_d64(t).requires_grad_(True) for t in (q, k, v, ig, fg)]
    igx, fgx = leaves[3], leaves[4]
    if expand:
        igx, fgx = igx.expand(*q.shape), fgx.expand(*q.shape)
    out = _loop(leaves[0], leaves[1], leaves[2], igx, fgx)
    out.backward(_d64(dh))
    return out, [t.grad for t in leaves]


# the reference's own test shapes (tests/test_kernels.py) plus ragged lengths
@pytest.mark.parametrize("shape,dv,per_channel,fmu", [
    ((2, 4, 64, 32), 32, True, 3.0), ((2, 4, 32, 16), 16, True, 0.0), ((1, 2, 16, 8), 8, True, 3.0),
    ((1, 2, 37, 16), 24, True, 0.0), ((2, 2, 130, 32), 32, False, 3.0), ((1, 1, 1, 8), 8, True, 3.0)])
def test_apply_tfla_grads_fp32(T, shape, dv, per_channel, fmu):
    case = _case(shape, dv, per_channel, fmu, seed=sum(shape), dtype=torch.float32)
    out, got = _grads_gpu(T, *case, expand=not per_channel)
    ref_out, want = _grads_ref(*case, expand=not per_channel)
    assert rel_err(_d64(out).numpy(), ref_out.detach().numpy()) < 1e-5
    for name, a, b in zip(("dq", "dk", "dv", "di", "df"), got, want):
        assert a.shape == b.shape, name
        assert rel_err(_d64(a).numpy(), b.numpy()) < TOL32, name


def test_apply_tfla_grads_normalizer_clamp_active(T):
    """Large q so that q.n > 1 on most steps: the den branch of the gradient."""
    case = _case((1, 2, 96, 16), 16, True, 2.0, seed=5, dtype=torch.float32, qscale=1.0)
    _, got = _grads_gpu(T, *case, expand=False)
    _, want = _grads_ref(*case, expand=False)
    for name, a, b in zip(("dq", "dk", "dv", "di", "df"), got, want):
        assert rel_err(_d64(a).numpy(), b.numpy()) < TOL32, name


def test_apply_tfla_grads_bf16_channel_gates(T):
    """mLSTMBlock-like: bf16 q, k, v, head 128, per-channel gates near sigmoid(N(0, 1))."""
    q, k, v, ig, fg, dh = _case((1, 2, 300, 128), 128, True, 0.0, seed=11, dtype=torch.bfloat16)
    out, got = _grads_gpu(T, q, k, v, ig, fg, dh, expand=False)
    _, want = _grads_ref(q, k, v, ig, fg, dh, expand=False)
    assert got[0].dtype == torch.bfloat16
    for name, a, b in zip(("dq", "dk", "dv", "di", "df"), got, want):
        assert rel_err(_d64(a).numpy(), b.numpy()) < TOL16, name


@pytest.mark.parametrize("per_channel,d,dv,L", [(True, 128, 128, 300), (False, 128, 96, 260), (False, 256, 256, 200),
                                                 (True, 512, 512, 150)])
def test_tensor_core_backward_bf16_vs_loop(T, per_channel, d, dv, L):
    """bf16 inputs take the tcgen05 chunk-GEMM backward (128-step chunks):
    every gradient of apply_tfla against float64 autograd of the loop, per-
    channel gates and per-head gates (expanded views), ragged lengths."""
    q, k, v, ig, fg, dh = _case((1, 2, L, d), dv, per_channel, 1.0, seed=d + L, dtype=torch.bfloat16)
    out, got = _grads_gpu(T, q, k, v, ig, fg, dh, expand=not per_channel)
    _, want = _grads_ref(q, k, v, ig, fg, dh, expand=not per_channel)
    for name, a, b in zip(("dq", "dk", "dv", "di", "df"), got, want):
        assert torch.isfinite(a).all(), name
        assert rel_err(_d64(a).numpy(), b.numpy()) < TOL16, name


@pytest.mark.parametrize("gates", ["head", "channel"])
@pytest.mark.parametrize("precise", [False, True])
def test_tensor_core_backward_matches_library_path(T, gates, precise):
    """The tcgen05 backward (bf16 high / low split operands) against the fp32
    library-GEMM path on the same bf16 inputs (batch 2, 4 heads, 700 steps,
    d 256): every output, per-head gate gradients through the W = dL/dS * S
    identity included.  precise (the default, all fp32 operands split):
    within 2e-4; precise=False (the gate-scaled q, k split): within 5e-2
    (2.9e-2 measured for the per-channel gates, whose normalizer gradient
    cancels over the long memory of these gates)."""
    bsz, nh, L, d = 2, 4, 700, 256
    g = torch.Generator().manual_seed(77)
    q = (torch.randn(bsz, nh, L, d, generator=g) / 16).to("cuda", torch.bfloat16)
    k, v, dh = (torch.randn(bsz, nh, L, d, generator=g).to("cuda", torch.bfloat16) for _ in range(3))
    gs = (bsz, nh, L) if gates == "head" else (bsz, nh, L, d)
    li = (torch.randn(*gs, generator=g) * 0.5).cuda()
    lf = torch.nn.functional.logsigmoid(torch.randn(*gs, generator=g) + 2.0).cuda()
    tc = T.mlstm_chunkwise_bwd(q, k, v, li, lf, dh, tensor_cores=True, precise=precise)
    lib = T.mlstm_chunkwise_bwd(q, k, v, li, lf, dh, tensor_cores=False, tf32=False)
    for name, a, b in zip(("dq", "dk", "dv", "dlog_i", "dlog_f", "di"), tc, lib):
        assert a.shape == b.shape, name
        assert rel_err(_d64(a).numpy(), _d64(b).numpy()) < (2e-4 if precise else 5e-2), name


def test_log_gate_entry_per_head_sums(T):
    """mlstm_chunkwise_bwd on (B, H, L) log gates returns the per-channel
    gate gradients summed over Dqk, and d(log i) = i * dL/di."""
    q, k, v, ig, fg, dh = (t.cuda() for t in _case((2, 2, 70, 16), 16, False, 3.0, seed=3, dtype=torch.float32))
    li, lf = torch.log(ig[..., 0]), torch.log(fg[..., 0])
    per_head = T.mlstm_chunkwise_bwd(q, k, v, li, lf, dh, chunk=32)
    per_chan = T.mlstm_chunkwise_bwd(q, k, v, li, lf, dh, chunk=32, gate_grads="channel")
    for a, b in zip(per_head[:3], per_chan[:3]):
        assert torch.equal(a, b)
    for a, b in zip(per_head[3:], per_chan[3:]):  # the same sums in another order
        assert a.shape == (2, 2, 70) and b.shape == (2, 2, 70, 16)
        assert rel_err(_d64(a).numpy(), _d64(b.sum(-1)).numpy()) < 1e-5
    assert torch.allclose(per_head[3], torch.exp(li) * per_head[5], rtol=1e-5, atol=1e-6)
    # a different chunk length gives the same gradients
    other = T.mlstm_chunkwise_bwd(q, k, v, li, lf, dh, chunk=64)
    for a, b in zip(per_head, other):
        assert rel_err(_d64(a).numpy(), _d64(b).numpy()) < 1e-5


def test_chunk_state_scan_forward_and_reverse(T):
    """hxm_chunk_state_scan through the C ABI vs a host loop, with and without
    decay (and with the row-scaled copy of the output), on the scalar path
    (9 columns) and the 16-byte path (8 columns)."""
    from hybrid_model_mamba_xlstm_b200 import _lib
    g = torch.Generator().manual_seed(4)
    for cols in (9, 8):
        x = torch.randn(2, 3, 5, 7, cols, generator=g)
        dec = torch.rand(2, 3, 5, 7, generator=g)
        scl = torch.rand(2, 3, 5, 7, generator=g) + 0.5
        for reverse in (0, 1):
            for use_decay in (True, False):
                xd = x.clone().cuda()
                dd = dec.cuda() if use_decay else None
                a = _lib.ChunkScanArgs()
                a.groups, a.nchunks, a.rows, a.cols = 6, 5, 7, cols
                a.x, a.decay, a.reverse = xd.data_ptr(), None if dd is None else dd.data_ptr(), reverse
                sc, out = (scl.cuda(), torch.empty_like(xd)) if use_decay else (None, None)
                if use_decay:
                    a.scale, a.scaled = sc.data_ptr(), out.data_ptr()
                _lib.call("hxm_chunk_state_scan", a, torch.cuda.current_stream().cuda_stream)
                want = torch.empty_like(x)
                s = torch.zeros(2, 3, 7, cols)
                order = range(4, -1, -1) if reverse else range(5)
                for kc in order:
                    want[:, :, kc] = s
                    s = (dec[:, :, kc, :, None] if use_decay else 1.0) * s + x[:, :, kc]
                assert torch.allclose(xd.cpu(), want, rtol=1e-6, atol=1e-6), (cols, reverse, use_decay)
                if use_decay:
                    assert torch.allclose(out.cpu(), scl[..., None] * want, rtol=1e-6, atol=1e-6), (cols, reverse)


@pytest.mark.parametrize("cols", [8, 136, 520])
def test_chunk_state_scan_row_mode_split_and_dot(T, cols):
    """Row mode of hxm_chunk_state_scan (the tensor-core backward's): the scaled
    exclusive states as bf16 high / low parts (x read only), and the chunk
    gradients <out[k], state[k + 1]> read back from a state scan's split copy
    divided by its scale, vs a host loop (float64)."""
    from hybrid_model_mamba_xlstm_b200 import _lib
    g = torch.Generator().manual_seed(cols)
    G, nch, rows = 3, 6, 5
    x = torch.randn(G, 1, nch, rows, cols, generator=g)
    dec = torch.rand(G, 1, nch, rows, generator=g)
    scl = torch.rand(G, 1, nch, rows, generator=g) + 0.5
    st = torch.cuda.current_stream().cuda_stream

    def scan(xs, reverse, scale, dot=None):
        xd = xs.cuda()
        hi = torch.empty(xd.shape, device="cuda", dtype=torch.bfloat16)
        lo = torch.empty_like(hi)
        dd, sd = dec.cuda(), scale.cuda()  # (kept alive until the scan has run)
        a = _lib.ChunkScanArgs()
        a.groups, a.nchunks, a.rows, a.cols = G, nch, rows, cols
        a.x, a.decay, a.reverse, a.scale = xd.data_ptr(), dd.data_ptr(), reverse, sd.data_ptr()
        a.scaled_hi, a.scaled_lo, a.skip_state = hi.data_ptr(), lo.data_ptr(), 1
        keep = [xd, dd, sd]
        dg = None
        if dot is not None:
            dg = torch.empty(G, 1, nch, rows, device="cuda")
            ds = dot[2].cuda()
            keep.append(ds)
            a.dot_hi, a.dot_lo, a.dot_scale, a.dot_out = dot[0].data_ptr(), dot[1].data_ptr(), ds.data_ptr(), dg.data_ptr()
        _lib.call("hxm_chunk_state_scan", a, st)
        torch.cuda.synchronize()
        assert torch.equal(xd.cpu(), xs)  # read only
        return hi, lo, dg

    def host(xs, reverse):
        out = torch.empty_like(xs, dtype=torch.float64)
        s = torch.zeros(G, 1, rows, cols, dtype=torch.float64)
        for kc in (range(nch - 1, -1, -1) if reverse else range(nch)):
            out[:, :, kc] = s
            s = dec[:, :, kc, :, None].double() * s + xs[:, :, kc].double()
        return out

    fh, fl, _ = scan(x, 0, scl)
    want_f = host(x, 0)
    assert rel_err((fh.double() + fl.double()).cpu().numpy(), (scl[..., None].double() * want_f).numpy()) < 2e-5
    y = torch.randn(G, 1, nch, rows, cols, generator=g)
    sy = torch.rand(G, 1, nch, rows, generator=g) + 0.5
    _, _, dg = scan(y, 1, sy, dot=(fh, fl, scl))
    want_y = host(y, 1)
    want_dg = torch.zeros(G, 1, nch, rows, dtype=torch.float64)
    want_dg[:, :, :-1] = (want_y[:, :, :-1] * want_f[:, :, 1:]).sum(-1)
    assert rel_err(dg.double().cpu().numpy(), want_dg.numpy()) < 2e-5


def test_bf16_tf32_gemms_close_to_fp32_gemms(T):
    """The bf16 default (TF32 chunk GEMMs) against tf32=False on the same
    inputs, per-channel and per-head gates: every gradient within 5e-3."""
    for pc in (True, False):
        q, k, v, ig, fg, dh = (t.cuda() for t in _case((2, 2, 256, 128), 128, pc, 0.0, seed=17,
                                                        dtype=torch.bfloat16))
        li, lf = torch.log(ig), torch.log(fg)
        if not pc:
            li, lf = li[..., 0], lf[..., 0]
        fast = T.mlstm_chunkwise_bwd(q, k, v, li, lf, dh)
        full = T.mlstm_chunkwise_bwd(q, k, v, li, lf, dh, tf32=False)
        for a, b in zip(fast, full):
            assert rel_err(_d64(a).numpy(), _d64(b).numpy()) < 5e-3, pc


def test_chunk_state_dot(T):
    """hxm_chunk_state_dot vs torch: <adj_k, state_{k+1}> per row, 0 for the last chunk."""
    from hybrid_model_mamba_xlstm_b200 import _lib
    g = torch.Generator().manual_seed(6)
    for cols in (9, 8):
        adj, state = torch.randn(2, 3, 5, 7, cols, generator=g), torch.randn(2, 3, 5, 7, cols, generator=g)
        out = torch.full((2, 3, 5, 7), float("nan")).cuda()
        a = _lib.ChunkDotArgs()
        a.groups, a.nchunks, a.rows, a.cols = 6, 5, 7, cols
        ad, sd = adj.cuda(), state.cuda()
        a.adj, a.state, a.out = ad.data_ptr(), sd.data_ptr(), out.data_ptr()
        _lib.call("hxm_chunk_state_dot", a, torch.cuda.current_stream().cuda_stream)
        want = torch.zeros(2, 3, 5, 7)
        want[:, :, :-1] = (adj[:, :, :-1] * state[:, :, 1:]).sum(-1)
        assert torch.allclose(out.cpu(), want, rtol=1e-5, atol=1e-5), cols
