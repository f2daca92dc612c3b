"""Selective scan on the GPU vs the oracle and the reference's golden vectors.

Tolerances (normwise relative error): fp32 I/O 1e-5; bf16 I/O 2e-2 against
the oracle run in float64 on the same bf16-rounded inputs.
"""
import numpy as np
import pytest
import torch

from oracle import numpy_ref as R
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu

TOL32, TOL16 = 1e-5, 2e-2


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from hybrid_model_mamba_xlstm_b200.kernels.selective_scan import scan_interface as si
    return si


def cu(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a)).to(device="cuda", dtype=dtype)


def np64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def test_golden_reference_api_fp32(ops, golden):
    g = golden("scan_small")
    y = ops.selective_scan(cu(g["x"]), cu(g["dt"]), cu(g["A"]), cu(g["B"]), cu(g["C"]), cu(g["D"]))
    assert rel_err(np64(y), g["y"]) < TOL32
    yz = ops.selective_scan(cu(g["x"]), cu(g["dt"]), cu(g["A"]), cu(g["B"]), cu(g["C"]), cu(g["D"]), z=cu(g["z"]))
    assert rel_err(np64(yz), g["y_z"]) < TOL32


def test_golden_fused_bdl_fp32(ops, golden):
    g = golden("scan_cfg1_slice")
    y = ops.selective_scan_fn(cu(g["u"]), cu(g["raw"]), cu(g["A"]), cu(g["B"]), cu(g["C"]), cu(g["D"]),
                              z=cu(g["z"]), delta_bias=cu(g["bias"]), delta_softplus=True)
    assert rel_err(np64(y), g["y"]) < TOL32


def _oracle_bdl(inp, dtype_round=None, disc="euler", h0=None):
    t = lambda a: np.swapaxes(np64(a), 1, 2)
    return R.selective_scan(t(inp.u), t(inp.delta), np64(inp.A), t(inp.B), t(inp.C), np64(inp.D), z=t(inp.z),
                            z_mode="silu", delta_bias=np64(inp.delta_bias), delta_softplus=True,
                            discretization=disc, h0=h0)


def test_fp32_full_parity_workload_with_final_state(ops):
    """batch 2, seqlen 512, dim 1536, dstate 16, fp32: y and h_L within 1e-5."""
    from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
    inp = scan_inputs(2, 512, 1536, 16, torch.float32, seed=0, device="cuda")
    y, h = ops.selective_scan_fn(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, z=inp.z,
                                 delta_bias=inp.delta_bias, delta_softplus=True, return_last_state=True)
    yr, hr = _oracle_bdl(inp)
    assert rel_err(np.swapaxes(np64(y), 1, 2), yr) < TOL32
    assert rel_err(np64(h), hr) < TOL32


@pytest.mark.parametrize("shape", [(2, 2048, 256, 16), (1, 1000, 200, 16), (3, 37, 40, 8), (1, 1, 64, 16)])
def test_bf16_parity(ops, shape):
    from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
    b, L, dm, n = shape
    inp = scan_inputs(b, L, dm, n, torch.bfloat16, seed=1, device="cuda")
    y, h = ops.selective_scan_fn(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, z=inp.z,
                                 delta_bias=inp.delta_bias, delta_softplus=True, return_last_state=True)
    yr, hr = _oracle_bdl(inp)
    assert rel_err(np.swapaxes(np64(y), 1, 2), yr) < TOL16
    assert rel_err(np64(h), hr) < TOL16


def _rand_blD(b, L, dm, n, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(b, L, dm, generator=g)
    dt = torch.nn.functional.softplus(torch.randn(b, L, dm, generator=g) - 2.0)
    A = -torch.exp(torch.randn(dm, n, generator=g))
    B = torch.randn(b, L, n, generator=g)
    C = torch.randn(b, L, n, generator=g)
    D = torch.randn(dm, generator=g)
    z = torch.randn(b, L, dm, generator=g)
    return [t.to("cuda", dtype) for t in (x, dt)] + [A.cuda()] + [t.to("cuda", dtype) for t in (B, C)] + \
        [D.cuda(), z.to("cuda", dtype)]


@pytest.mark.parametrize("layout", ["bld", "bdl", "strided", "unaligned"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_layouts_general_A(ops, layout, dtype):
    """Reference layout (B,L,D), time-major memory, non-unit strides and
    16-byte-misaligned bases all give the oracle's answer (general-A path)."""
    b, L, dm, n = 2, 77, 96, 16
    x, dt, A, B, C, D, z = _rand_blD(b, L, dm, n, 3, dtype)

    def relayout(t):
        if layout == "bld":
            return t
        if layout == "bdl":
            return t.transpose(1, 2).contiguous().transpose(1, 2)
        if layout == "strided":
            big = torch.zeros(t.shape[0], t.shape[1], 2 * t.shape[2], device=t.device, dtype=t.dtype)
            big[:, :, ::2] = t
            return big[:, :, ::2]
        buf = torch.zeros(t.numel() + 1, device=t.device, dtype=t.dtype)
        v = buf[1:].view(t.shape)
        v.copy_(t)
        return v

    xs, dts, Bs, Cs, zs = (relayout(t) for t in (x, dt, B, C, z))
    y = ops.selective_scan(xs, dts, A, Bs, Cs, D, z=zs)
    yr, _ = R.selective_scan(np64(x), np64(dt), np64(A), np64(B), np64(C), np64(D), z=np64(z), z_mode="mul")
    tol = TOL32 if dtype == torch.float32 else TOL16
    assert rel_err(np64(y), yr) < tol


@pytest.mark.parametrize("n", [1, 4, 16, 33, 64])
def test_dstate_sizes(ops, n):
    x, dt, A, B, C, D, z = _rand_blD(1, 50, 64, n, 4, torch.float32)
    y, h = ops.selective_scan_raw(x, dt, A, B, C, D, return_last_state=True)
    yr, hr = R.selective_scan(np64(x), np64(dt), np64(A), np64(B), np64(C), np64(D))
    assert rel_err(np64(y), yr) < TOL32
    assert rel_err(np64(h), hr) < TOL32


def test_golden_zoh_reference_fp32(ops, golden):
    """discretization="zoh" against the reference's own ZOH / Taylor scan
    (mamba_block_v2.py:280-351), generated by running it: fp32 within 1e-5."""
    g = golden("scan_zoh")
    y = ops.selective_scan_raw(cu(g["x"]), cu(g["delta"]), cu(g["A"]), cu(g["B"]), cu(g["C"]), cu(g["D"]),
                               discretization="zoh")
    assert rel_err(np64(y), g["y"]) < TOL32


def test_zoh_discretization(ops):
    x, dt, A, B, C, D, z = _rand_blD(2, 64, 64, 16, 5, torch.float32)
    dt = dt * 0.2  # straddle the |dt*A| < 0.01 Taylor threshold
    y, h = ops.selective_scan_raw(x, dt, A, B, C, D, discretization="zoh", return_last_state=True)
    yr, hr = R.selective_scan(np64(x), np64(dt), np64(A), np64(B), np64(C), np64(D), discretization="zoh")
    assert rel_err(np64(y), yr) < TOL32
    assert rel_err(np64(h), hr) < TOL32


def test_segmented_equals_whole(ops):
    """Final state out + initial state in: two segments reproduce one pass."""
    from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
    inp = scan_inputs(2, 300, 128, 16, torch.float32, seed=6, device="cuda")
    kw = dict(delta_bias=inp.delta_bias, delta_softplus=True, return_last_state=True)
    y, h = ops.selective_scan_fn(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, z=inp.z, **kw)
    s = slice(0, 131)
    e = slice(131, None)
    y1, h1 = ops.selective_scan_fn(inp.u[..., s], inp.delta[..., s], inp.A, inp.B[..., s], inp.C[..., s], inp.D,
                                   z=inp.z[..., s], **kw)
    y2, h2 = ops.selective_scan_fn(inp.u[..., e], inp.delta[..., e], inp.A, inp.B[..., e], inp.C[..., e], inp.D,
                                   z=inp.z[..., e], initial_state=h1, **kw)
    assert rel_err(np64(torch.cat([y1, y2], -1)), np64(y)) < 1e-6
    assert rel_err(np64(h2), np64(h)) < 1e-6


def test_empty_and_deterministic(ops):
    x, dt, A, B, C, D, z = _rand_blD(2, 40, 64, 16, 7, torch.bfloat16)
    y1 = ops.selective_scan(x, dt, A, B, C, D)
    y2 = ops.selective_scan(x, dt, A, B, C, D)
    assert torch.equal(y1, y2)
    h0 = torch.randn(2, 64, 16, device="cuda")
    y0, hT = ops.selective_scan_raw(x[:, :0], dt[:, :0], A, B[:, :0], C[:, :0], D, h0=h0, return_last_state=True)
    assert y0.shape == (2, 0, 64) and torch.equal(hT, h0)
    e = ops.selective_scan(x[:0], dt[:0], A, B[:0], C[:0], D)
    assert e.shape == (0, 40, 64)


def test_large_workload_sampled_channels(ops):
    """batch 8, seqlen 32768, dim 4096, dstate 16, bf16 (the GB/s workload):
    a sample of channels checked against the float64 oracle at full length."""
    from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
    inp = scan_inputs(8, 32768, 4096, 16, torch.bfloat16, seed=0, device="cuda", on_device=True)
    y, h = ops.selective_scan_fn(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, z=inp.z,
                                 delta_bias=inp.delta_bias, delta_softplus=True, return_last_state=True)
    assert torch.isfinite(y).all()
    chans = torch.tensor([0, 1, 777, 2048, 4095], device="cuda")
    for b in (0, 7):
        t = lambda a: np.swapaxes(np64(a[b:b + 1, chans]), 1, 2)
        tb = lambda a: np.swapaxes(np64(a[b:b + 1]), 1, 2)
        yr, hr = R.selective_scan(t(inp.u), t(inp.delta), np64(inp.A[chans]), tb(inp.B), tb(inp.C),
                                  np64(inp.D[chans]), z=t(inp.z), z_mode="silu",
                                  delta_bias=np64(inp.delta_bias[chans]), delta_softplus=True)
        assert rel_err(np.swapaxes(np64(y[b:b + 1, chans]), 1, 2), yr) < TOL16
        assert rel_err(np64(h[b:b + 1, chans]), hr) < TOL16


@pytest.mark.parametrize("shape", [(2, 1000, 200, 16), (3, 37, 40, 8), (1, 4100, 512, 16)])
def test_bf16_channel_major_fast_path(ops, shape):
    """(batch, seqlen, dim) memory with unit channel stride — the reference's own
    selective_scan layout and the Mamba layer's — runs the fast kernel's
    channel-major variant: softplus(dt + bias), y * silu(z), final state."""
    from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
    b, L, dm, n = shape
    inp = scan_inputs(b, L, dm, n, torch.bfloat16, seed=2, device="cuda")
    t = lambda a: a.transpose(1, 2).contiguous()        # (B, L, D) / (B, L, N) dense
    y, h = ops.selective_scan_raw(t(inp.u), t(inp.delta), inp.A, t(inp.B), t(inp.C), inp.D, t(inp.z), z_mode="silu",
                                  delta_bias=inp.delta_bias, delta_softplus=True, return_last_state=True)
    yr, hr = _oracle_bdl(inp)
    assert rel_err(np64(y), yr) < TOL16
    assert rel_err(np64(h), hr) < TOL16


def test_bf16_channel_major_projection_views(ops):
    """The Mamba layer's views: x / z halves of one in_proj output and the B / C
    column slices of the x_proj output (row strides 2*dim and r + 2n)."""
    g = torch.Generator(device="cuda").manual_seed(5)
    b, L, dm, n, r = 2, 300, 128, 16, 8
    xz = torch.randn(b, L, 2 * dm, device="cuda", generator=g).to(torch.bfloat16)
    dbc = torch.randn(b, L, r + 2 * n, device="cuda", generator=g).to(torch.bfloat16)
    dt = (torch.randn(b, L, dm, device="cuda", generator=g) * 0.5 - 3.0).to(torch.bfloat16)
    A = -torch.arange(1, n + 1, device="cuda", dtype=torch.float32).repeat(dm, 1)
    D = torch.ones(dm, device="cuda")
    bias = torch.full((dm,), -1.0, device="cuda")
    u, z = xz[..., :dm], xz[..., dm:]
    Bm, Cm = dbc[..., r:r + n], dbc[..., r + n:]
    y = ops.selective_scan_raw(u, dt, A, Bm, Cm, D, z, z_mode="silu", delta_bias=bias, delta_softplus=True)
    yr, _ = R.selective_scan(np64(u), np64(dt), np64(A), np64(Bm), np64(Cm), np64(D), z=np64(z), z_mode="silu",
                             delta_bias=np64(bias), delta_softplus=True)
    assert rel_err(np64(y), yr) < TOL16


# ---------------------------------------------------------------- time segments --
def _fused(ops, inp, h0=None, nseg=None):
    """selective_scan_fn with HXM_SCAN_NSEG forcing the segment count (None: automatic)."""
    import os
    old = os.environ.get("HXM_SCAN_NSEG")
    if nseg is not None:
        os.environ["HXM_SCAN_NSEG"] = str(nseg)
    try:
        return ops.selective_scan_fn(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, z=inp.z, delta_bias=inp.delta_bias,
                                     delta_softplus=True, return_last_state=True, initial_state=h0)
    finally:
        if nseg is not None:
            if old is None:
                del os.environ["HXM_SCAN_NSEG"]
            else:
                os.environ["HXM_SCAN_NSEG"] = old


@pytest.mark.parametrize("L,nseg", [(1000, 2), (1000, 3), (4101, 16), (9000, None)])
def test_time_segments_match_one_pass_and_oracle(ops, L, nseg):
    """A grid too small for the GPU (one batch row, 256 channels) runs as
    parallel time segments after a state-only pass: y and the final state
    match the float64 oracle (bf16 2e-2) and the one-pass kernel (1e-3: the
    carry uses exp(A * sum delta) instead of the product of per-step
    factors), from a nonzero initial state, with ragged segment ends."""
    from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
    inp = scan_inputs(1, L, 256, 16, torch.bfloat16, seed=21, device="cuda")
    h0 = torch.randn(1, 256, 16, generator=torch.Generator().manual_seed(22)).cuda()
    y, h = _fused(ops, inp, h0, nseg)
    y1, h1 = _fused(ops, inp, h0, 1)
    yr, hr = _oracle_bdl(inp, h0=np64(h0))
    assert rel_err(np64(y), np.swapaxes(yr, 1, 2)) < TOL16
    assert rel_err(np64(h), hr) < TOL16
    assert rel_err(np64(y), np64(y1)) < 1e-3
    assert rel_err(np64(h), np64(h1)) < 1e-3


def test_time_segments_channel_major_views(ops):
    """The Mamba layer's (B, L, D) projection views (channel-major fast path)
    with few channels: segmented run vs the one-pass run and the oracle."""
    g = torch.Generator().manual_seed(23)
    bt, L, dm, n = 1, 1500, 128, 16
    xz = torch.randn(bt, L, 2 * dm, generator=g).to("cuda", torch.bfloat16)
    x, zz = xz[..., :dm], xz[..., dm:]
    dt = (torch.rand(bt, L, dm, generator=g) * 0.1).to("cuda", torch.bfloat16)
    bc = torch.randn(bt, L, 2 * n, generator=g).to("cuda", torch.bfloat16)
    A = -torch.arange(1, n + 1, dtype=torch.float32).repeat(dm, 1).cuda()
    D = torch.ones(dm, device="cuda")
    import os
    ys = []
    for nseg in ("4", "1"):
        os.environ["HXM_SCAN_NSEG"] = nseg
        try:
            ys.append(ops.selective_scan_raw(x, dt, A, bc[..., :n], bc[..., n:], D, zz, z_mode="silu",
                                             return_last_state=True))
        finally:
            del os.environ["HXM_SCAN_NSEG"]
    yr, hr = R.selective_scan(np64(x), np64(dt), np64(A), np64(bc[..., :n]), np64(bc[..., n:]), np64(D),
                              z=np64(zz), z_mode="silu")
    assert rel_err(np64(ys[0][0]), yr) < TOL16 and rel_err(np64(ys[0][1]), hr) < TOL16
    assert rel_err(np64(ys[0][0]), np64(ys[1][0])) < 1e-3


@pytest.mark.slow
def test_time_segments_one_row_of_the_long_workload(ops):
    """One batch row of the long-context scan (32768 steps x 4096 channels:
    one GPU's share when batch 8 is split over 8 GPUs) runs in automatic time
    segments; three channels checked against the C oracle over all steps."""
    from hybrid_model_mamba_xlstm_b200.workloads import scan_rows
    from oracle import build as OC
    inp = scan_rows(range(5, 6), 32768, 4096, 16, torch.bfloat16, seed=11, device="cuda")
    y, h = _fused(ops, inp)
    for d in (0, 2049, 4095):
        f = lambda t: t[:, d:d + 1].float().cpu().numpy()  # noqa: E731
        yr, hr = OC.scan(f(inp.u), f(inp.delta), inp.A[d:d + 1].cpu().numpy(), inp.B.float().cpu().numpy(),
                         inp.C.float().cpu().numpy(), inp.D[d:d + 1].cpu().numpy(), f(inp.z),
                         inp.delta_bias[d:d + 1].cpu().numpy(), softplus=True, z_mode=2, disc=0)
        assert rel_err(np64(y[0, d]), yr[0, 0]) < TOL16, d
        assert rel_err(np64(h[0, d]), hr[0, 0]) < TOL16, d
