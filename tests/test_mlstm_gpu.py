"""mLSTM (TFLA) forward on the GPU vs the reference's golden vectors and the oracle.

Tolerances (normwise relative): fp32 I/O 1e-5 against float64; bf16 I/O
2e-2 against the float64 oracle on the same bf16-rounded inputs.  Final
states are compared as exp(m) * (C, n) against the oracle's true state.
"""
import math

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
    from hybrid_model_mamba_xlstm_b200.kernels.tfla import tfla_interface as ti
    return ti


def cu(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a)).to(device="cuda", dtype=dtype)


def np64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("name", ["tfla_1x2x16x8", "tfla_2x4x32x16", "tfla_2x4x64x32"])
def test_golden_apply_tfla_fp32_channel_gates(ops, golden, name):
    """The reference's own test shapes (tests/test_kernels.py), per-channel gates."""
    g = golden(name)
    ig = cu(np.exp(g["i_pre"].astype(np.float64)))
    fg = cu(1 / (1 + np.exp(-g["f_pre"].astype(np.float64))))
    h = ops.apply_tfla(cu(g["q"]), cu(g["k"]), cu(g["v"]), ig, fg)
    assert h.dtype == torch.float32
    assert rel_err(np64(h), g["h"]) < TOL32


def test_golden_scalar_gates_broadcast_view(ops, golden):
    """Per-head gates given as expand()ed (B,H,L,D) views take the scalar path."""
    g = golden("tfla_scalar_gates")
    b, h, L, d = g["q"].shape
    ig = cu(np.exp(g["i_pre"].astype(np.float64)))[..., None].expand(b, h, L, d)
    fg = cu(1 / (1 + np.exp(-g["f_pre"].astype(np.float64))))[..., None].expand(b, h, L, d)
    out = ops.apply_tfla(cu(g["q"]), cu(g["k"]), cu(g["v"]), ig, fg)
    assert rel_err(np64(out), g["h"]) < TOL32
    out16 = ops.apply_tfla(cu(g["q"], torch.bfloat16), cu(g["k"], torch.bfloat16), cu(g["v"], torch.bfloat16), ig, fg)
    q16, k16, v16 = (np64(cu(g[n], torch.bfloat16)) for n in ("q", "k", "v"))
    ref16, _, _ = R.tfla_recurrent(q16, k16, v16, np64(ig[..., 0]), np64(fg[..., 0]))
    assert rel_err(np64(out16), ref16) < TOL16


def _oracle_state(inp_np, C0=None, n0=None):
    q, k, v, li, lf = inp_np
    return R.tfla_recurrent(q, k, v, np.exp(li), np.exp(lf), C0=C0, n0=n0)


@pytest.mark.parametrize("shape,dtype", [((2, 4, 256, 64), torch.float32), ((1, 2, 200, 128), torch.bfloat16),
                                         ((2, 4, 2048, 256), torch.bfloat16), ((1, 1, 300, 512), torch.bfloat16),
                                         ((1, 2, 130, 96), torch.bfloat16)])
def test_scalar_gate_parity_with_states(ops, shape, dtype):
    """Config-2 value distributions (q/sqrt(d), exp input gate ~N(0,1),
    logsigmoid forget gate ~N(3,1)); h and the final (C, n) state."""
    from hybrid_model_mamba_xlstm_b200.workloads import mlstm_inputs
    b, h, L, d = shape
    inp = mlstm_inputs(b, h, L, d, dtype, seed=2, device="cuda")
    out, (C, n, m) = ops.mlstm_chunkwise_fwd(inp.q, inp.k, inp.v, inp.log_i, inp.log_f, return_state=True)
    ref_h, ref_C, ref_n = _oracle_state([np64(t) for t in (inp.q, inp.k, inp.v, inp.log_i, inp.log_f)])
    tol = TOL32 if dtype == torch.float32 else TOL16
    assert rel_err(np64(out), ref_h) < tol
    em = np.exp(np64(m))
    assert rel_err(np64(C) * em[..., None, None], ref_C) < tol
    assert rel_err(np64(n) * em[..., None], ref_n) < tol


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_channel_gate_parity_layer_distribution(ops, dtype):
    """Per-channel gates as mLSTMBlock makes them: i = exp(pre), f = sigmoid(pre)."""
    g = torch.Generator().manual_seed(5)
    b, h, L, d = 2, 2, 96, 64
    q, k, v = (torch.randn(b, h, L, d, generator=g) for _ in range(3))
    ipre = torch.randn(b, h, L, d, generator=g) * 0.5
    fpre = torch.randn(b, h, L, d, generator=g) + 1.0
    ig, fg = ipre.exp(), torch.sigmoid(fpre)
    out = ops.apply_tfla(*(t.to("cuda", dtype) for t in (q, k, v)), ig.cuda(), fg.cuda())
    qn, kn, vn = (np64(t.to("cuda", dtype)) for t in (q, k, v))
    ref, _, _ = R.tfla_recurrent(qn, kn, vn, ig.double().numpy(), fg.double().numpy())
    assert rel_err(np64(out), ref) < (TOL32 * 10 if dtype == torch.float32 else TOL16)


def test_segmented_state_roundtrip(ops):
    """Final (C, n, m) fed back as the initial state continues the sequence."""
    from hybrid_model_mamba_xlstm_b200.workloads import mlstm_inputs
    inp = mlstm_inputs(1, 2, 384, 64, torch.bfloat16, seed=3, device="cuda")
    full = ops.mlstm_chunkwise_fwd(inp.q, inp.k, inp.v, inp.log_i, inp.log_f)
    s = 200
    a, st = ops.mlstm_chunkwise_fwd(inp.q[:, :, :s], inp.k[:, :, :s], inp.v[:, :, :s], inp.log_i[:, :, :s],
                                    inp.log_f[:, :, :s], return_state=True)
    b2 = ops.mlstm_chunkwise_fwd(inp.q[:, :, s:], inp.k[:, :, s:], inp.v[:, :, s:], inp.log_i[:, :, s:],
                                 inp.log_f[:, :, s:], *st)
    assert rel_err(np64(torch.cat([a, b2], 2)), np64(full)) < 1e-2


@pytest.mark.parametrize("d", [128, 256])
def test_tensor_core_path_segmented_state(ops, d):
    """The tcgen05 chunkwise kernel (bf16, per-head gates, dqk 128/256): a
    sequence split at a non-chunk boundary with the stabilized (C, n, m)
    carried over matches one pass and the float64 oracle."""
    from hybrid_model_mamba_xlstm_b200.workloads import mlstm_inputs
    inp = mlstm_inputs(2, 2, 700, d, torch.bfloat16, seed=11, device="cuda")
    full, (C, n, m) = ops.mlstm_chunkwise_fwd(inp.q, inp.k, inp.v, inp.log_i, inp.log_f, return_state=True)
    s = 333
    a, st = ops.mlstm_chunkwise_fwd(inp.q[:, :, :s], inp.k[:, :, :s], inp.v[:, :, :s], inp.log_i[:, :, :s],
                                    inp.log_f[:, :, :s], return_state=True)
    b2, st2 = ops.mlstm_chunkwise_fwd(inp.q[:, :, s:], inp.k[:, :, s:], inp.v[:, :, s:], inp.log_i[:, :, s:],
                                      inp.log_f[:, :, s:], *st, return_state=True)
    ref_h, ref_C, ref_n = _oracle_state([np64(t) for t in (inp.q, inp.k, inp.v, inp.log_i, inp.log_f)])
    assert rel_err(np64(full), ref_h) < TOL16
    assert rel_err(np64(torch.cat([a, b2], 2)), ref_h) < TOL16
    for (Cx, nx, mx) in ((C, n, m), st2):
        em = np.exp(np64(mx))
        assert rel_err(np64(Cx) * em[..., None, None], ref_C) < TOL16
        assert rel_err(np64(nx) * em[..., None], ref_n) < TOL16


def test_den_clamp_and_large_input_gates(ops):
    """Large input-gate pre-activations (exp(60) would overflow the reference's
    unstabilized fp32 state) stay finite and match the float64 oracle."""
    g = torch.Generator().manual_seed(9)
    b, h, L, d = 1, 1, 64, 32
    q, k, v = (torch.randn(b, h, L, d, generator=g, dtype=torch.float64) for _ in range(3))
    li = torch.randn(b, h, L, generator=g, dtype=torch.float64) * 3 + 60.0
    lf = torch.nn.functional.logsigmoid(torch.randn(b, h, L, generator=g, dtype=torch.float64))
    out = ops.mlstm_chunkwise_fwd(q.float().cuda(), k.float().cuda(), v.float().cuda(), li.float().cuda(),
                                  lf.float().cuda())
    ref, _, _ = R.tfla_recurrent(q.numpy(), k.numpy(), v.numpy(), np.exp(li.numpy()), np.exp(lf.numpy()))
    assert np.isfinite(np64(out)).all()
    assert rel_err(np64(out), ref) < 1e-4


def test_empty_sequence_keeps_state(ops):
    q = torch.zeros(1, 2, 0, 32, device="cuda")
    C0 = torch.randn(1, 2, 32, 32, device="cuda")
    n0 = torch.randn(1, 2, 32, device="cuda")
    m0 = torch.zeros(1, 2, device="cuda")
    h, (C, n, m) = ops.mlstm_chunkwise_fwd(q, q, q, q[..., 0], q[..., 0], C0, n0, m0, return_state=True)
    assert h.shape == (1, 2, 0, 32)
    assert torch.allclose(C * m.exp()[..., None, None], C0) and torch.allclose(n * m.exp()[..., None], n0)


@pytest.mark.parametrize("d,odd", [(128, False), (256, False), (512, False), (128, True)])
def test_stream_kernel_channel_gates(ops, d, odd):
    """Per-channel gates (mLSTMBlock's i = exp(pre), f = sigmoid(pre), one per
    key channel) on the key-streaming tcgen05 kernel vs the float64 oracle.
    odd: the gate rows are views of (.., d + 1)-wide memory (odd time stride)."""
    g = torch.Generator().manual_seed(21)
    b, h, L = 1, 2, 300
    q = (torch.randn(b, h, L, d, generator=g) / d ** 0.5).to("cuda", torch.bfloat16)
    k = torch.randn(b, h, L, d, generator=g).to("cuda", torch.bfloat16)
    v = torch.randn(b, h, L, d, generator=g).to("cuda", torch.bfloat16)
    ipre = torch.randn(b, h, L, d, generator=g) * 0.5
    fpre = torch.randn(b, h, L, d, generator=g) + 1.0
    li, lf = ipre.cuda(), torch.nn.functional.logsigmoid(fpre).cuda()
    if odd:
        wide = torch.zeros(2, b, h, L, d + 1, device="cuda")
        wide[0, ..., :d], wide[1, ..., :d] = li, lf
        li, lf = wide[0, ..., :d], wide[1, ..., :d]
        assert li.stride(2) % 2 == 1
    out, (C, n, m) = ops.mlstm_chunkwise_fwd(q, k, v, li, lf, return_state=True)
    ref, Cr, nr = R.tfla_recurrent(np64(q), np64(k), np64(v), np.exp(np64(li)), np.exp(np64(lf)))
    assert rel_err(np64(out), ref) < TOL16
    em = np.exp(np64(m))
    assert rel_err(np64(C) * em[..., None, None], Cr) < TOL16
    assert rel_err(np64(n) * em[..., None], nr) < TOL16


@pytest.mark.parametrize("d", [128, 512])
def test_stream_kernel_strong_channel_decay_segmented(ops, d):
    """Per-channel forget gates near sigmoid(N(0, 1)) (mLSTMBlock at init): the
    log forget gate of one 128-step chunk sums to about -100 per channel, so
    the per-chunk factors e^(g/2) of two chunks multiply below the fp32 normal
    range; the carried state must still reach the next chunk and the next call."""
    g = torch.Generator().manual_seed(23)
    b, h, L = 1, 2, 512
    q = (torch.randn(b, h, L, d, generator=g) / d ** 0.5).to("cuda", torch.bfloat16)
    k = torch.randn(b, h, L, d, generator=g).to("cuda", torch.bfloat16)
    v = torch.randn(b, h, L, d, generator=g).to("cuda", torch.bfloat16)
    li = (torch.randn(b, h, L, d, generator=g) * 0.5).cuda()
    lf = torch.nn.functional.logsigmoid(torch.randn(b, h, L, d, generator=g)).cuda()
    ref, Cr, nr = R.tfla_recurrent(np64(q), np64(k), np64(v), np.exp(np64(li)), np.exp(np64(lf)))
    out, (C, n, m) = ops.mlstm_chunkwise_fwd(q, k, v, li, lf, return_state=True)
    assert rel_err(np64(out), ref) < TOL16
    em = np.exp(np64(m))
    assert rel_err(np64(C) * em[..., None, None], Cr) < TOL16
    assert rel_err(np64(n) * em[..., None], nr) < TOL16
    s = 256
    a, st = ops.mlstm_chunkwise_fwd(q[:, :, :s], k[:, :, :s], v[:, :, :s], li[:, :, :s], lf[:, :, :s],
                                    return_state=True)
    b2 = ops.mlstm_chunkwise_fwd(q[:, :, s:], k[:, :, s:], v[:, :, s:], li[:, :, s:], lf[:, :, s:], *st)
    assert rel_err(np64(b2), ref[:, :, s:]) < TOL16


def test_stream_kernel_scalar_gates_d512_segmented(ops):
    """Per-head gates with dqk = dv = 512 (the long-context configuration's head
    size) on the streaming kernel; state carried across a split."""
    from hybrid_model_mamba_xlstm_b200.workloads import mlstm_inputs
    inp = mlstm_inputs(1, 2, 640, 512, torch.bfloat16, seed=13, device="cuda")
    full, (C, n, m) = ops.mlstm_chunkwise_fwd(inp.q, inp.k, inp.v, inp.log_i, inp.log_f, return_state=True)
    ref_h, ref_C, ref_n = _oracle_state([np64(t) for t in (inp.q, inp.k, inp.v, inp.log_i, inp.log_f)])
    assert rel_err(np64(full), ref_h) < TOL16
    em = np.exp(np64(m))
    assert rel_err(np64(C) * em[..., None, None], ref_C) < TOL16
    s = 300
    a, st = ops.mlstm_chunkwise_fwd(inp.q[:, :, :s], inp.k[:, :, :s], inp.v[:, :, :s], inp.log_i[:, :, :s],
                                    inp.log_f[:, :, :s], return_state=True)
    b2 = ops.mlstm_chunkwise_fwd(inp.q[:, :, s:], inp.k[:, :, s:], inp.v[:, :, s:], inp.log_i[:, :, s:],
                                 inp.log_f[:, :, s:], *st)
    assert rel_err(np64(torch.cat([a, b2], 2)), ref_h) < TOL16


def test_mlstm_block_bf16_head512_matches_fp32_path(ops):
    """mLSTMBlock with 4 heads x 512 (the prefill's mLSTM layer): bf16 on the
    streaming tensor-core kernel vs the same block in fp32 on the exact
    recurrence (itself pinned to the reference's block output), on the same
    bf16-rounded weights and input: 2e-2."""
    import hybrid_model_mamba_xlstm_b200.layers as Lyr
    torch.manual_seed(3)
    blk = Lyr.mLSTMBlock(256, head_dim=512, num_heads=4).cuda()
    with torch.no_grad():
        for prm in blk.parameters():
            prm.copy_(torch.randn_like(prm).mul_(0.02).to(torch.bfloat16).float())
    x = torch.randn(2, 200, 256, device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        ref = blk.float()(x.float())
        out = blk.to(torch.bfloat16)(x)
    assert rel_err(np64(out), np64(ref)) < TOL16


@pytest.mark.parametrize("path", ["tc_head_gates_d256", "stream_channel_gates_d128", "recurrent_fp32_d64"])
def test_time_strided_views(ops, path):
    """q, k, v, gates and the output in (B, L, H, d) memory passed as (B, H, L, d)
    views (time stride H*d): the layer's projection layout, no transpose copies."""
    g = torch.Generator().manual_seed(31)
    dtype = torch.float32 if path.startswith("recurrent") else torch.bfloat16
    d = {"tc_head_gates_d256": 256, "stream_channel_gates_d128": 128, "recurrent_fp32_d64": 64}[path]
    b, h, L = 2, 3, 200
    blhd = lambda: torch.randn(b, L, h, d, generator=g)
    q = (blhd() / d ** 0.5).to("cuda", dtype).transpose(1, 2)
    k, v = (blhd().to("cuda", dtype).transpose(1, 2) for _ in range(2))
    if path.startswith("tc"):
        li = (torch.randn(b, L, h, generator=g)).cuda().transpose(1, 2)
        lf = torch.nn.functional.logsigmoid(torch.randn(b, L, h, generator=g) + 3).cuda().transpose(1, 2)
    else:
        li = (blhd() * 0.5).cuda().transpose(1, 2)
        lf = torch.nn.functional.logsigmoid(blhd() + 1.0).cuda().transpose(1, 2)
    out_mem = torch.empty(b, L, h, d, device="cuda", dtype=dtype)
    out = ops.mlstm_chunkwise_fwd(q, k, v, li, lf, out=out_mem.transpose(1, 2))
    assert out.data_ptr() == out_mem.data_ptr()
    ref, _, _ = R.tfla_recurrent(np64(q), np64(k), np64(v), np.exp(np64(li)), np.exp(np64(lf)))
    assert rel_err(np64(out), ref) < (TOL32 * 10 if dtype == torch.float32 else TOL16)
