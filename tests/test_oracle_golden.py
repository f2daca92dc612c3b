"""Pin the oracle: numpy restatements vs golden vectors made by the reference.

The fixtures were produced by running the reference package itself in float64
(tests/golden/make_golden.py).  Agreement here is to float64 rounding (1e-12),
which is what makes the oracle a valid stand-in for the reference.
"""
import numpy as np
import pytest

from oracle import numpy_ref as R
from tests.conftest import rel_err

TOL64 = 1e-12


def test_scan_small_matches_reference(golden):
    g = golden("scan_small")
    y, _ = R.selective_scan(g["x"], g["dt"], g["A"], g["B"], g["C"], g["D"])
    assert rel_err(y, g["y"]) < TOL64
    yz, _ = R.selective_scan(g["x"], g["dt"], g["A"], g["B"], g["C"], g["D"], z=g["z"], z_mode="mul")
    assert rel_err(yz, g["y_z"]) < TOL64


def test_scan_zoh_matches_reference(golden):
    """The ZOH / Taylor rule against MambaBlock._selective_scan_pytorch of the
    v2 block (mamba_block_v2.py:280-351), both branches present."""
    g = golden("scan_zoh")
    assert 0.02 < float(g["taylor_fraction"]) < 0.98
    y, _ = R.selective_scan(g["x"], g["delta"], g["A"], g["B"], g["C"], g["D"], discretization="zoh")
    assert rel_err(y, g["y"]) < TOL64


def test_scan_cfg1_slice_matches_reference(golden):
    g = golden("scan_cfg1_slice")
    t = lambda a: np.swapaxes(a, 1, 2)
    y, _ = R.selective_scan(t(g["u"]), t(g["raw"]), g["A"], t(g["B"]), t(g["C"]), g["D"], z=t(g["z"]),
                            z_mode="silu", delta_bias=g["bias"], delta_softplus=True)
    assert rel_err(y, t(g["y"])) < TOL64


def test_scan_final_state_and_segmenting():
    """h_final restated: running two halves with the carried state equals one pass."""
    rng = np.random.default_rng(0)
    bt, L, dm, n = 2, 40, 8, 4
    x, dt = rng.standard_normal((bt, L, dm)), np.abs(rng.standard_normal((bt, L, dm))) * 0.1
    A = -np.exp(rng.standard_normal((dm, n)))
    B, C = rng.standard_normal((bt, L, n)), rng.standard_normal((bt, L, n))
    for disc in ("euler", "zoh"):
        y, h = R.selective_scan(x, dt, A, B, C, None, discretization=disc)
        y1, h1 = R.selective_scan(x[:, :17], dt[:, :17], A, B[:, :17], C[:, :17], None, discretization=disc)
        y2, h2 = R.selective_scan(x[:, 17:], dt[:, 17:], A, B[:, 17:], C[:, 17:], None, discretization=disc, h0=h1)
        assert rel_err(np.concatenate([y1, y2], 1), y) < 1e-13
        assert rel_err(h2, h) < 1e-13


@pytest.mark.parametrize("name", ["tfla_1x2x16x8", "tfla_2x4x32x16", "tfla_2x4x64x32"])
def test_tfla_channel_gates_match_reference(golden, name):
    g = golden(name)
    h, _, _ = R.tfla_recurrent(g["q"], g["k"], g["v"], np.exp(g["i_pre"].astype(np.float64)),
                               R.sigmoid(g["f_pre"]))
    assert rel_err(h, g["h"]) < TOL64


def test_tfla_scalar_gates_match_reference(golden):
    g = golden("tfla_scalar_gates")
    h, _, _ = R.tfla_recurrent(g["q"], g["k"], g["v"], np.exp(g["i_pre"].astype(np.float64)),
                               R.sigmoid(g["f_pre"]))
    assert rel_err(h, g["h"]) < TOL64


def test_slstm_matches_reference_block(golden):
    g = golden("slstm_block")
    nh, hd = int(g["heads"]), int(g["head_dim"])
    bsz, L, _ = g["gates"].shape
    gates = g["gates"].reshape(bsz, L, nh, 4, hd)
    h_seq, h, c = R.slstm_recurrent(gates, g["norm_w"])
    assert rel_err(h_seq.reshape(bsz, L, nh * hd), g["h_seq"]) < TOL64
    assert rel_err(h, g["h"]) < TOL64
    assert rel_err(c, g["c"]) < TOL64


def test_ssd_equals_headwise_scan():
    """SSD restatement == per-head loop of the reference Euler recurrence."""
    rng = np.random.default_rng(1)
    bt, L, nh, p, n = 1, 12, 2, 3, 4
    x = rng.standard_normal((bt, L, nh, p))
    dt = np.abs(rng.standard_normal((bt, L, nh))) * 0.2
    A = -rng.uniform(1, 4, nh)
    B, C = rng.standard_normal((bt, L, n)), rng.standard_normal((bt, L, n))
    y, h = R.ssd_scan(x, dt, A, B, C, np.ones(nh))
    hh = np.zeros((bt, nh, p, n))
    for t in range(L):
        for hi in range(nh):
            hh[:, hi] = np.exp(dt[:, t, hi] * A[hi])[:, None, None] * hh[:, hi] + \
                (dt[:, t, hi, None] * x[:, t, hi])[:, :, None] * B[:, t, None, :]
            yt = np.einsum("bpn,bn->bp", hh[:, hi], C[:, t]) + x[:, t, hi]
            assert np.allclose(yt, y[:, t, hi], rtol=1e-12, atol=1e-12)
    assert np.allclose(h, hh, rtol=1e-12, atol=1e-12)


def test_slstm_recurrent_R_zero_is_reference():
    rng = np.random.default_rng(2)
    g = rng.standard_normal((1, 9, 2, 4, 8))
    w = rng.uniform(0.5, 1.5, 8)
    a = R.slstm_recurrent(g, w)
    b = R.slstm_recurrent(g, w, R=np.zeros((2, 8, 32)))
    for u, v in zip(a, b):
        assert np.array_equal(u, v)


def test_conv_matches_reference(golden):
    """The conv restatement reproduces the reference MambaBlock's conv + SiLU."""
    g = golden("conv_block")
    out, fin = R.causal_conv1d(g["x_inner"], g["weight"], g["bias"], activation="silu")
    assert rel_err(out, g["conv_silu"]) < TOL64
    assert np.array_equal(fin, np.swapaxes(g["x_inner"][:, -3:, :], 1, 2))


def test_conv_continuation():
    """Running two halves with the carried state equals one pass (the state is the last width-1 inputs)."""
    rng = np.random.default_rng(1)
    x, w, b = rng.standard_normal((2, 30, 6)), rng.standard_normal((6, 4)), rng.standard_normal(6)
    whole, fin = R.causal_conv1d(x, w, b, activation="silu")
    a, s = R.causal_conv1d(x[:, :11], w, b, activation="silu")
    c, fin2 = R.causal_conv1d(x[:, 11:], w, b, activation="silu", init_state=s)
    assert np.allclose(np.concatenate([a, c], 1), whole, rtol=0, atol=1e-12)
    assert np.array_equal(fin, fin2)
