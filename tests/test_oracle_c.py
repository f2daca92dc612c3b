"""The C oracle (timed CPU baseline, fast checker) agrees with the numpy
oracle, which the golden vectors pin to the reference."""
import numpy as np

from oracle import build as C
from oracle import numpy_ref as R
from tests.conftest import rel_err


def test_c_scan_matches_numpy_all_modes():
    rng = np.random.default_rng(0)
    b, d, L, n = 2, 12, 70, 16
    u, z = rng.standard_normal((b, d, L)), rng.standard_normal((b, d, L))
    raw = rng.standard_normal((b, d, L)) * 0.5 - 3
    bias = rng.standard_normal(d) * 0.1
    A = -np.exp(rng.standard_normal((d, n)))
    B, Cm = rng.standard_normal((b, n, L)), rng.standard_normal((b, n, L))
    D = rng.standard_normal(d)
    h0 = rng.standard_normal((b, d, n))
    t = lambda a: np.swapaxes(a, 1, 2)
    for disc, dname in ((0, "euler"), (1, "zoh")):
        for zm, zname in ((0, None), (1, "mul"), (2, "silu")):
            y, h = C.scan(u, raw, A, B, Cm, D, z if zm else None, bias, True, zm, disc, h0)
            yr, hr = R.selective_scan(t(u), t(raw), A, t(B), t(Cm), D, z=t(z) if zm else None,
                                      z_mode=zname or "mul", delta_bias=bias, delta_softplus=True,
                                      discretization=dname, h0=h0)
            assert rel_err(t(y), yr) < 1e-5
            assert rel_err(h, hr) < 1e-5


def test_c_mlstm_matches_golden(golden):
    for name in ("tfla_2x4x32x16", "tfla_scalar_gates"):
        g = golden(name)
        ig = np.exp(g["i_pre"].astype(np.float64))
        fg = R.sigmoid(g["f_pre"])
        h, Cs, ns = C.mlstm(g["q"], g["k"], g["v"], ig, fg)
        assert rel_err(h, g["h"]) < 1e-4
        _, Cr, nr = R.tfla_recurrent(g["q"], g["k"], g["v"], ig, fg)
        assert rel_err(Cs, Cr) < 1e-5 and rel_err(ns, nr) < 1e-5


def test_c_slstm_matches_golden_and_R():
    rng = np.random.default_rng(3)
    g = rng.standard_normal((2, 30, 3, 4, 16))
    w = rng.uniform(0.5, 1.5, 16)
    Rm = rng.standard_normal((3, 16, 64)) / 16
    for Rx in (None, Rm):
        out, h, c = C.slstm(g, w, Rx)
        outr, hr, cr = R.slstm_recurrent(g, w, R=Rx)
        assert rel_err(out, outr) < 1e-5 and rel_err(h, hr) < 1e-5 and rel_err(c, cr) < 1e-5
