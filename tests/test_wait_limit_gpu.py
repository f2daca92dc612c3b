"""Bounded device waits: a wait that runs out is reported, and the GPU stays usable.

Every mbarrier / cluster wait in the tensor-core kernels (chunkwise mLSTM and
SSD, key-streaming mLSTM, the sLSTM cluster exchange) gives up after
``wait_limit_cycles`` SM cycles (about 2 s by default).  A negative limit
makes the waits run out for certain: in the chunkwise and key-streaming
kernels every wait gives up at once, after the first TMA loads were issued;
in the sLSTM cluster kernel every CTA waits (for -limit cycles) on the first
exchange before any CTA sends it.  The kernel then raises its abort flag,
drains what it has in flight (its own MMAs and loads, on a separate bound),
frees its TMEM, sets the caller's error word and returns.  The test checks
the word on the host, that the CUDA context reports no error, and that the
next call with the default limit gives the same result as before.  No
fault, trap or hang is involved.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
GIVE_UP = -100000  # negative: the waits run out (the sLSTM exchange after 1e5 cycles, ~50 us)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)


def _run_three(fn):
    """fn(error_flag, wait_limit_cycles) -> tensors; default limit, GIVE_UP, default again."""
    flag = torch.zeros(1, device="cuda", dtype=torch.int32)
    first = [t.clone() for t in fn(flag, 0)]
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    fn(flag, GIVE_UP)
    torch.cuda.synchronize()  # raises if the context had faulted
    assert int(flag.item()) == 1
    flag.zero_()
    again = fn(flag, 0)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    for a, b in zip(first, again):
        assert torch.equal(a, b)


@pytest.mark.parametrize("d,per_channel", [(128, False), (256, False), (128, True), (512, False)])
def test_mlstm_wait_runs_out(dev, d, per_channel):
    """d 128 / 256 per-head: tcgen05 chunkwise kernel; per-channel or d 512:
    key-streaming kernel."""
    from hybrid_model_mamba_xlstm_b200.kernels.tfla.tfla_interface import mlstm_chunkwise_fwd
    g = torch.Generator().manual_seed(d)
    b, h, L = 1, 2, 384
    q = (torch.randn(b, h, L, d, generator=g) / d ** 0.5).to(dev, torch.bfloat16)
    k, v = (torch.randn(b, h, L, d, generator=g).to(dev, torch.bfloat16) for _ in range(2))
    gs = (b, h, L, d) if per_channel else (b, h, L)
    li = torch.randn(*gs, generator=g).to(dev)
    lf = torch.nn.functional.logsigmoid(torch.randn(*gs, generator=g) + 3.0).to(dev)

    def fn(flag, lim):
        out, st = mlstm_chunkwise_fwd(q, k, v, li, lf, return_state=True, error_flag=flag, wait_limit_cycles=lim)
        return (out, *st)
    _run_three(fn)


def test_ssd_wait_runs_out(dev):
    from hybrid_model_mamba_xlstm_b200.kernels.ssd import ssd_chunk_scan
    from hybrid_model_mamba_xlstm_b200.workloads import ssd_inputs
    inp = ssd_inputs(1, 512, 2, 64, 128, seed=3, device="cuda")

    def fn(flag, lim):
        return ssd_chunk_scan(inp.x, inp.dt, inp.A, inp.B, inp.C, inp.D, error_flag=flag, wait_limit_cycles=lim)
    _run_three(fn)


def test_slstm_cluster_wait_runs_out(dev):
    """head_dim 128 with recurrent weights: the 8-CTA cluster kernel, whose
    per-step exchanges between the CTAs are the bounded waits."""
    from hybrid_model_mamba_xlstm_b200.kernels.slstm import slstm_scan
    g = torch.Generator().manual_seed(5)
    b, L, h, hd = 2, 64, 2, 128
    gates = torch.randn(b, L, h, 4, hd, generator=g).to(dev, torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hd, generator=g)).to(dev)
    R = (torch.randn(h, hd, 4 * hd, generator=g) / 16).to(dev, torch.bfloat16)

    def fn(flag, lim):
        out, st = slstm_scan(gates, w, R=R, error_flag=flag, wait_limit_cycles=lim)
        return (out, *st)
    _run_three(fn)
