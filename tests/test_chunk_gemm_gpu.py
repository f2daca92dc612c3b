"""hxm_chunk_gemm (tcgen05 batched chunk GEMM) against float64 matmul of the
same bf16 operands: every transpose combination, two products with different
inner lengths, ragged m / n / K (tiles partly past the stored extent), the
causal mask and decay weighting, accumulation, fp32 and bf16 stores, strided
views, and a bounded wait that runs out (error word set, no fault).

Tolerance: the products of bf16 operands are exact in fp32, so only the
accumulation order differs from float64: 1e-5 normwise relative error (fp32
output); bf16 output within bf16 rounding (4e-3)."""
import numpy as np
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cg():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from hybrid_model_mamba_xlstm_b200.kernels.chunk_gemm import chunk_gemm
    return chunk_gemm


def _mat(g, rows, cols, seed, scale=1.0):
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn(g, rows, cols, generator=gen) * scale).to("cuda", torch.bfloat16)


def _ref(products, alpha=1.0, mask=False, decay=None, acc=None):
    d = None
    for A, ta, B, tb in products:
        a = A.double().cpu()
        b = B.double().cpu()
        a = a.transpose(1, 2) if ta else a
        b = b.transpose(1, 2) if tb else b
        d = a @ b if d is None else d + a @ b
    d = d * alpha
    if mask:
        m, n = d.shape[1:]
        keep = torch.arange(n)[None, :] <= torch.arange(m)[:, None]
        if decay is not None:
            bd = decay.double().cpu()
            w = torch.exp(bd[:, :, None] - bd[:, None, :n])
            d = d * torch.where(keep, w, torch.zeros_like(w))
        else:
            d = d * keep
    if acc is not None:
        d = d + acc.double().cpu()
    return d.numpy()


def _stored(shape_mk, trans):
    """Stored (rows, cols) of an op() of logical shape shape_mk."""
    r, c = shape_mk
    return (c, r) if trans else (r, c)


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(128, 128, 128), (128, 64, 192), (64, 200, 72), (256, 528, 520)])
def test_single_product(cg, ta, tb, m, n, k):
    g = 3
    A = _mat(g, *_stored((m, k), ta), seed=m + k)
    B = _mat(g, *_stored((k, n), tb), seed=n + 7)
    out, _ = cg([(A, ta, B, tb)])
    torch.cuda.synchronize()
    assert rel_err(out.cpu().double().numpy(), _ref([(A, ta, B, tb)])) < 1e-5


def test_two_products_ragged_and_bf16_out(cg):
    """dQ = dS K + dN X^T shape: (c x c)(c x dqk) + (c x w)(w x dqk), w = 264."""
    g, c, dqk, w = 5, 128, 256, 264
    dS = _mat(g, c, c, 1)
    K = _mat(g, c, dqk, 2)
    dN = _mat(g, c, w, 3)
    X = _mat(g, dqk, w, 4)
    prods = [(dS, 0, K, 0), (dN, 0, X, 1)]
    outb = torch.empty(g, c, dqk, device="cuda", dtype=torch.bfloat16)
    out, _ = cg(prods, out=torch.empty(g, c, dqk, device="cuda"), out_bf16=outb, alpha=0.5)
    torch.cuda.synchronize()
    ref = _ref(prods, alpha=0.5)
    assert rel_err(out.cpu().double().numpy(), ref) < 1e-5
    assert rel_err(outb.float().cpu().double().numpy(), ref) < 4e-3


@pytest.mark.parametrize("c", [128, 64])
def test_causal_mask_decay_and_accumulate(cg, c):
    """S = causal(Q K^T) * exp(b_t - b_s) (the per-head decay matrix), then an
    accumulating product into an existing output."""
    g, d = 4, 128
    Q = _mat(g, c, d, 11, 0.2)
    K = _mat(g, c, d, 12)
    gen = torch.Generator().manual_seed(13)
    b = torch.nn.functional.logsigmoid(torch.randn(g, c, generator=gen) + 2).cumsum(-1).cuda()
    S, Sb = cg([(Q, 0, K, 1)], out=torch.empty(g, c, c, device="cuda"),
               out_bf16=torch.empty(g, c, c, device="cuda", dtype=torch.bfloat16), mask=True, decay=b)
    torch.cuda.synchronize()
    ref = _ref([(Q, 0, K, 1)], mask=True, decay=b)
    assert rel_err(S.cpu().double().numpy(), ref) < 1e-5
    assert rel_err(Sb.float().cpu().double().numpy(), ref) < 4e-3
    assert (np.triu(S.cpu().numpy(), 1) == 0).all()
    # out += S^T V (S read transposed from its bf16 copy)
    V = _mat(g, c, 96, 14)
    acc = torch.randn(g, c, 96, device="cuda")
    before = acc.clone()
    cg([(Sb, 1, V, 0)], out=acc, accumulate=True)
    torch.cuda.synchronize()
    assert rel_err(acc.cpu().double().numpy(), _ref([(Sb, 1, V, 0)], acc=before)) < 1e-5


def test_strided_views(cg):
    """Operands and output as views of wider buffers (row / group strides
    larger than the extent)."""
    g, m, n, k = 3, 128, 128, 64
    Abuf = _mat(g, m, k + 64, 21)
    Bbuf = _mat(g + 1, k, n + 32, 22)
    A = Abuf[:, :, 32:32 + k]
    B = Bbuf[1:, :, :n]
    obuf = torch.zeros(g, m, n + 16, device="cuda")
    out = obuf[:, :, 8:8 + n]
    cg([(A, 0, B, 0)], out=out)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().double().numpy(), _ref([(A, 0, B, 0)])) < 1e-5
    assert (obuf[:, :, :8] == 0).all() and (obuf[:, :, 8 + n:] == 0).all()


def test_wait_runs_out(cg):
    """A negative wait limit makes the bounded waits give up at once: the
    error word is set, the context stays usable and the next call matches."""
    g = 2
    A = _mat(g, 128, 128, 31)
    B = _mat(g, 128, 128, 32)
    flag = torch.zeros(1, device="cuda", dtype=torch.int32)
    first, _ = cg([(A, 0, B, 1)], error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    cg([(A, 0, B, 1)], error_flag=flag, wait_limit_cycles=-100000)
    torch.cuda.synchronize()
    assert int(flag.item()) == 1
    flag.zero_()
    again, _ = cg([(A, 0, B, 1)], error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0 and torch.equal(first, again)


def test_split_output_and_accumulate_into_bf16(cg):
    """out_bf16 / out_bf16_lo: high + low parts reproduce the fp32 result to
    ~2^-16; with accumulate every output holds the accumulated sum."""
    g, m, n, k = 3, 128, 192, 128
    A = _mat(g, m, k, 41)
    B = _mat(g, k, n, 42)
    acc = torch.randn(g, m, n, device="cuda")
    before = acc.clone()
    hi = torch.empty(g, m, n, device="cuda", dtype=torch.bfloat16)
    lo = torch.empty_like(hi)
    cg([(A, 0, B, 0)], out=acc, out_bf16=hi, out_bf16_lo=lo, accumulate=True)
    torch.cuda.synchronize()
    ref = _ref([(A, 0, B, 0)], acc=before)
    assert rel_err(acc.cpu().double().numpy(), ref) < 1e-5
    assert rel_err(hi.float().cpu().double().numpy(), ref) < 4e-3
    both = hi.double() + lo.double()
    assert rel_err(both.cpu().numpy(), acc.cpu().double().numpy()) < 2e-5
