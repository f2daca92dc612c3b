"""C-ABI library checks that need no GPU: it loads, exports every symbol the
header declares, reports its ABI version and rejects malformed arguments
with HXM_EBADARG before touching CUDA."""
import ctypes as ct
import os
import re

import pytest

from hybrid_model_mamba_xlstm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            text = open(os.path.join(ROOT, "include", f)).read()
            names |= set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(hxm_[a-z0-9_]+)\s*\(", text, re.M))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    declared = _declared_symbols()
    assert {"hxm_selective_scan_fwd", "hxm_mlstm_chunkwise_fwd", "hxm_ssd_chunk_scan_fwd",
            "hxm_slstm_scan_fwd", "hxm_last_error_string", "hxm_abi_version"} <= declared
    for name in declared:
        assert hasattr(lib, name), name
    assert set(_lib.SYMBOLS) >= declared


def test_abi_version():
    assert _lib.lib().hxm_abi_version() == 1


def test_struct_sizes_match_header_layout():
    # the C side checks struct_size == sizeof(struct); a mismatch is HXM_EBADARG
    for cls, fn in [(_lib.ScanArgs, "hxm_selective_scan_fwd"), (_lib.MlstmArgs, "hxm_mlstm_chunkwise_fwd"),
                    (_lib.SsdArgs, "hxm_ssd_chunk_scan_fwd"), (_lib.SlstmArgs, "hxm_slstm_scan_fwd"),
                    (_lib.ConvArgs, "hxm_causal_conv1d_fwd"), (_lib.RmsnormArgs, "hxm_rmsnorm_fwd"),
                    (_lib.MlstmGatesArgs, "hxm_mlstm_gate_prologue"), (_lib.MlstmGatesArgs, "hxm_mlstm_gate_epilogue"),
                    (_lib.ScanBwdArgs, "hxm_selective_scan_bwd"), (_lib.MlstmBwdArgs, "hxm_mlstm_bwd_prepare"),
                    (_lib.MlstmBwdArgs, "hxm_mlstm_bwd_finalize"), (_lib.ChunkScanArgs, "hxm_chunk_state_scan"),
                    (_lib.MlstmBwdNormArgs, "hxm_mlstm_bwd_normalizer"), (_lib.ChunkDotArgs, "hxm_chunk_state_dot"),
                    (_lib.SsdBwdIntraArgs, "hxm_ssd_bwd_intra"), (_lib.SsdBwdRowsArgs, "hxm_ssd_bwd_rows"),
                    (_lib.ChunkGemmArgs, "hxm_chunk_gemm")]:
        a = cls()
        a.struct_size = ct.sizeof(a) + 8
        st = getattr(_lib.lib(), fn)(ct.byref(a), None)
        assert st == _lib.HXM_EBADARG, fn
        assert b"struct_size" in _lib.lib().hxm_last_error_string()


def test_scan_rejects_bad_arguments_without_cuda():
    lib = _lib.lib()
    assert lib.hxm_selective_scan_fwd(None, None) == _lib.HXM_EBADARG
    a = _lib.ScanArgs()
    a.struct_size = ct.sizeof(a)
    a.batch, a.seqlen, a.dim, a.dstate = 1, 4, 8, 0  # dstate 0 invalid
    assert lib.hxm_selective_scan_fwd(ct.byref(a), None) == _lib.HXM_EBADARG
    a.dstate = 65
    assert lib.hxm_selective_scan_fwd(ct.byref(a), None) == _lib.HXM_EUNSUPPORTED
    a.dstate, a.z_mode = 16, 2  # silu gate without z
    assert lib.hxm_selective_scan_fwd(ct.byref(a), None) == _lib.HXM_EBADARG
    a.z_mode, a.io_dtype = 0, 7
    assert lib.hxm_selective_scan_fwd(ct.byref(a), None) == _lib.HXM_EBADARG
    # empty batch is a no-op success (nothing is launched)
    a.io_dtype, a.batch = _lib.HXM_F32, 0
    assert lib.hxm_selective_scan_fwd(ct.byref(a), None) == _lib.HXM_OK


def test_python_wrapper_refuses_cpu_tensors():
    import torch
    from hybrid_model_mamba_xlstm_b200.kernels import selective_scan
    x = torch.zeros(1, 4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        selective_scan(x, x, torch.zeros(8, 16), torch.zeros(1, 4, 16), torch.zeros(1, 4, 16), torch.ones(8))


def test_conv_rejects_bad_arguments_without_cuda():
    lib = _lib.lib()
    assert lib.hxm_causal_conv1d_fwd(None, None) == _lib.HXM_EBADARG
    a = _lib.ConvArgs()
    a.struct_size = ct.sizeof(a)
    a.batch, a.seqlen, a.channels, a.width, a.io_dtype = 1, 4, 8, 5, _lib.HXM_BF16
    assert lib.hxm_causal_conv1d_fwd(ct.byref(a), None) == _lib.HXM_EUNSUPPORTED   # width > 4
    a.width, a.activation = 4, 3
    assert lib.hxm_causal_conv1d_fwd(ct.byref(a), None) == _lib.HXM_EBADARG
    a.activation = 1
    assert lib.hxm_causal_conv1d_fwd(ct.byref(a), None) == _lib.HXM_EBADARG        # NULL weight
    a.batch = 0
    assert lib.hxm_causal_conv1d_fwd(ct.byref(a), None) == _lib.HXM_OK


def test_mlstm_backward_entries_validate_without_cuda():
    """The ctypes layouts of the backward structs match the header (the size
    check passes and the next check fires), bad sizes are rejected and empty
    work is a no-op success."""
    lib = _lib.lib()
    a = _lib.MlstmBwdArgs()
    a.struct_size = ct.sizeof(a)
    a.batch, a.heads, a.seqlen, a.dqk, a.chunk = 1, 1, 8, 4, 0
    for fn in ("hxm_mlstm_bwd_prepare", "hxm_mlstm_bwd_finalize"):
        assert getattr(lib, fn)(ct.byref(a), None) == _lib.HXM_EBADARG
        assert b"chunk" in lib.hxm_last_error_string()
    a.chunk, a.gate_mode = 4, 2
    assert lib.hxm_mlstm_bwd_prepare(ct.byref(a), None) == _lib.HXM_EBADARG
    assert b"gate_mode" in lib.hxm_last_error_string()
    s = _lib.ChunkScanArgs()
    s.struct_size = ct.sizeof(s)
    s.groups, s.nchunks, s.rows, s.cols = 1, 3, 0, 4
    assert lib.hxm_chunk_state_scan(ct.byref(s), None) == _lib.HXM_EBADARG
    assert b"rows=0" in lib.hxm_last_error_string()
    s.rows, s.groups = 2, 0
    assert lib.hxm_chunk_state_scan(ct.byref(s), None) == _lib.HXM_OK
    s.groups, s.cols, s.x, s.scaled_hi, s.dot_hi, s.dot_out = 1, 6, 1 << 20, 1 << 20, 1 << 20, 1 << 20
    assert lib.hxm_chunk_state_scan(ct.byref(s), None) == _lib.HXM_EUNSUPPORTED  # row mode needs cols % 4 == 0
    assert b"row mode" in lib.hxm_last_error_string()
    n = _lib.MlstmBwdNormArgs()
    n.struct_size = ct.sizeof(n)
    n.batch, n.heads, n.seqlen, n.padded_len, n.dv, n.width, n.normalize = 1, 1, 8, 4, 4, 8, 1
    assert lib.hxm_mlstm_bwd_normalizer(ct.byref(n), None) == _lib.HXM_EBADARG  # padded_len < seqlen
    assert b"padded_len=4" in lib.hxm_last_error_string()
    n.padded_len, n.width = 8, 4  # no room for the den column
    assert lib.hxm_mlstm_bwd_normalizer(ct.byref(n), None) == _lib.HXM_EBADARG
    n.width, n.batch = 8, 0
    assert lib.hxm_mlstm_bwd_normalizer(ct.byref(n), None) == _lib.HXM_OK


def test_chunk_gemm_validates_without_cuda():
    """hxm_chunk_gemm: the ctypes layout matches (the size check passes and the
    next check fires), shape mismatches and misaligned strides are rejected,
    empty work is a no-op success."""
    lib = _lib.lib()
    a = _lib.ChunkGemmArgs()
    a.struct_size = ct.sizeof(a)
    a.groups, a.m, a.n, a.nprod = 2, 128, 64, 5
    assert lib.hxm_chunk_gemm(ct.byref(a), None) == _lib.HXM_EBADARG
    assert b"nprod" in lib.hxm_last_error_string()
    a.nprod = 1
    assert lib.hxm_chunk_gemm(ct.byref(a), None) == _lib.HXM_EBADARG  # no output
    assert b"no output" in lib.hxm_last_error_string()
    a.out = 4096
    for o, (rows, cols, trans) in ((a.a[0], (128, 96, 0)), (a.b[0], (96, 64, 0))):
        o.ptr, o.rows, o.cols, o.trans = 1 << 20, rows, cols, trans
        o.row_stride, o.group_stride = cols, rows * cols
    a.b[0].rows = 80  # inner lengths 96 vs 80
    assert lib.hxm_chunk_gemm(ct.byref(a), None) == _lib.HXM_EBADARG
    assert b"inner lengths" in lib.hxm_last_error_string()
    a.b[0].rows, a.a[0].row_stride = 96, 100  # row stride not a multiple of 8 elements
    assert lib.hxm_chunk_gemm(ct.byref(a), None) == _lib.HXM_EBADARG
    assert b"multiples of 8" in lib.hxm_last_error_string()
    a.a[0].row_stride, a.a[0].trans = 96, 1  # op(A) = 96 x 128: m mismatch
    assert lib.hxm_chunk_gemm(ct.byref(a), None) == _lib.HXM_EBADARG
    assert b"rows for m" in lib.hxm_last_error_string()
    a.a[0].trans, a.groups = 0, 0
    assert lib.hxm_chunk_gemm(ct.byref(a), None) == _lib.HXM_OK


def test_scan_workspace_query_without_a_gpu():
    """hxm_selective_scan_workspace_size: the fast path's time segments need
    scratch only for a long sequence on a small grid (one batch row x 256
    channels x 8192 steps), none for a short sequence, a large grid, fp32 or
    the ZOH rule, and bad args report 0."""
    lib = _lib.lib()
    a = _lib.ScanArgs()
    a.struct_size = ct.sizeof(a)
    a.batch, a.seqlen, a.dim, a.dstate, a.io_dtype = 1, 8192, 256, 16, _lib.HXM_BF16
    base = 1 << 20  # aligned placeholders: the query reads no memory
    for f in ("u", "delta", "B", "C", "y", "A"):
        setattr(a, f, base)
    a.u_stride = a.delta_stride = a.y_stride = (256 * 8192, 1, 8192)  # time-major (b, t, d) view
    a.B_stride = a.C_stride = (16 * 8192, 1, 8192)
    small = lib.hxm_selective_scan_workspace_size(ct.byref(a))
    assert small > 0 and small % (17 * 4 * 256) == 0
    a.seqlen = 4096  # short sequences run one pass
    assert lib.hxm_selective_scan_workspace_size(ct.byref(a)) == 0
    a.seqlen = 8192
    a.batch = 128  # 512 CTAs of 64 channels: over 2 per SM on 148 SMs
    assert lib.hxm_selective_scan_workspace_size(ct.byref(a)) == 0
    a.batch, a.discretization = 1, 1
    assert lib.hxm_selective_scan_workspace_size(ct.byref(a)) == 0
    a.discretization, a.struct_size = 0, 8
    assert lib.hxm_selective_scan_workspace_size(ct.byref(a)) == 0
