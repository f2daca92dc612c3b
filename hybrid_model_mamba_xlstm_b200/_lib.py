"""ctypes binding of libhxm.so (include/hxm.h).

The library is the product: every public op in this package ends in one of
these C-ABI calls.  There is no CPU fallback — if the library is missing or
a CUDA device is absent, calls raise.
"""
from __future__ import annotations

import ctypes as ct
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("HXM_LIB", os.path.join(_HERE, "lib", "libhxm.so"))

HXM_OK, HXM_EBADARG, HXM_EUNSUPPORTED, HXM_ECUDA, HXM_ETIMEOUT = range(5)
_STATUS = {0: "HXM_OK", 1: "HXM_EBADARG", 2: "HXM_EUNSUPPORTED", 3: "HXM_ECUDA", 4: "HXM_ETIMEOUT"}
HXM_F32, HXM_BF16, HXM_F16 = 0, 1, 2

_i64x3 = ct.c_int64 * 3
_i64x2 = ct.c_int64 * 2


class ScanArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("batch", ct.c_int32), ("seqlen", ct.c_int32), ("dim", ct.c_int32), ("dstate", ct.c_int32),
        ("io_dtype", ct.c_int),
        ("u", ct.c_void_p), ("u_stride", _i64x3),
        ("delta", ct.c_void_p), ("delta_stride", _i64x3),
        ("A", ct.c_void_p), ("A_stride", _i64x2),
        ("B", ct.c_void_p), ("B_stride", _i64x3),
        ("C", ct.c_void_p), ("C_stride", _i64x3),
        ("D", ct.c_void_p),
        ("z", ct.c_void_p), ("z_stride", _i64x3),
        ("delta_bias", ct.c_void_p),
        ("y", ct.c_void_p), ("y_stride", _i64x3),
        ("h0", ct.c_void_p),
        ("hT", ct.c_void_p),
        ("z_mode", ct.c_int32), ("delta_softplus", ct.c_int32), ("discretization", ct.c_int32),
        ("workspace", ct.c_void_p), ("workspace_bytes", ct.c_size_t),
    ]


class ScanBwdArgs(ct.Structure):
    _fields_ = [
        ("fwd", ScanArgs),
        ("struct_size", ct.c_size_t),
        ("dout", ct.c_void_p), ("dout_stride", _i64x3),
        ("du", ct.c_void_p), ("ddelta", ct.c_void_p), ("dz", ct.c_void_p),
        ("dA", ct.c_void_p), ("dB", ct.c_void_p), ("dC", ct.c_void_p), ("dD", ct.c_void_p),
        ("ddelta_bias", ct.c_void_p), ("dh0", ct.c_void_p),
        ("workspace", ct.c_void_p), ("workspace_bytes", ct.c_size_t),
    ]


class MlstmArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("batch", ct.c_int32), ("heads", ct.c_int32), ("seqlen", ct.c_int32), ("dqk", ct.c_int32),
        ("dv", ct.c_int32), ("chunk", ct.c_int32), ("gate_mode", ct.c_int32),
        ("io_dtype", ct.c_int),
        ("q", ct.c_void_p), ("q_stride", _i64x2),
        ("k", ct.c_void_p), ("k_stride", _i64x2),
        ("v", ct.c_void_p), ("v_stride", _i64x2),
        ("log_i", ct.c_void_p), ("i_stride", _i64x2),
        ("log_f", ct.c_void_p), ("f_stride", _i64x2),
        ("h", ct.c_void_p), ("h_stride", _i64x2),
        ("C0", ct.c_void_p), ("n0", ct.c_void_p), ("m0", ct.c_void_p),
        ("CT", ct.c_void_p), ("nT", ct.c_void_p), ("mT", ct.c_void_p),
        ("workspace", ct.c_void_p), ("workspace_bytes", ct.c_size_t),
        ("q_tstride", ct.c_int64), ("k_tstride", ct.c_int64), ("v_tstride", ct.c_int64),
        ("h_tstride", ct.c_int64), ("i_tstride", ct.c_int64), ("f_tstride", ct.c_int64),
        ("error_flag", ct.c_void_p), ("wait_limit_cycles", ct.c_int64),
    ]


class SsdArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("batch", ct.c_int32), ("seqlen", ct.c_int32), ("heads", ct.c_int32), ("headdim", ct.c_int32),
        ("dstate", ct.c_int32), ("chunk", ct.c_int32),
        ("io_dtype", ct.c_int),
        ("x", ct.c_void_p), ("dt", ct.c_void_p), ("A", ct.c_void_p),
        ("B", ct.c_void_p), ("C", ct.c_void_p),
        ("D", ct.c_void_p), ("dt_bias", ct.c_void_p), ("dt_softplus", ct.c_int32),
        ("y", ct.c_void_p), ("h0", ct.c_void_p), ("hT", ct.c_void_p),
        ("workspace", ct.c_void_p), ("workspace_bytes", ct.c_size_t),
        ("error_flag", ct.c_void_p), ("wait_limit_cycles", ct.c_int64),
    ]


class SlstmArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("batch", ct.c_int32), ("seqlen", ct.c_int32), ("heads", ct.c_int32), ("head_dim", ct.c_int32),
        ("io_dtype", ct.c_int),
        ("gates_pre", ct.c_void_p), ("R", ct.c_void_p), ("norm_weight", ct.c_void_p),
        ("eps", ct.c_float), ("exponential_gate", ct.c_int32),
        ("h_out", ct.c_void_p),
        ("h0", ct.c_void_p), ("c0", ct.c_void_p),
        ("hT", ct.c_void_p), ("cT", ct.c_void_p),
        ("error_flag", ct.c_void_p), ("wait_limit_cycles", ct.c_int64),
    ]


class ConvArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("batch", ct.c_int32), ("seqlen", ct.c_int32), ("channels", ct.c_int32), ("width", ct.c_int32),
        ("io_dtype", ct.c_int),
        ("x", ct.c_void_p), ("x_stride", ct.c_int64 * 3),
        ("weight", ct.c_void_p), ("bias", ct.c_void_p),
        ("out", ct.c_void_p), ("out_stride", ct.c_int64 * 3),
        ("init_state", ct.c_void_p), ("final_state", ct.c_void_p),
        ("activation", ct.c_int32),
    ]


class RmsnormArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("rows", ct.c_int64), ("dim", ct.c_int32),
        ("io_dtype", ct.c_int),
        ("x", ct.c_void_p), ("x_row_stride", ct.c_int64),
        ("residual", ct.c_void_p), ("residual_row_stride", ct.c_int64),
        ("sum_out", ct.c_void_p), ("sum_row_stride", ct.c_int64),
        ("weight", ct.c_void_p), ("eps", ct.c_float),
        ("out", ct.c_void_p), ("out_row_stride", ct.c_int64),
    ]


class MlstmGatesArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("rows", ct.c_int64), ("dim", ct.c_int32),
        ("io_dtype", ct.c_int),
        ("i_pre", ct.c_void_p), ("i_row_stride", ct.c_int64),
        ("f_pre", ct.c_void_p), ("f_row_stride", ct.c_int64),
        ("log_i", ct.c_void_p), ("log_i_row_stride", ct.c_int64),
        ("log_f", ct.c_void_p), ("log_f_row_stride", ct.c_int64),
        ("h", ct.c_void_p), ("h_row_stride", ct.c_int64),
        ("o_pre", ct.c_void_p), ("o_row_stride", ct.c_int64),
        ("x_gate", ct.c_void_p), ("x_gate_row_stride", ct.c_int64),
        ("out", ct.c_void_p), ("out_row_stride", ct.c_int64),
    ]


class MlstmBwdArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("batch", ct.c_int32), ("heads", ct.c_int32), ("seqlen", ct.c_int32), ("dqk", ct.c_int32),
        ("chunk", ct.c_int32), ("gate_mode", ct.c_int32),
        ("io_dtype", ct.c_int),
        ("q", ct.c_void_p), ("q_stride", _i64x3),
        ("k", ct.c_void_p), ("k_stride", _i64x3),
        ("log_i", ct.c_void_p), ("i_stride", _i64x3),
        ("log_f", ct.c_void_p), ("f_stride", _i64x3),
        ("q_scaled", ct.c_void_p), ("k_scaled", ct.c_void_p),
        ("rho", ct.c_void_p), ("e_rho", ct.c_void_p), ("e_g", ct.c_void_p),
        ("q_decayed", ct.c_void_p), ("k_decayed", ct.c_void_p),
        ("split_planes", ct.c_void_p),
        ("dq_scaled", ct.c_void_p), ("dk_scaled", ct.c_void_p),
        ("chunk_dg", ct.c_void_p),
        ("dq", ct.c_void_p), ("dk", ct.c_void_p), ("dlog_i", ct.c_void_p), ("dlog_f", ct.c_void_p),
        ("d_i", ct.c_void_p),
    ]


class ChunkScanArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("groups", ct.c_int64),
        ("nchunks", ct.c_int32), ("rows", ct.c_int32), ("cols", ct.c_int32),
        ("x", ct.c_void_p), ("decay", ct.c_void_p),
        ("reverse", ct.c_int32),
        ("scale", ct.c_void_p), ("scaled", ct.c_void_p),
        ("scaled_hi", ct.c_void_p), ("scaled_lo", ct.c_void_p),
        ("skip_state", ct.c_int32),
        ("dot_hi", ct.c_void_p), ("dot_lo", ct.c_void_p),
        ("dot_scale", ct.c_void_p), ("dot_out", ct.c_void_p),
    ]


class SsdBwdIntraArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("batch", ct.c_int32), ("nchunks", ct.c_int32), ("heads", ct.c_int32), ("chunk", ct.c_int32),
        ("cb", ct.c_void_p), ("bcum", ct.c_void_p), ("dt", ct.c_void_p), ("dS", ct.c_void_p),
        ("S", ct.c_void_p), ("M", ct.c_void_p), ("ddt", ct.c_void_p), ("db", ct.c_void_p),
    ]


class SsdBwdRowsArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("batch", ct.c_int32), ("nchunks", ct.c_int32), ("chunk", ct.c_int32), ("heads", ct.c_int32),
        ("headdim", ct.c_int32), ("seqlen", ct.c_int32),
        ("xh", ct.c_void_p), ("dyh", ct.c_void_p), ("dxi", ct.c_void_p),
        ("BY", ct.c_void_p), ("CZ", ct.c_void_p), ("alpha", ct.c_void_p), ("D", ct.c_void_p),
        ("dx", ct.c_void_p), ("xby", ct.c_void_p), ("dycz", ct.c_void_p), ("dyx", ct.c_void_p),
    ]


class ChunkDotArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("groups", ct.c_int64),
        ("nchunks", ct.c_int32), ("rows", ct.c_int32), ("cols", ct.c_int32),
        ("adj", ct.c_void_p), ("state", ct.c_void_p), ("out", ct.c_void_p),
    ]


class MlstmBwdNormArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("batch", ct.c_int32), ("heads", ct.c_int32), ("seqlen", ct.c_int32), ("padded_len", ct.c_int32),
        ("dv", ct.c_int32), ("width", ct.c_int32),
        ("normalize", ct.c_int32),
        ("io_dtype", ct.c_int),
        ("outputs", ct.c_void_p),
        ("dh", ct.c_void_p), ("dh_stride", _i64x3),
        ("out", ct.c_void_p),
        ("out_hi", ct.c_void_p), ("out_lo", ct.c_void_p),
    ]


class ScaleSplitArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("batch", ct.c_int32), ("seqlen", ct.c_int32), ("padded_len", ct.c_int32), ("cols", ct.c_int32),
        ("group", ct.c_int32),
        ("io_dtype", ct.c_int),
        ("x", ct.c_void_p), ("x_stride", ct.c_int64 * 2),
        ("scale", ct.c_void_p),
        ("hi", ct.c_void_p), ("lo", ct.c_void_p),
    ]


class GemmOperand(ct.Structure):
    _fields_ = [
        ("ptr", ct.c_void_p),
        ("group_stride", ct.c_int64), ("row_stride", ct.c_int64),
        ("rows", ct.c_int32), ("cols", ct.c_int32),
        ("trans", ct.c_int32),
    ]


class ChunkGemmArgs(ct.Structure):
    _fields_ = [
        ("struct_size", ct.c_size_t),
        ("groups", ct.c_int64),
        ("m", ct.c_int32), ("n", ct.c_int32), ("nprod", ct.c_int32),
        ("a", GemmOperand * 4), ("b", GemmOperand * 4),
        ("alpha", ct.c_float),
        ("mask", ct.c_int32),
        ("decay", ct.c_void_p), ("decay_stride", ct.c_int64),
        ("accumulate", ct.c_int32),
        ("out", ct.c_void_p), ("out_group_stride", ct.c_int64), ("out_row_stride", ct.c_int64),
        ("out_bf16", ct.c_void_p), ("outb_group_stride", ct.c_int64), ("outb_row_stride", ct.c_int64),
        ("out_bf16_lo", ct.c_void_p),
        ("error_flag", ct.c_void_p),
        ("wait_limit_cycles", ct.c_int64),
    ]


# symbol -> (restype, argtypes)
SYMBOLS = {
    "hxm_abi_version": (ct.c_int, []),
    "hxm_last_error_string": (ct.c_char_p, []),
    "hxm_selective_scan_fwd": (ct.c_int, [ct.POINTER(ScanArgs), ct.c_void_p]),
    "hxm_selective_scan_workspace_size": (ct.c_size_t, [ct.POINTER(ScanArgs)]),
    "hxm_selective_scan_bwd_workspace_size": (ct.c_size_t, [ct.POINTER(ScanBwdArgs)]),
    "hxm_selective_scan_bwd": (ct.c_int, [ct.POINTER(ScanBwdArgs), ct.c_void_p]),
    "hxm_mlstm_workspace_size": (ct.c_size_t, [ct.POINTER(MlstmArgs)]),
    "hxm_mlstm_chunkwise_fwd": (ct.c_int, [ct.POINTER(MlstmArgs), ct.c_void_p]),
    "hxm_mlstm_chunkwise_fwd_noalloc": (ct.c_int, [ct.POINTER(MlstmArgs), ct.c_void_p]),
    "hxm_mlstm_bwd_prepare": (ct.c_int, [ct.POINTER(MlstmBwdArgs), ct.c_void_p]),
    "hxm_mlstm_bwd_finalize": (ct.c_int, [ct.POINTER(MlstmBwdArgs), ct.c_void_p]),
    "hxm_chunk_state_scan": (ct.c_int, [ct.POINTER(ChunkScanArgs), ct.c_void_p]),
    "hxm_mlstm_bwd_normalizer": (ct.c_int, [ct.POINTER(MlstmBwdNormArgs), ct.c_void_p]),
    "hxm_chunk_state_dot": (ct.c_int, [ct.POINTER(ChunkDotArgs), ct.c_void_p]),
    "hxm_chunk_gemm": (ct.c_int, [ct.POINTER(ChunkGemmArgs), ct.c_void_p]),
    "hxm_scale_split": (ct.c_int, [ct.POINTER(ScaleSplitArgs), ct.c_void_p]),
    "hxm_ssd_bwd_intra": (ct.c_int, [ct.POINTER(SsdBwdIntraArgs), ct.c_void_p]),
    "hxm_ssd_bwd_rows": (ct.c_int, [ct.POINTER(SsdBwdRowsArgs), ct.c_void_p]),
    "hxm_ssd_workspace_size": (ct.c_size_t, [ct.POINTER(SsdArgs)]),
    "hxm_ssd_chunk_scan_fwd": (ct.c_int, [ct.POINTER(SsdArgs), ct.c_void_p]),
    "hxm_slstm_scan_fwd": (ct.c_int, [ct.POINTER(SlstmArgs), ct.c_void_p]),
    "hxm_causal_conv1d_fwd": (ct.c_int, [ct.POINTER(ConvArgs), ct.c_void_p]),
    "hxm_rmsnorm_fwd": (ct.c_int, [ct.POINTER(RmsnormArgs), ct.c_void_p]),
    "hxm_mlstm_gate_prologue": (ct.c_int, [ct.POINTER(MlstmGatesArgs), ct.c_void_p]),
    "hxm_mlstm_gate_epilogue": (ct.c_int, [ct.POINTER(MlstmGatesArgs), ct.c_void_p]),
}

_lib = None
_lock = threading.Lock()


class HxmError(RuntimeError):
    """A non-OK hxm_status from the C ABI."""

    def __init__(self, fn, status, msg):
        super().__init__(f"{fn} returned {_STATUS.get(status, status)}: {msg}")
        self.status = status


def lib() -> ct.CDLL:
    """Load libhxm.so once (raises if it is missing: build it first)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(f"{LIB_PATH} not found: run `python -m hybrid_model_mamba_xlstm_b200.build`")
                l = ct.CDLL(LIB_PATH)
                for name, (res, args) in SYMBOLS.items():
                    f = getattr(l, name)
                    f.restype = res
                    f.argtypes = args
                _lib = l
    return _lib


def check(fn: str, status: int):
    if status != HXM_OK:
        msg = lib().hxm_last_error_string()
        raise HxmError(fn, status, msg.decode() if msg else "")


def call(fn: str, args, stream: int = 0):
    """Call an hxm entry point with an args struct on `stream` (raw cudaStream_t)."""
    args.struct_size = ct.sizeof(args)
    check(fn, getattr(lib(), fn)(ct.byref(args), ct.c_void_p(stream)))
