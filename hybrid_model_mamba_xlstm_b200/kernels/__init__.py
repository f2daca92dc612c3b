"""B200 kernels behind the reference's kernel entry points
(hybrid_xmamba/kernels/__init__.py:3-9): ``apply_tfla`` and ``selective_scan``,
plus the extended entries ``selective_scan_fn``, ``mlstm_chunkwise_fwd`` /
``mlstm_chunkwise_bwd``, ``ssd_chunk_scan`` / ``ssd_chunk_scan_fn`` (with its
backward), ``slstm_scan``, ``causal_conv1d`` and ``rmsnorm``."""
from .selective_scan.scan_interface import selective_scan, selective_scan_fn
from .tfla.tfla_interface import apply_tfla, mlstm_chunkwise_bwd, mlstm_chunkwise_fwd
from .ssd import ssd_chunk_scan, ssd_chunk_scan_bwd, ssd_chunk_scan_fn
from .slstm import slstm_scan
from .conv import causal_conv1d
from .norm import rmsnorm

__all__ = ["apply_tfla", "selective_scan", "selective_scan_fn", "mlstm_chunkwise_fwd", "mlstm_chunkwise_bwd",
           "ssd_chunk_scan", "ssd_chunk_scan_bwd", "ssd_chunk_scan_fn", "slstm_scan", "causal_conv1d", "rmsnorm"]
