"""Chunkwise mLSTM ("TFLA") — mirrors hybrid_xmamba/kernels/tfla/__init__.py."""
from .tfla_bwd import mlstm_chunkwise_bwd
from .tfla_interface import TFLAFunction, apply_tfla, mlstm_chunkwise_fwd

__all__ = ["apply_tfla", "mlstm_chunkwise_fwd", "mlstm_chunkwise_bwd", "TFLAFunction"]
