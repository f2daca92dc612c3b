"""Layer callers of the hot path (mirror of hybrid_xmamba.layers / .models)."""
from .blocks import HybridBlock, MambaBlock, RMSNorm, mLSTMBlock, sLSTMBlock
from .model import GraphDecoder, HybridConfig, HybridLanguageModel, PrefillGraph, hybrid_350m_config

__all__ = ["RMSNorm", "MambaBlock", "mLSTMBlock", "sLSTMBlock", "HybridBlock", "HybridConfig",
           "HybridLanguageModel", "GraphDecoder", "PrefillGraph", "hybrid_350m_config"]
