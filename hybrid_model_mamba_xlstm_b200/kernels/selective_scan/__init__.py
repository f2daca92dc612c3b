"""Selective scan (Mamba S6) — mirrors hybrid_xmamba/kernels/selective_scan/__init__.py."""
from .scan_interface import SelectiveScanFunction, selective_scan, selective_scan_fn

__all__ = ["selective_scan", "selective_scan_fn", "SelectiveScanFunction"]
