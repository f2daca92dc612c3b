"""hybrid_model_mamba_xlstm_b200 — B200-native recurrent hot path of the hybrid
Mamba / xLSTM model (krishankb-de/hybrid_model_mamba_xlstm).

The kernels live in ``lib/libhxm.so`` (sm_100a, built from ``csrc/`` by
``python -m hybrid_model_mamba_xlstm_b200.build``) behind the C ABI in
``include/hxm.h``.  ``kernels`` mirrors the reference's
``hybrid_xmamba.kernels`` entry points; ``layers`` holds the reference's layer
callers (Mamba / mLSTM / sLSTM blocks, hybrid block, LM) wired to them;
``integration`` rebinds the names inside an installed reference package.
"""
__version__ = "0.1.0"
