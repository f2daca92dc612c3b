"""Oracle: CPU restatement of the reference's recurrent hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm may import or execute anything in
this package, and only as the checker or the timed CPU baseline.  The product
path (``hybrid_model_mamba_xlstm_b200``) never imports it and has no CPU
fallback.

Contents
  ``numpy_ref``   float64 numpy restatements of the reference loops
                  (hybrid_xmamba/kernels/selective_scan/scan_interface.py,
                  hybrid_xmamba/kernels/tfla/tfla_interface.py,
                  hybrid_xmamba/layers/slstm_block.py) plus the final states
                  the reference keeps local.
  ``c/hxm_oracle.c``  the same loops in plain C (OpenMP over independent
                  channels / heads), fp32 like the reference's own arithmetic;
                  used as the timed CPU baseline and as a fast checker on
                  slices of large configurations.  Built by ``oracle/build.py``.

Pinning: every restatement is checked against golden vectors produced by
running the reference itself (``tests/golden/make_golden.py``, which imports
the reference package) — see ``tests/test_oracle_golden.py``.
"""
