"""CPU oracle for the fused KL-GEMM distillation loss (test infrastructure only).

Nothing in the product path imports this package: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` use it,
and only as the expected results of parity checks or as the timed CPU baseline.
"""
