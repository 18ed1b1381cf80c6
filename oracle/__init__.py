"""CPU oracle for the FP8 quantized-linear path (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline / reference arm of
bench.py import this package, and only as the checker or the timed CPU
baseline.  The product library never links or calls it.
"""
