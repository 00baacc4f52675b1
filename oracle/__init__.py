"""Test infrastructure: the reference-build recipe and the CPU oracle.

Nothing in the product imports this package. Only tests, the smoke check and
the CPU-baseline leg of bench.py use it, as the checker.
"""
