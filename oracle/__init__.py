"""Test infrastructure: CPU oracle for path-ordered geometric attention.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import this package, and only as the checker or the timed CPU
baseline.  The product (holonomyawareattention_b200) never imports it.
"""
