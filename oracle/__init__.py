"""The oracle: CPU restatements of the reference's commitment hashing.

Test infrastructure only -- used by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py as the checker, never by the product path.
"""
