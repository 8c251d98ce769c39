"""CPU oracle for the α-entmax block-sparse attention path.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker.  The splash_attention package
never imports it.
"""
